"""The packer (nebw.pack) against the reference's own packer.

The golden (tests/golden/pack_tiny_bert.json, made by
tests/golden/make_pack_golden.py) is the reference packer's --dtype f32
container for a seeded synthetic BERT checkpoint: config, tensor order, and
per tensor dtype, role, shape and SHA-256 of the bytes.  nebw.pack's host
layout must reproduce it exactly; its tma_bf16 layout must hold the same
tensors with every GEMM operand as bf16 RNE of the transpose.
"""

import hashlib
import json
import sys

import numpy as np
import pytest

from conftest import REPO

GOLDEN = REPO / "tests" / "golden"
sys.path.insert(0, str(GOLDEN))


def _checkpoint(tmp_path):
    from make_pack_golden import synthetic_checkpoint
    d = tmp_path / "tiny-bert"
    synthetic_checkpoint(d)
    return d


def test_pack_host_matches_reference_packer(tmp_path):
    from make_pack_golden import MAX_SEQ, describe

    from nebw.pack import pack_bert
    d = _checkpoint(tmp_path)
    out = tmp_path / "host.npue"
    pack_bert(d, out, layout="host", max_seq=MAX_SEQ)
    got = describe(out)
    want = json.loads((GOLDEN / "pack_tiny_bert.json").read_text())
    assert got["order"] == want["order"]
    assert got["config"] == want["config"]
    for name, e in want["tensors"].items():
        assert got["tensors"][name] == e, name


def test_pack_tma_layout(tmp_path):
    from make_pack_golden import MAX_SEQ

    from nebw.npue import ContainerReader
    from nebw.pack import pack_bert, to_bf16_bits
    d = _checkpoint(tmp_path)
    pack_bert(d, tmp_path / "host.npue", layout="host", max_seq=MAX_SEQ)
    pack_bert(d, tmp_path / "tma.npue", layout="tma_bf16", max_seq=MAX_SEQ)
    with ContainerReader(tmp_path / "host.npue") as h, ContainerReader(tmp_path / "tma.npue") as t:
        assert t.config["gemm_layout"] == "tma_bf16" and t.config["a_dtype"] == "bf16"
        assert list(t.entries) == list(h.entries)
        for name, e in h.entries.items():
            if e["role"] == "gemm_b_host":
                te = t.entries[name]
                K, N = e["logical_shape"]
                assert te["dtype"] == "BF16" and te["role"] == "gemm_b_tma"
                assert te["logical_shape"] == [N, K]
                np.testing.assert_array_equal(t.tensor(name), to_bf16_bits(h.tensor(name).T))
            else:
                np.testing.assert_array_equal(t.tensor(name), h.tensor(name))


def _repack(src, dst, layout_of):
    """Copy a container entry by entry, with each entry's layout replaced by
    layout_of(name, entry) (None: no layout keys)."""
    from nebw.npue import ContainerReader, ContainerWriter
    with ContainerReader(src) as r:
        w = ContainerWriter(r.config, arch=r.arch, flags=r.flags)
        for name, e in r.entries.items():
            w.add(name, np.array(r.tensor(name)), e["dtype"], e["role"], e["logical_shape"],
                  layout=layout_of(name, e))
        w.write(dst)


def test_tma_operands_carry_the_library_layout_hash(tmp_path):
    from make_pack_golden import MAX_SEQ

    import nebw
    from nebw.npue import ContainerReader, layout_hash, tma_b_layout
    from nebw.pack import pack_bert
    d = _checkpoint(tmp_path)
    pack_bert(d, tmp_path / "tma.npue", layout="tma_bf16", max_seq=MAX_SEQ)
    lib_hash = nebw.lib().nebw_tma_layout_hash().decode()
    assert lib_hash == layout_hash(tma_b_layout())
    # the canonical text the hash is taken over, as the library states it
    assert layout_hash(tma_b_layout()) == hashlib.sha256(
        b'{"dtype":"BF16","kind":"dense","order":"n,k"}').hexdigest()
    with ContainerReader(tmp_path / "tma.npue") as t:
        n_gemm = 0
        for name, e in t.entries.items():
            if e["role"] == "gemm_b_tma":
                n_gemm += 1
                assert e["layout"] == tma_b_layout() and e["layout_hash"] == lib_hash, name
            else:
                assert "layout_hash" not in e, name
        assert n_gemm == 4 * t.config["num_layers"]


@pytest.mark.parametrize("case", ["foreign", "missing"])
def test_loader_refuses_a_mismatched_layout_without_a_gpu(tmp_path, case):
    """The reference refuses a design whose b_layout_hash differs from the
    model's (runtime/src/runtime.cpp:190-222); here one operand's descriptor
    differs, or the operands carry none.  The container is checked before any
    device use, so a null device reaches the refusal."""
    import ctypes as C

    from make_pack_golden import MAX_SEQ

    import nebw
    from nebw.npue import tma_b_layout
    from nebw.pack import pack_bert
    d = _checkpoint(tmp_path)
    good = tmp_path / "tma.npue"
    pack_bert(d, good, layout="tma_bf16", max_seq=MAX_SEQ)
    panel = {"kind": "block_panel", "tile_k": 64, "tile_n": 64, "order": "k,n,kt,nt",
             "inner": "s,t", "mac_s": 8, "mac_t": 8, "dtype": "BF16"}

    def layout_of(name, e):
        if e["role"] != "gemm_b_tma" or case == "missing":
            return None
        return panel if name == "layer.1.ffn_up" else tma_b_layout()

    bad = tmp_path / "bad.npue"
    _repack(good, bad, layout_of)
    lib = nebw.lib()
    h = C.c_void_p()
    assert lib.nebw_model_load_npue(None, str(bad).encode(), C.byref(h)) == 1  # NEBW_EINVAL
    msg = lib.nebw_last_error().decode()
    assert "layout_hash" in msg and ("layer.1.ffn_up" if case == "foreign" else "layer.0.qkv") in msg
    assert ("(none)" in msg) == (case == "missing")
    assert not h.value
    # the unaltered container passes the check and stops only at the device
    assert lib.nebw_model_load_npue(None, str(good).encode(), C.byref(h)) != 0
    assert "layout_hash" not in lib.nebw_last_error().decode()


def test_read_safetensors_widens_exactly(tmp_path):
    from nebw.pack import read_safetensors
    x = np.random.default_rng(1).standard_normal((3, 5)).astype(np.float32)
    bits = (x.view(np.uint32) >> 16).astype(np.uint16)
    hdr = json.dumps({"a": {"dtype": "F16", "shape": [3, 5], "data_offsets": [0, 30]},
                      "b": {"dtype": "BF16", "shape": [3, 5], "data_offsets": [30, 60]}}).encode()
    (tmp_path / "t.safetensors").write_bytes(len(hdr).to_bytes(8, "little") + hdr +
                                             x.astype(np.float16).tobytes() + bits.tobytes())
    got = read_safetensors(tmp_path / "t.safetensors")
    np.testing.assert_array_equal(got["a"], x.astype(np.float16).astype(np.float32))
    np.testing.assert_array_equal(got["b"], (bits.astype(np.uint32) << 16).view(np.float32))


def test_pack_refuses_other_models(tmp_path):
    from nebw.pack import pack_bert
    d = _checkpoint(tmp_path)
    cfg = json.loads((d / "config.json").read_text())
    cfg["model_type"] = "vit"
    (d / "config.json").write_text(json.dumps(cfg))
    with pytest.raises(SystemExit, match="model_type"):
        pack_bert(d, tmp_path / "x.npue")
