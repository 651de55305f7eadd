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


# ---- the C++ packer in the library (nebw_pack_checkpoint) ----

@pytest.mark.parametrize("layout", ["host", "tma_bf16"])
@pytest.mark.parametrize("fold", [True, False])
def test_cpp_packer_is_byte_identical(tmp_path, layout, fold):
    """nebw_pack_checkpoint (C++, host only) writes the very bytes nebw.pack
    writes -- header, JSON directory (config keys and number formatting,
    source SHA-256, layout hash) and every tensor; the host layout is thereby
    pinned to the reference packer's golden through the test above."""
    from make_pack_golden import MAX_SEQ, describe

    import nebw
    from nebw.pack import pack_bert
    d = _checkpoint(tmp_path)
    pack_bert(d, tmp_path / "py.npue", layout=layout, max_seq=MAX_SEQ, fold_scale=fold)
    n = nebw.pack_checkpoint(d, tmp_path / "cc.npue", layout, MAX_SEQ, fold)
    want = (tmp_path / "py.npue").read_bytes()
    assert n == len(want)
    assert (tmp_path / "cc.npue").read_bytes() == want
    if layout == "host" and fold:
        golden = json.loads((GOLDEN / "pack_tiny_bert.json").read_text())
        got = describe(tmp_path / "cc.npue")
        assert got["config"] == golden["config"] and got["order"] == golden["order"]


def test_cpp_packer_reads_bf16_and_f16_checkpoints(tmp_path):
    """A checkpoint stored as BF16 / F16 safetensors (widened exactly) packs
    to the same bytes in C++ and Python, prefixed tensor names included."""
    import nebw
    from nebw.pack import pack_bert, read_safetensors
    d = _checkpoint(tmp_path)
    src = read_safetensors(d / "model.safetensors")
    hdr, blobs, off = {}, [], 0
    for i, (name, a) in enumerate(sorted(src.items())):
        if i % 2:
            b = (a.astype(np.float32).view(np.uint32) >> 16).astype(np.uint16).tobytes()
            dt = "BF16"
        else:
            b = a.astype(np.float16).tobytes()
            dt = "F16"
        hdr["bert." + name] = {"dtype": dt, "shape": list(a.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    h = json.dumps(hdr).encode()
    (d / "model.safetensors").write_bytes(len(h).to_bytes(8, "little") + h + b"".join(blobs))
    pack_bert(d, tmp_path / "py.npue", layout="tma_bf16", max_seq=32)
    nebw.pack_checkpoint(d, tmp_path / "cc.npue", "tma_bf16", 32, True)
    assert (tmp_path / "cc.npue").read_bytes() == (tmp_path / "py.npue").read_bytes()


def test_cpp_packer_refusals(tmp_path):
    import nebw
    d = _checkpoint(tmp_path)
    with pytest.raises(nebw.NebwError, match="layout"):
        nebw.pack_checkpoint(d, tmp_path / "x.npue", "panels", 32, True)
    cfg = json.loads((d / "config.json").read_text())
    cfg["model_type"] = "vit"
    (d / "config.json").write_text(json.dumps(cfg))
    with pytest.raises(nebw.NebwError, match="model_type"):
        nebw.pack_checkpoint(d, tmp_path / "x.npue", "host", 32, True)
    cfg["model_type"] = "bert"
    (d / "config.json").write_text(json.dumps(cfg))
    (d / "1_Pooling" / "config.json").write_text(json.dumps({"pooling_mode_max_tokens": True}))
    with pytest.raises(nebw.NebwError, match="pooling"):
        nebw.pack_checkpoint(d, tmp_path / "x.npue", "host", 32, True)
    with pytest.raises(nebw.NebwError, match="config.json"):
        nebw.pack_checkpoint(tmp_path, tmp_path / "x.npue", "host", 32, True)
    (d / "model.safetensors").unlink()
    (d / "1_Pooling" / "config.json").write_text(json.dumps({"pooling_mode_cls_token": True}))
    with pytest.raises(nebw.NebwError, match="safetensors"):
        nebw.pack_checkpoint(d, tmp_path / "x.npue", "host", 32, True)


# ---- the reference's pre-tiled containers (block panels, bf16 / int8) ----

def test_block_panel_order_and_round_trip():
    """untile_block_panel against the axis order written out element by
    element: flat index over (kb, nb, ri, ci, si, ti), ti fastest, k = kb*tk
    + ri*s + si, n = nb*tn + ci*t + ti."""
    from nebw.npue import block_panel_layout, tile_block_panel, untile_block_panel
    K, N = 32, 48
    lay = block_panel_layout(16, 24, 4, 8, "I8")
    flat = np.arange(K * N, dtype=np.int32)
    want = np.empty((K, N), np.int32)
    f = 0
    for kb in range(K // 16):
        for nb in range(N // 24):
            for ri in range(16 // 4):
                for ci in range(24 // 8):
                    for si in range(4):
                        for ti in range(8):
                            want[kb * 16 + ri * 4 + si, nb * 24 + ci * 8 + ti] = flat[f]
                            f += 1
    np.testing.assert_array_equal(untile_block_panel(flat, K, N, lay), want)
    np.testing.assert_array_equal(tile_block_panel(want, lay), flat)
    with pytest.raises(ValueError, match="does not tile"):
        untile_block_panel(flat, K, N, block_panel_layout(16, 20, 4, 8, "I8"))


def _gemm_kn(lib, path, name, K, N):
    out = np.zeros((K, N), np.float32)
    rc = lib.nebw_npue_gemm_kn(str(path).encode(), name.encode(), out.ctypes.data, K, N)
    return rc, out


def _assert_reader_matches_reference(path, ref_oracle):
    import ctypes as C

    import nebw
    from nebw.npue import ContainerReader
    lib = nebw.lib()
    f = ref_oracle.lib.nebw_ref_host_b_kn
    f.argtypes = [C.c_char_p, C.c_char_p, C.c_void_p, C.c_int64, C.c_int64]
    n = 0
    with ContainerReader(path) as r:
        ops = [(k, e["logical_shape"]) for k, e in r.entries.items() if e["role"] == "gemm_b"]
    for name, (K, N) in ops:
        rc, mine = _gemm_kn(lib, path, name, K, N)
        assert rc == 0, lib.nebw_last_error().decode()
        theirs = np.zeros((K, N), np.float32)
        assert f(str(path).encode(), name.encode(), theirs.ctypes.data, K, N) == 0
        np.testing.assert_array_equal(mine.view(np.uint32), theirs.view(np.uint32), err_msg=name)
        n += 1
    assert n > 0


@pytest.mark.parametrize("a_dtype", ["bf16", "i8"])
def test_pretiled_reader_bit_exact_vs_reference_on_our_containers(tmp_path, ref_oracle, a_dtype):
    """nebw_npue_gemm_kn (the library's reader) against the reference's
    host_b_kn, compiled from its tree, on containers nebw.npue writes."""
    from nebw import synth
    from nebw.npue import write_bert_container
    w = synth.config_weights(synth.CONFIGS["minilm"], layers=2)
    path = tmp_path / f"{a_dtype}.npue"
    write_bert_container(path, w, max_seq_len=64, gemm_layout="pretiled_bf16", a_dtype=a_dtype,
                         tile=(64, 48), smooth_seed=1)
    _assert_reader_matches_reference(path, ref_oracle)


@pytest.mark.parametrize("dtype,extra", [("bf16", ("--tile-n", "32")), ("i8", ("--tile-n", "32"))])
def test_pretiled_reader_bit_exact_on_reference_packed_containers(tmp_path, ref_oracle, dtype,
                                                                  extra):
    """Containers made by the reference's own packer (--dtype bf16, and --dtype
    i8 with its SmoothQuant calibration) read bit-identically by the library
    and by the reference's host_b_kn."""
    from conftest import has_reference
    if not has_reference():
        pytest.skip("the reference tree is not here")
    from make_pack_golden import reference_pack
    path = reference_pack(tmp_path, dtype, extra)
    from nebw.npue import ContainerReader
    with ContainerReader(path) as r:
        assert r.config["gemm_layout"] == "pretiled_bf16" and r.config["a_dtype"] == dtype
    _assert_reader_matches_reference(path, ref_oracle)


def test_pretiled_golden_containers_regenerate():
    """The containers behind tests/golden/pretiled_*.npz come back byte for
    byte from nebw.npue, so the GPU test reads what the reference read."""
    import make_golden
    cases = [(n, make_golden.write_pretiled, k, a) for n, (k, a) in make_golden.PRETILED.items()]
    cases += [(n, make_golden.write_vit_pretiled, k, a)
              for n, (k, a) in make_golden.VIT_PRETILED.items()]
    for name, write, key, a_dtype in cases:
        g = np.load(GOLDEN / f"{name}.npz")
        with __import__("tempfile").TemporaryDirectory(dir=GOLDEN) as td:
            digest = write(f"{td}/c.npue", key, a_dtype)
        assert digest == str(g["container_sha256"]), name


def test_gemm_kn_refusals(tmp_path):
    """The reader refuses, by name, what it cannot read: an axis order it does
    not define, tiles that do not divide the operand, an int8 operand without
    its .wscale."""
    import nebw
    from nebw.npue import ContainerWriter, block_panel_layout, tile_block_panel
    lib = nebw.lib()
    K, N = 64, 64
    q = np.arange(K * N, dtype=np.int64).reshape(K, N).astype(np.int8)

    def one(layout, with_ws=True):
        w = ContainerWriter({"arch": "bert_abs_gelu_postln"})
        w.add("layer.0.qkv", tile_block_panel(q, block_panel_layout(32, 32, 8, 8, "I8")), "I8",
              "gemm_b", [K, N], layout=layout)
        if with_ws:
            w.add("layer.0.qkv.wscale", np.ones(N, np.float32), "F32", "quant_scale", [N])
        path = tmp_path / "c.npue"
        w.write(path)
        rc, _ = _gemm_kn(lib, path, "layer.0.qkv", K, N)
        return rc, lib.nebw_last_error().decode()

    good = block_panel_layout(32, 32, 8, 8, "I8")
    assert one(good)[0] == 0
    rc, msg = one(dict(good, order="n,k,nt,kt"))
    assert rc != 0 and "refused" in msg
    rc, msg = one(dict(good, tile_n=48))
    assert rc != 0 and "does not tile" in msg
    rc, msg = one(good, with_ws=False)
    assert rc != 0 and ".wscale" in msg


def test_loader_refuses_int4_containers_without_a_gpu(tmp_path):
    import ctypes as C

    import nebw
    from nebw import synth
    from nebw.npue import write_bert_container
    w = synth.config_weights(synth.CONFIGS["minilm"], layers=1)
    path = tmp_path / "i4.npue"
    write_bert_container(path, w, max_seq_len=64, gemm_layout="pretiled_bf16", a_dtype="i8",
                         config_overrides={"a_dtype": "i4"})
    h = C.c_void_p()
    assert nebw.lib().nebw_model_load_npue(None, str(path).encode(), C.byref(h)) == 1
    assert "a_dtype 'i4'" in nebw.lib().nebw_last_error().decode()


def test_vit_loader_refuses_int4_containers_without_a_gpu(tmp_path):
    import ctypes as C

    import nebw
    from nebw import synth
    from nebw.npue import write_vit_container
    w = synth.vit_config_weights(synth.VIT_CONFIGS["vit-base"], layers=1)
    path = tmp_path / "v.npue"
    write_vit_container(path, w, gemm_layout="pretiled_bf16", a_dtype="bf16")
    raw = path.read_bytes().replace(b'"a_dtype":"BF16"', b'"a_dtype":"I4__"', 1)
    path.write_bytes(raw)
    h = C.c_void_p()
    assert nebw.lib().nebw_vit_load_npue(None, str(path).encode(), C.byref(h)) == 1
    assert "a_dtype 'i4__'" in nebw.lib().nebw_last_error().decode()
