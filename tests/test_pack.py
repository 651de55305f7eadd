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
