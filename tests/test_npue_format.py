"""The `.npue` container (CPU, no GPU): this repository's writer against the
reference's own writer (tools/lib/npue.py, imported read-only from the
reference tree where it exists), and the reader's refusals."""

import importlib.util
import struct

import numpy as np
import pytest

from conftest import REFERENCE, has_reference


def _ref_npue():
    spec = importlib.util.spec_from_file_location("ref_npue", REFERENCE / "tools" / "lib" / "npue.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.mark.skipif(not has_reference(), reason="reference tree not present")
def test_writer_byte_identical_to_reference_writer(tmp_path):
    from nebw.npue import ContainerWriter
    ref = _ref_npue()
    rng = np.random.default_rng(0)
    tensors = [("a", rng.standard_normal((3, 5)).astype(np.float32), "F32", "embedding", [3, 5]),
               ("b", rng.integers(0, 9, size=7).astype(np.int32), "I32", "ids", [7]),
               ("c", rng.standard_normal(4100).astype(np.float32), "F32", "bias", [4100])]
    cfg = {"arch": "bert_abs_gelu_postln", "num_layers": 1, "hidden": 8}
    mine, theirs = ContainerWriter(cfg), ref.Writer(cfg)
    for name, arr, dt, role, shape in tensors:
        mine.add(name, arr, dt, role, shape)
        theirs.add(name, arr, dt, role, shape)
    mine.write(tmp_path / "mine.npue")
    theirs.write(tmp_path / "theirs.npue")
    assert (tmp_path / "mine.npue").read_bytes() == (tmp_path / "theirs.npue").read_bytes()


@pytest.mark.skipif(not has_reference(), reason="reference tree not present")
def test_reference_reader_reads_bert_container(tmp_path):
    from nebw import synth
    from nebw.npue import write_bert_container
    ref = _ref_npue()
    w = synth.make_weights(synth.MINILM, seed=1, cls_pool=False, layers=1, vocab=64)
    write_bert_container(tmp_path / "m.npue", w, max_seq_len=32)
    r = ref.Reader(tmp_path / "m.npue")
    assert r.config["gemm_layout"] == "host" and r.config["max_seq_len"] == 32
    np.testing.assert_array_equal(np.asarray(r.raw("layer.0.qkv")).reshape(384, 1152),
                                  w.w_qkv[0])
    r.close()


def test_reader_roundtrip_and_refusals(tmp_path):
    from nebw import synth
    from nebw.npue import ContainerReader, write_bert_container
    w = synth.make_weights(synth.MINILM, seed=2, cls_pool=True, layers=2, vocab=100)
    p = tmp_path / "m.npue"
    write_bert_container(p, w, max_seq_len=16)
    with ContainerReader(p) as r:
        assert r.config["pooling"] == "cls"
        np.testing.assert_array_equal(r.tensor("layer.1.ffn_down"), w.w_dn[1])
        np.testing.assert_array_equal(r.tensor("embeddings.position"), w.pos[:16])
        assert r.data_offset % 4096 == 0
        for e in r.entries.values():
            assert e["offset"] % 4096 == 0
    bad = bytearray(p.read_bytes())
    bad[:4] = b"XXXX"
    (tmp_path / "bad.npue").write_bytes(bytes(bad))
    with pytest.raises(ValueError, match="not a .npue"):
        ContainerReader(tmp_path / "bad.npue")
    bad = bytearray(p.read_bytes())
    bad[4:8] = struct.pack("<I", 2)
    (tmp_path / "v2.npue").write_bytes(bytes(bad))
    with pytest.raises(ValueError, match="version"):
        ContainerReader(tmp_path / "v2.npue")


@pytest.mark.parametrize("key,arch,act", [("nomic-base", "nomic_bert_rope_swiglu", "silu"),
                                          ("gte-base", "gte_new_rope_geglu", "gelu")])
def test_gated_rotary_container_keys(tmp_path, key, arch, act):
    """The gated / rotary containers carry the keys the reference's
    set_model_shape reads (app_state.hpp:440-560): arch, rope position
    encoding, gated_ffn, the FFN-up halves' order, the gate activation, and
    theta (nomic) or the frequency list as a JSON string (gte); ffn_up is
    [hidden, 2 * intermediate]."""
    import json
    from nebw import synth
    from nebw.npue import ContainerReader, write_bert_container
    w = synth.config_weights(synth.CONFIGS[key], layers=1)
    path = tmp_path / "g.npue"
    write_bert_container(path, w, max_seq_len=64)
    with ContainerReader(path) as r:
        c = r.config
        assert c["arch"] == arch and c["position_embedding_type"] == "rope"
        assert c["gated_ffn"] is True and c["activation"] == act
        assert r.entries["layer.0.ffn_up"]["logical_shape"] == [w.hidden, 2 * w.ffn]
        assert r.entries["layer.0.ffn_up.bias"]["logical_shape"] == [2 * w.ffn]
        if key == "nomic-base":
            assert c["swiglu_halves"] == "fc11_up|fc12_gate" and c["rope_theta"] == 1000.0
            assert not np.any(r.tensor("layer.0.qkv.bias"))  # nomic has no biases
        else:
            assert c["glu_halves"].startswith("up_first|gate_second")
            freq = json.loads(c["rope_inv_freq"])
            assert len(freq) == w.head_dim // 2
            np.testing.assert_array_equal(np.float32(freq), np.float32(w.rope_inv_freq))
        assert not np.any(r.tensor("embeddings.position"))  # the zero placeholder
