"""The C++ host side (host/gpu_bert_encoder.hpp through host/nebw_embed) on a
B200: file in, file out, against the CPU oracle, including the reference's
empty-row behaviour (mean pooling: zero vector; CLS pooling: refused)."""

import subprocess

import numpy as np
import pytest

from conftest import PKG, parity

pytestmark = pytest.mark.gpu

TOOL = PKG / "host" / "nebw_embed"


def _run(tmp_path, w, ids, mask, seq):
    from nebw.npue import write_bert_container
    write_bert_container(tmp_path / "m.npue", w, max_seq_len=seq)
    ids.astype("<i4").tofile(tmp_path / "ids.i32")
    mask.astype("<i4").tofile(tmp_path / "mask.i32")
    return subprocess.run([str(TOOL), str(tmp_path / "m.npue"), str(tmp_path / "ids.i32"),
                           str(tmp_path / "mask.i32"), str(seq), str(tmp_path / "out.f32")],
                          capture_output=True, text=True, timeout=300)


def test_cpp_tool_matches_oracle_with_empty_row(tmp_path, port_oracle):
    from nebw import synth
    w = synth.make_weights(synth.MINILM, seed=12, cls_pool=False, layers=2)
    lens = np.array([5, 0, 128, 33], np.int32)
    ids, mask = synth.make_tokens(4, 128, np.maximum(lens, 1), seed=13)
    mask[1] = 0
    r = _run(tmp_path, w, ids, mask, 128)
    assert r.returncode == 0, r.stderr
    got = np.fromfile(tmp_path / "out.f32", np.float32).reshape(4, w.hidden)
    want = port_oracle.encode(w, ids, mask)
    np.testing.assert_array_equal(got[1], np.zeros(w.hidden, np.float32))
    np.testing.assert_array_equal(want[1], np.zeros(w.hidden, np.float32))
    keep = [0, 2, 3]
    cos, err = parity(got[keep], want[keep])
    assert cos >= 0.9999 and err <= 2e-3, (cos, err)


def test_cpp_tool_refuses_empty_row_under_cls(tmp_path):
    from nebw import synth
    w = synth.make_weights(synth.MINILM, seed=14, cls_pool=True, layers=1)
    ids, mask = synth.make_tokens(2, 64, np.array([10, 1], np.int32), seed=15)
    mask[1] = 0
    r = _run(tmp_path, w, ids, mask, 64)
    assert r.returncode == 1 and "CLS pooling" in r.stderr, r.stderr


def test_cpp_tool_text_path(tmp_path, port_oracle):
    """`nebw_embed --text`: text lines -> the host WordPiece with the
    container's own vocabulary -> the GPU encoder; the same embeddings as the
    ids path on the tokenizer's output, and the oracle's within the gate."""
    import sys

    from conftest import REPO
    sys.path.insert(0, str(REPO / "tests" / "golden"))
    from make_pack_golden import synthetic_checkpoint
    from test_gpu_pack import _weights_from_container

    from nebw.pack import pack_bert
    d = tmp_path / "tiny-bert"
    synthetic_checkpoint(d)
    model = tmp_path / "m.npue"
    pack_bert(d, model, layout="tma_bf16", max_seq=64)
    texts = ["tok1 tok22 tok333, tok7!", "TOK5 tok6tok7 unknownword", "", "tok9 " * 80]
    (tmp_path / "t.txt").write_text("\n".join(texts) + "\n")
    r = subprocess.run([str(TOOL), "--text", str(model), str(tmp_path / "t.txt"), "64",
                        str(tmp_path / "out.f32")], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    got = np.fromfile(tmp_path / "out.f32", np.float32).reshape(len(texts), -1)
    r = subprocess.run([str(TOOL), "--tokenize", str(model), str(tmp_path / "t.txt"), "64",
                        str(tmp_path / "ids.i32"), str(tmp_path / "mask.i32")],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    ids = np.fromfile(tmp_path / "ids.i32", np.int32).reshape(len(texts), 64)
    mask = np.fromfile(tmp_path / "mask.i32", np.int32).reshape(len(texts), 64)
    assert ids[0, 0] == 2 and mask[3].sum() == 64  # [CLS] first; the long line is truncated
    r = subprocess.run([str(TOOL), str(model), str(tmp_path / "ids.i32"), str(tmp_path / "mask.i32"),
                        "64", str(tmp_path / "out2.f32")], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stderr
    np.testing.assert_array_equal(got, np.fromfile(tmp_path / "out2.f32", np.float32).reshape(got.shape))
    # the oracle on the host-layout container of the same checkpoint
    pack_bert(d, tmp_path / "host.npue", layout="host", max_seq=64)
    want = port_oracle.encode(_weights_from_container(tmp_path / "host.npue"), ids, mask)
    cos, err = parity(got, want)
    assert np.isfinite(got).all() and cos >= 0.9999 and err <= 2e-3, (cos, err)
