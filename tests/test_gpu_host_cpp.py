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
