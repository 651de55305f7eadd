"""The host tools' WordPiece tokenizer (host/wordpiece.cpp, used by
`nebw_embed --text`) against the reference's own tokenizer
(runtime/src/tokenizers/wordpiece.cpp): token ids and masks bit for bit.

  * a seeded multilingual synthetic corpus with a synthetic vocabulary, whose
    ids the reference's compiled tokenizer produced
    (tests/golden/make_tokenizer_golden.py) -- always;
  * the reference's own golden token ids for its corpus sentences with the
    real checkpoint vocabularies (reference/goldens/*_s64_boundary.npz) --
    only where the reference tree is present.
"""

import subprocess
import sys

import numpy as np
import pytest

from conftest import PKG, REFERENCE, REPO

TOOL = PKG / "host" / "nebw_embed"


def run_tokenizer(tmp_path, vocab_bytes, lines, max_len):
    v = tmp_path / "vocab.txt"
    v.write_bytes(vocab_bytes)
    t = tmp_path / "texts.txt"
    t.write_bytes(b"\n".join(lines) + b"\n")
    ids, mask = tmp_path / "ids.i32", tmp_path / "mask.i32"
    r = subprocess.run([str(TOOL), "--tokenize", str(v), str(t), str(max_len), str(ids), str(mask)],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return (np.fromfile(ids, np.int32).reshape(-1, max_len),
            np.fromfile(mask, np.int32).reshape(-1, max_len))


def test_tokenizer_matches_reference_on_synthetic_corpus(tmp_path):
    g = dict(np.load(REPO / "tests" / "golden" / "tokenizer_synth.npz"))
    lines = [bytes(x) for x in g["texts"]]
    ids, mask = run_tokenizer(tmp_path, g["vocab"].tobytes(), lines, int(g["max_len"]))
    bad = np.nonzero((ids != g["ids"]).any(1))[0]
    assert not len(bad), f"{len(bad)} lines differ, first {lines[bad[0]]!r}: " \
                         f"{ids[bad[0]][:20]} vs {g['ids'][bad[0]][:20]}"
    np.testing.assert_array_equal(mask, g["mask"])


@pytest.mark.skipif(not (REFERENCE / "reference" / "goldens").exists(),
                    reason="the reference tree (its goldens and vocabularies) is not here")
@pytest.mark.parametrize("golden,model", [
    ("minilm_l6_s64_boundary.npz", "all-MiniLM-L6-v2"),
    ("bge-small-en-v1.5_l12_s64_boundary.npz", "bge-small-en-v1.5"),
    ("bge-base-en-v1.5_l12_s64_boundary.npz", "bge-base-en-v1.5")])
def test_tokenizer_matches_reference_goldens(tmp_path, golden, model):
    sys.path.insert(0, str(REFERENCE / "reference"))
    from corpus import SENTENCES
    g = np.load(REFERENCE / "reference" / "goldens" / golden)
    vocab = (REFERENCE / "models" / model / "vocab.txt").read_bytes()
    ids, mask = run_tokenizer(tmp_path, vocab, [s.encode("utf-8") for s in SENTENCES],
                              g["input_ids"].shape[1])
    np.testing.assert_array_equal(ids, g["input_ids"])
    np.testing.assert_array_equal(mask, g["attention_mask"])
