"""Golden token ids from the reference's own WordPiece for the tokenizer test.

    python tests/golden/make_tokenizer_golden.py     (needs oracle/_ref built)

1. A seeded synthetic corpus (tokenizer_synth.npz: `texts`, UTF-8 bytes per
   line) that exercises every step of the BERT basic tokenizer: ASCII words
   in mixed case, digits and punctuation, accented Latin, Greek sigmas,
   Cyrillic, Han ideographs (split per character), Hiragana, Katakana and
   Hangul (not split), emoji, combining marks, control and format
   characters, no-break and ideographic spaces, tabs, the special tokens
   written in the text, words over 100 characters, and bytes that are not
   UTF-8.
2. A synthetic vocabulary (`vocab`) built from that corpus: the special
   tokens, every folded character alone and as a "##" continuation, and
   seeded 2-4 character chunks of the folded words, so that greedy
   longest-match, continuations and [UNK] all occur.
3. The reference's WordPiece (runtime/src/tokenizers/wordpiece.cpp, compiled
   into oracle/_ref, nebw_ref_wordpiece) encodes every line at max_len 64:
   `ids`, `mask`.

tests/test_tokenizer.py runs the host tools' tokenizer (host/wordpiece.cpp)
over the same texts and vocabulary and compares bit for bit.
"""

from __future__ import annotations

import ctypes as C
import sys
import tempfile
import unicodedata
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
MAX_LEN = 64
SEED = 20261202

ALPHABETS = {
    "ascii": "abcdefghijklmnopqrstuvwxyzABCDEFGHIJKLMNOPQRSTUVWXYZ",
    "digits": "0123456789",
    "punct": "!\"#$%&'()*+,-./:;<=>?@[\\]^_`{|}~",
    "latin": "éèêëÉÈàáâäÀÁÂÄöóòÖñÑçÇßøØåÅæÆœŒıİ",
    "greek": "αβγδεζηθικλμνξοπρσςτυφχψωΑΒΓΔΣΩΆΈΉΊΌΎΏ",
    "cyrillic": "абвгдеёжзийклмнопрстуфхцчшщъыьэюяАБВГДЁЖЗИЙ",
    "han": "漢字中文日本語言語計算機學習深度神經網絡",
    "kana": "ひらがなカタカナテストです",
    "hangul": "한국어텍스트토큰화",
    "emoji": "🙂🚀🎉👍",
    "other_punct": "¿¡«»—–…“”‘’·、。「」",
}
SPECIAL_CHARS = ["́", "̈", "​", " ", "　", "\t", "\x07", "­",
                 "﻿"]


def synth_corpus(n_lines=240):
    rng = np.random.default_rng(SEED)
    keys = list(ALPHABETS)
    lines = []
    for i in range(n_lines):
        words = []
        for _ in range(int(rng.integers(1, 14))):
            k = keys[int(rng.integers(len(keys)))]
            a = ALPHABETS[k]
            n = int(rng.integers(1, 9))
            w = "".join(a[int(rng.integers(len(a)))] for _ in range(n))
            if rng.random() < 0.15:
                w += SPECIAL_CHARS[int(rng.integers(len(SPECIAL_CHARS)))]
            if rng.random() < 0.05:
                w = "[CLS]" if rng.random() < 0.5 else "[MASK]"
            words.append(w)
        sep = " " if rng.random() < 0.8 else "\t"
        line = sep.join(words)
        if i % 37 == 5:
            line += " " + "x" * 120                      # a word over 100 characters
        b = line.encode("utf-8")
        if i % 41 == 7:
            b += b" \xff\xfe broken"                      # bytes that are not UTF-8
        lines.append(b)
    return lines


def fold(text):
    s = unicodedata.normalize("NFD", text.lower())
    return "".join(c for c in s if unicodedata.category(c) != "Mn")


def synth_vocab(lines):
    rng = np.random.default_rng(SEED + 1)
    chars, chunks = set(), set()
    for b in lines:
        t = fold(b.decode("utf-8", "replace"))
        for w in t.split():
            chars.update(w)
            if len(w) >= 2:
                for _ in range(2):
                    a = int(rng.integers(0, len(w)))
                    n = int(rng.integers(2, 5))
                    chunks.add(w[a:a + n])
    vocab = ["[PAD]", "[UNK]", "[CLS]", "[SEP]", "[MASK]"]
    for c in sorted(chars):
        if c.strip():
            vocab += [c, "##" + c]
    for ch in sorted(chunks):
        if ch.strip() and " " not in ch:
            vocab.append(ch if rng.random() < 0.5 else "##" + ch)
    # drop one ASCII letter's continuation so some pieces have no match ([UNK])
    vocab = [v for v in vocab if v != "##q"]
    seen, out = set(), []
    for v in vocab:
        if v not in seen:
            seen.add(v)
            out.append(v)
    return out


def main():
    lib = C.CDLL(str(REPO / "oracle" / "_ref" / "libnebw_ref.so"))
    fn = lib.nebw_ref_wordpiece
    i32p = C.POINTER(C.c_int32)
    fn.argtypes = [C.c_char_p, C.c_char_p, C.c_int32, i32p, i32p, C.c_char_p, C.c_int32]
    fn.restype = C.c_int
    lines = synth_corpus()
    vocab = synth_vocab(lines)
    with tempfile.TemporaryDirectory() as td:
        vpath = Path(td) / "vocab.txt"
        vpath.write_text("\n".join(vocab) + "\n", encoding="utf-8")
        ids = np.zeros((len(lines), MAX_LEN), np.int32)
        mask = np.zeros((len(lines), MAX_LEN), np.int32)
        err = C.create_string_buffer(1024)
        for i, b in enumerate(lines):
            if fn(str(vpath).encode(), b, MAX_LEN, ids[i].ctypes.data_as(i32p),
                  mask[i].ctypes.data_as(i32p), err, 1024):
                raise RuntimeError(err.value.decode())
    texts = np.array(lines, dtype=object)
    np.savez_compressed(HERE / "tokenizer_synth.npz", texts=np.array([t for t in texts], dtype="S"),
                        vocab=np.frombuffer(("\n".join(vocab) + "\n").encode("utf-8"), np.uint8),
                        ids=ids, mask=mask, max_len=np.int32(MAX_LEN),
                        provenance="reference WordPiece (runtime/src/tokenizers/wordpiece.cpp) "
                                   "via oracle/_ref nebw_ref_wordpiece, seed %d" % SEED)
    unk = int((ids == 1).sum())
    print(f"tokenizer_synth.npz: {len(lines)} lines, vocab {len(vocab)}, {unk} [UNK], "
          f"{int(mask.sum())} real positions")


if __name__ == "__main__":
    sys.exit(main())
