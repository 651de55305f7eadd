"""The C++ host side (host/gpu_bert_encoder.hpp through host/nebw_embed) on a
B200: file in, file out, against the CPU oracle, including the reference's
empty-row behaviour (mean pooling: zero vector; CLS pooling: refused); and
the serving drop-in (host/npue_gpu_encoder.hpp) compiled against the
reference's own headers and tokenizer (oracle/_ref/npue_encoder_check)."""

import subprocess

import numpy as np
import pytest

from conftest import PKG, REPO, parity

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


CHECK = REPO / "oracle" / "_ref" / "npue_encoder_check"


def synthetic_vocab(n: int) -> bytes:
    """A WordPiece vocabulary of n entries: the specials, whole words w0..,
    and '##' continuations of single digits."""
    words = ["[PAD]", "[UNK]", "[CLS]", "[SEP]", "[MASK]"] + [f"##{d}" for d in range(10)]
    words += [f"w{i}" for i in range(n - len(words))]
    return ("\n".join(words) + "\n").encode()


def synthetic_texts(n: int, seed: int, max_words: int) -> list:
    rng = np.random.default_rng(seed)
    out = []
    for i in range(n):
        k = int(rng.integers(1, max_words + 1))
        ws = [f"w{int(x)}" for x in rng.integers(0, 30000, k)]
        if i % 7 == 0:
            ws.append(f"W{int(rng.integers(0, 99))}99999!")  # case fold, "##" digits, punctuation
        out.append(" ".join(ws))
    return out


@pytest.mark.skipif(not CHECK.exists(),
                    reason="built only where the reference tree is (oracle/Makefile encoder_check)")
def test_npue_encoder_adapter_through_reference_interface(tmp_path, port_oracle):
    """nebw::GpuNpueEncoder as the reference's npue::Encoder, with the
    reference's own tokenizer (app::load_tokenizer on the container): texts
    -> embeddings, against the CPU oracle on the very ids and mask that
    tokenizer produced; those ids equal this repo's WordPiece's."""
    from nebw import synth
    from nebw.npue import write_bert_container
    w = synth.make_weights(synth.BGE_SMALL, seed=71, cls_pool=True, layers=2)
    vocab = synthetic_vocab(w.vocab)
    model = tmp_path / "m.npue"
    write_bert_container(model, w, max_seq_len=128, vocab=vocab)
    texts = synthetic_texts(24, 72, 140) + ["", "W1 w2, w3."]
    (tmp_path / "t.txt").write_text("\n".join(texts) + "\n")
    r = subprocess.run([str(CHECK), str(model), str(tmp_path / "t.txt"), "128",
                        str(tmp_path / "out.f32"), str(tmp_path / "ids.i32"),
                        str(tmp_path / "mask.i32")], capture_output=True, text=True, timeout=300)
    # a text longer than 128 tokens is refused, as the runtime refuses it
    assert r.returncode == 1 and "tokens; the limit is 128" in r.stderr, r.stdout + r.stderr
    texts = synthetic_texts(24, 72, 90) + ["", "W1 w2, w3."]
    (tmp_path / "t.txt").write_text("\n".join(texts) + "\n")
    r = subprocess.run([str(CHECK), str(model), str(tmp_path / "t.txt"), "128",
                        str(tmp_path / "out.f32"), str(tmp_path / "ids.i32"),
                        str(tmp_path / "mask.i32")], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    n = len(texts)
    got = np.fromfile(tmp_path / "out.f32", np.float32).reshape(n, w.hidden)
    ids = np.fromfile(tmp_path / "ids.i32", np.int32).reshape(n, 128)
    mask = np.fromfile(tmp_path / "mask.i32", np.int32).reshape(n, 128)
    assert (ids[:, 0] == 2).all() and int(r.stdout.split()[3]) == int(mask.sum())
    want = port_oracle.encode(w, ids, mask)
    cos, err = parity(got, want)
    assert np.isfinite(got).all() and cos >= 0.9999 and err <= 2e-3, (cos, err)
    # this repo's tokenizer gives the same ids and mask
    (tmp_path / "v.txt").write_bytes(vocab)
    r = subprocess.run([str(TOOL), "--tokenize", str(tmp_path / "v.txt"), str(tmp_path / "t.txt"),
                        "128", str(tmp_path / "ids2.i32"), str(tmp_path / "mask2.i32")],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    np.testing.assert_array_equal(np.fromfile(tmp_path / "ids2.i32", np.int32).reshape(n, 128), ids)
    np.testing.assert_array_equal(np.fromfile(tmp_path / "mask2.i32", np.int32).reshape(n, 128),
                                  mask)


def test_cpp_tool_over_several_gpus(tmp_path):
    """`nebw_embed ... 0,1,...`: GpuBertEncoder over every visible GPU
    (nebw_comm_init_all + nebw_encode_multi) gives the single-GPU bytes."""
    import torch
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs two GPUs")
    from nebw import synth
    w = synth.make_weights(synth.MINILM, seed=16, cls_pool=False, layers=2)
    lens = np.random.default_rng(17).integers(1, 129, 37).astype(np.int32)
    ids, mask = synth.make_tokens(37, 128, lens, seed=18)
    r = _run(tmp_path, w, ids, mask, 128)
    assert r.returncode == 0, r.stderr
    one = np.fromfile(tmp_path / "out.f32", np.float32)
    devs = ",".join(str(i) for i in range(min(n, 8)))
    r = subprocess.run([str(TOOL), str(tmp_path / "m.npue"), str(tmp_path / "ids.i32"),
                        str(tmp_path / "mask.i32"), "128", str(tmp_path / "multi.f32"), devs],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    np.testing.assert_array_equal(np.fromfile(tmp_path / "multi.f32", np.float32), one)


SERVE = REPO / "oracle" / "_ref" / "npue_serve_gpu"


@pytest.mark.skipif(not SERVE.exists(),
                    reason="built only where the reference tree is (oracle/Makefile serve_check)")
def test_reference_http_serve_with_gpu_backend(tmp_path, port_oracle):
    """`serve` as the runtime runs it: the reference's own HTTP server and
    /v1/embeddings handler (app::serve_http) with the reference's tokenizer,
    the GPU encoder behind its EmbedBackend.  base64 embeddings equal the
    adapter's bytes; float ones the oracle's within the gate; an over-long
    input is the runtime's 400; SIGTERM stops the server."""
    import base64
    import json
    import signal
    import socket
    import time
    import urllib.error
    import urllib.request

    from nebw import synth
    from nebw.npue import write_bert_container
    w = synth.make_weights(synth.BGE_SMALL, seed=81, cls_pool=True, layers=2)
    model = tmp_path / "m.npue"
    write_bert_container(model, w, max_seq_len=128, vocab=synthetic_vocab(w.vocab))
    texts = synthetic_texts(9, 82, 60)
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    proc = subprocess.Popen([str(SERVE), str(model), str(port), "128"], stdout=subprocess.PIPE,
                            stderr=subprocess.PIPE, text=True)
    try:
        def post(body, path="/v1/embeddings"):
            req = urllib.request.Request(f"http://127.0.0.1:{port}{path}",
                                         data=json.dumps(body).encode(),
                                         headers={"Content-Type": "application/json"})
            try:
                with urllib.request.urlopen(req, timeout=60) as r:
                    return r.status, json.loads(r.read())
            except urllib.error.HTTPError as e:
                return e.code, json.loads(e.read())

        deadline = time.time() + 120
        while True:
            try:
                with urllib.request.urlopen(f"http://127.0.0.1:{port}/health", timeout=5) as r:
                    assert json.loads(r.read())["status"] == "ok"
                break
            except (urllib.error.URLError, ConnectionError):
                assert proc.poll() is None, proc.communicate()[1]
                assert time.time() < deadline, "server did not come up"
                time.sleep(0.5)
        st, b64 = post({"input": texts, "encoding_format": "base64"})
        assert st == 200, b64
        got = np.stack([np.frombuffer(base64.b64decode(d["embedding"]), np.float32)
                        for d in b64["data"]])
        st, fl = post({"input": texts})
        assert st == 200
        np.testing.assert_allclose(np.array([d["embedding"] for d in fl["data"]], np.float32), got,
                                   rtol=1e-6, atol=1e-7)  # %.7g text of the same floats
        # the adapter on the same texts gives the same bytes
        (tmp_path / "t.txt").write_text("\n".join(texts) + "\n")
        r = subprocess.run([str(CHECK), str(model), str(tmp_path / "t.txt"), "128",
                            str(tmp_path / "o.f32"), str(tmp_path / "i.i32"), str(tmp_path / "m.i32")],
                           capture_output=True, text=True, timeout=300)
        assert r.returncode == 0, r.stderr
        np.testing.assert_array_equal(got, np.fromfile(tmp_path / "o.f32", np.float32).reshape(got.shape))
        ids = np.fromfile(tmp_path / "i.i32", np.int32).reshape(len(texts), 128)
        mask = np.fromfile(tmp_path / "m.i32", np.int32).reshape(len(texts), 128)
        assert b64["usage"]["prompt_tokens"] == int(mask.sum())
        cos, err = parity(got, port_oracle.encode(w, ids, mask))
        assert cos >= 0.9999 and err <= 2e-3, (cos, err)
        st, e = post({"input": ["w1 " * 200]})
        assert st == 400 and "128" in e["error"]["message"], e
        st, e = post({"input": texts}, path="/v1/nothing")
        assert st == 404
    finally:
        proc.send_signal(signal.SIGTERM)
        try:
            proc.wait(timeout=60)
        except subprocess.TimeoutExpired:
            proc.kill()
            proc.wait(timeout=30)
    assert proc.returncode == 0, proc.stderr.read() if proc.stderr else ""
