"""Pinning the oracle (CPU, no GPU).

The C restatement (oracle/bert_oracle.c) is checked two ways:
  * against the reference's own host path compiled from its tree
    (oracle/_ref), op by op and end to end, bit for bit -- where that build
    exists;
  * against the committed golden fixtures (tests/golden/*.npz), which that
    compiled reference produced (tests/golden/make_golden.py) -- always.
"""

import numpy as np
import pytest

from conftest import REPO

GOLDEN = REPO / "tests" / "golden"


def load_golden(name):
    return dict(np.load(GOLDEN / f"{name}.npz"))


def test_port_ops_bit_exact_vs_reference(port_oracle, ref_oracle):
    rng = np.random.default_rng(0)
    for M, K, N in ((37, 64, 40), (9, 384, 1152), (1, 8, 8)):
        A = rng.standard_normal((M, K)).astype(np.float32)
        B = rng.standard_normal((K, N)).astype(np.float32)
        b = rng.standard_normal(N).astype(np.float32)
        np.testing.assert_array_equal(port_oracle.gemm_nt(A, B, b), ref_oracle.gemm_nt(A, B, b))
    v = np.concatenate([np.linspace(-12, 12, 8192, dtype=np.float32),
                        rng.standard_normal(4096).astype(np.float32) * 3])
    np.testing.assert_array_equal(port_oracle.gelu8(v), ref_oracle.gelu8(v))
    e = np.linspace(-120, 0, 16384, dtype=np.float32)
    np.testing.assert_array_equal(port_oracle.exp2(e), ref_oracle.exp2(e))
    x = rng.standard_normal(10000).astype(np.float32) * 1e3
    x[:4] = [0.0, -0.0, 65504.0, 3.3895314e38]
    np.testing.assert_array_equal(port_oracle.to_bf16(x), ref_oracle.to_bf16(x))


@pytest.mark.parametrize("cls", [0, 1])
def test_port_pool_bit_exact_vs_reference(port_oracle, ref_oracle, cls):
    rng = np.random.default_rng(cls)
    S, H = 64, 384
    h = rng.standard_normal((5, S, H)).astype(np.float32)
    am = (np.arange(S)[None, :] < np.array([[1], [7], [64], [33], [2]])).astype(np.float32)
    np.testing.assert_array_equal(port_oracle.pool_rows(h, am, S, cls),
                                  ref_oracle.pool_rows(h, am, S, cls))


def test_pool_refuses_masked_cls(port_oracle, ref_oracle):
    h = np.zeros((1, 8, 16), np.float32)
    am = np.zeros((1, 8), np.float32)
    for o in (port_oracle, ref_oracle):
        with pytest.raises(RuntimeError, match="CLS"):
            o.pool_rows(h, am, 8, 1)


def test_port_encode_bit_exact_vs_reference(port_oracle, ref_oracle):
    from nebw import synth
    cfg = synth.CONFIGS["minilm"]
    w = synth.config_weights(cfg, layers=2)
    ids, mask, _ = synth.config_batch(cfg)
    a, ha = port_oracle.encode(w, ids[:5], mask[:5], hidden=True)
    b, hb = ref_oracle.encode(w, ids[:5], mask[:5], hidden=True)
    np.testing.assert_array_equal(ha, hb)
    np.testing.assert_array_equal(a, b)


def test_golden_weights_regenerate():
    """The generator still makes the weights the fixtures were made with."""
    import sys
    sys.path.insert(0, str(GOLDEN))
    from make_golden import weights_fingerprint

    from nebw import synth
    g = load_golden("minilm_c1")
    w = synth.config_weights(synth.CONFIGS[str(g["config"])])
    assert weights_fingerprint(w) == str(g["weights_fingerprint"])
    ids, mask, lens = synth.config_batch(synth.CONFIGS[str(g["config"])])
    np.testing.assert_array_equal(ids[g["rows"]], g["ids"])
    np.testing.assert_array_equal(mask[g["rows"]], g["mask"])


def test_port_matches_golden_minilm(port_oracle):
    from nebw import synth
    g = load_golden("minilm_c1")
    w = synth.config_weights(synth.CONFIGS["minilm"])
    got = port_oracle.encode(w, g["ids"], g["mask"])
    np.testing.assert_array_equal(got, g["embeddings"])


def test_port_matches_golden_bge_small_row(port_oracle):
    from nebw import synth
    g = load_golden("bge_small_c2")
    w = synth.config_weights(synth.CONFIGS["bge-small"])
    r = int(np.argmin(g["lens"]))
    got = port_oracle.encode(w, g["ids"][r:r + 1], g["mask"][r:r + 1])
    np.testing.assert_array_equal(got, g["embeddings"][r:r + 1])


def test_golden_fixtures_are_sane():
    for name in ("minilm_c1", "bge_small_c2", "bge_base_c3", "bge_large_c4"):
        g = load_golden(name)
        e = g["embeddings"]
        assert np.isfinite(e).all()
        np.testing.assert_allclose(np.linalg.norm(e, axis=1), 1.0, rtol=1e-5)
        assert (g["mask"].sum(1) == g["lens"]).all()
        assert (g["ids"][:, 0] == 101).all()


# ---- ViT (benchmark configuration 5) ---------------------------------------

def _small_vit():
    from nebw import synth
    arch = synth.VitArch("vit-test", 2, 768, 12, 3072, image_size=32)
    return arch, synth.make_vit_weights(arch, 7), synth.make_images(3, arch, 8)


def test_port_vit_bit_exact_vs_reference(port_oracle, ref_oracle):
    """The C restatement of VitEncoder::run against the reference's own
    vit/encoder.cpp + whisper/npu_ops.cpp host path: every row, bit for bit."""
    _, w, imgs = _small_vit()
    a, ha = port_oracle.vit_encode(w, imgs, hidden=True)
    b, hb = ref_oracle.vit_encode(w, imgs, hidden=True)
    np.testing.assert_array_equal(ha, hb)
    np.testing.assert_array_equal(a, b)


def test_vit_im2col_order(port_oracle):
    """Patch row p*n+q holds channel-major (c, i, j) pixels
    (runtime/src/vit/image.cpp:732-755), checked against numpy's reshape."""
    from nebw import synth
    img = synth.make_images(1, synth.VIT_BASE, 3)[0]
    P, n = 16, 224 // 16
    want = img.reshape(3, n, P, n, P).transpose(1, 3, 0, 2, 4).reshape(n * n, 3 * P * P)
    np.testing.assert_array_equal(port_oracle.vit_im2col(img, P), want)


def test_vit_golden_inputs_regenerate():
    import hashlib
    import sys
    sys.path.insert(0, str(GOLDEN))
    from make_golden import weights_fingerprint

    from nebw import synth
    g = load_golden("vit_base_c5")
    cfg = synth.VIT_CONFIGS[str(g["config"])]
    assert weights_fingerprint(synth.vit_config_weights(cfg)) == str(g["weights_fingerprint"])
    imgs = synth.vit_config_images(cfg, n=int(g["n_images"]))
    assert hashlib.sha256(imgs.tobytes()).hexdigest() == str(g["image_sha256"])
    assert np.isfinite(g["embeddings"]).all()


def test_port_matches_golden_vit(port_oracle):
    from nebw import synth
    g = load_golden("vit_base_c5")
    cfg = synth.VIT_CONFIGS["vit-base"]
    got = port_oracle.vit_encode(synth.vit_config_weights(cfg),
                                 synth.vit_config_images(cfg, n=1))
    np.testing.assert_array_equal(got, g["embeddings"][:1])


@pytest.mark.parametrize("key", ["nomic-base", "gte-base"])
def test_port_gated_rope_bit_exact_vs_reference(port_oracle, ref_oracle, key):
    """The rotary / gated families (nomic: RoPE theta, SwiGLU, no biases;
    gte: RoPE frequency data, erf GeGLU): the restatement against the
    reference's own host path on the same 2-layer container, every hidden
    row and the pooled output, bit for bit."""
    from nebw import synth
    cfg = synth.CONFIGS[key]
    w = synth.config_weights(cfg, layers=2)
    lens = np.array([64, 1, 33, 63, 17], np.int32)
    ids, mask = synth.make_tokens(len(lens), 64, lens, seed=41)
    a, ha = port_oracle.encode(w, ids, mask, hidden=True)
    b, hb = ref_oracle.encode(w, ids, mask, hidden=True)
    np.testing.assert_array_equal(ha, hb)
    np.testing.assert_array_equal(a, b)


@pytest.mark.parametrize("name,key", [("nomic_c6", "nomic-base"), ("gte_c7", "gte-base")])
def test_port_matches_golden_gated(port_oracle, name, key):
    """The restatement reproduces the reference's golden rows of the full
    12-layer models (shortest row of each fixture), bit for bit."""
    import sys
    sys.path.insert(0, str(GOLDEN))
    from make_golden import weights_fingerprint

    from nebw import synth
    g = load_golden(name)
    w = synth.config_weights(synth.CONFIGS[key])
    assert weights_fingerprint(w) == str(g["weights_fingerprint"])
    r = int(np.argmin(g["lens"]))
    got = port_oracle.encode(w, g["ids"][r:r + 1], g["mask"][r:r + 1])
    np.testing.assert_array_equal(got, g["embeddings"][r:r + 1])


# ---- the int8 datapath's host steps --------------------------------------

def _int8_golden_module():
    import sys
    sys.path.insert(0, str(GOLDEN))
    import make_golden
    return make_golden


def _bits_equal(a, b):
    a, b = np.asarray(a), np.asarray(b)
    assert a.shape == b.shape and a.dtype == b.dtype
    if a.dtype == np.float32:
        a, b = a.view(np.uint32), b.view(np.uint32)
    np.testing.assert_array_equal(a, b)


def test_port_int8_steps_bit_exact_vs_reference(port_oracle, ref_oracle):
    """quantise_a_int8, dequantise_c (int32 C) and dequant_act_quant (gelu8)
    of host_kernels.hpp, compiled from the reference tree, against the C
    restatement: bit for bit, on seeded inputs with rounding ties, a zero
    row, a scalar tail and int32 values that round when widened."""
    mg = _int8_golden_module()
    for seed in (mg.INT8_SEED, 7, 8):
        inp = mg.int8_step_inputs(seed)
        got = mg.int8_step_outputs(port_oracle, inp)
        want = mg.int8_step_outputs(ref_oracle, inp)
        for k in want:
            _bits_equal(got[k], want[k])


def test_port_int8_matches_golden(port_oracle):
    mg = _int8_golden_module()
    g = load_golden("int8_steps")
    inp = mg.int8_step_inputs(int(g["seed"]))
    assert mg.int8_inputs_sha256(inp) == str(g["inputs_sha256"])
    got = mg.int8_step_outputs(port_oracle, inp)
    for k, v in got.items():
        _bits_equal(v, g[k])
    # the crafted row: 127 sets the scale to 1, ties round to even
    np.testing.assert_array_equal(got["q"][1, :9], [127, 0, 2, 2, 0, -2, -2, 126, -126])
    assert got["scale"][0] == 1.0 and not got["q"][0].any()  # an all-zero row


def test_port_int8_quantise_invariants(port_oracle):
    rng = np.random.default_rng(5)
    a = rng.standard_normal((64, 384)).astype(np.float32) * 10
    ias = (1.0 / rng.lognormal(0.0, 0.5, 384)).astype(np.float32)
    q, sc = port_oracle.quantise_rows(a, ias)
    assert np.abs(q.astype(np.int32)).max() <= 127
    assert (np.abs(q.astype(np.int32)).max(axis=1) == 127).all()
    # each value is within half a step of its quantised value
    assert (np.abs(q * sc[:, None] - a * ias) <= 0.5 * sc[:, None] * (1 + 1e-6)).all()


def test_port_gemm_i8_exact(port_oracle):
    rng = np.random.default_rng(6)
    for M, K, N in ((7, 64, 40), (33, 1024, 96)):
        A = rng.integers(-127, 128, (M, K), dtype=np.int8)
        B = rng.integers(-127, 128, (K, N), dtype=np.int8)
        want = (A.astype(np.int64) @ B.astype(np.int64)).astype(np.int32)
        np.testing.assert_array_equal(port_oracle.gemm_i8(A, B, threads=2), want)


# ---- the int8 pass: BertEncoder::run's array path ---------------------------

def test_port_int8_pass_bit_exact_vs_reference(port_oracle, ref_oracle, tmp_path):
    """The C restatement of the int8 array path (nebw_oracle_encode_i8)
    against the reference's own BertEncoder::run with every GEMM on the array
    (oracle/ref_driver.cpp nebw_ref_encode_array: the reference's int8 host
    steps and fused epilogues, each dispatch the exact int32 product), on the
    int8 pre-tiled MiniLM container: embeddings and every hidden row bit for
    bit.  The array path really quantises: it differs from the reference's
    host path on the same container, within int8 rounding."""
    mg = _int8_golden_module()
    from nebw import synth
    cfg = synth.CONFIGS["minilm"]
    w = synth.config_weights(cfg)
    ids, mask, lens = synth.config_batch(cfg)
    rows = mg.sample_rows(lens, 4)
    path = tmp_path / "c.npue"
    mg.write_pretiled(path, "minilm", "i8")
    want, want_h = ref_oracle.encode_container(path, cfg.seq, ids[rows], mask[rows],
                                               hidden_size=cfg.arch.hidden, array=True,
                                               hidden=True)
    got, got_h = port_oracle.encode_i8(w, path, ids[rows], mask[rows], hidden=True)
    _bits_equal(got, want)
    _bits_equal(got_h, want_h)
    host = ref_oracle.encode_container(path, cfg.seq, ids[rows], mask[rows],
                                       hidden_size=cfg.arch.hidden)
    cos = (host * got).sum(1) / np.linalg.norm(host, axis=1) / np.linalg.norm(got, axis=1)
    assert not np.array_equal(host, got) and cos.min() >= 0.999, cos.min()


@pytest.mark.parametrize("name", ["i8_array_c1", "i8_array_c2"])
def test_port_matches_golden_i8_array(port_oracle, tmp_path, name):
    """The int8 restatement against the reference's array-path rows committed
    in tests/golden (made by make_golden.py on the regenerated container, whose
    SHA-256 is checked), bit for bit."""
    mg = _int8_golden_module()
    from nebw import synth
    g = load_golden(name)
    key, _n = mg.I8_ARRAY[name]
    path = tmp_path / "c.npue"
    assert mg.write_pretiled(path, key, "i8") == str(g["container_sha256"])
    w = synth.config_weights(synth.CONFIGS[key])
    got = port_oracle.encode_i8(w, path, g["ids"], g["mask"])
    _bits_equal(got, g["embeddings"])
