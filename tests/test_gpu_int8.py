"""The int8 datapath on the tcgen05 tensor cores (nebw_quantise_rows,
nebw_stage_weight_i8, nebw_gemm_i8) against the CPU oracle's restatement of
the reference's int8 host steps, which is pinned bit-exact to the reference
itself and to tests/golden/int8_steps.npz (tests/test_oracle_pin.py).

The integer product is exact and every floating-point step is the
reference's own IEEE operation, so every comparison here is bit for bit.
"""

import sys

import numpy as np
import pytest

from conftest import REPO, parity

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
sys.path.insert(0, str(REPO / "tests" / "golden"))


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def test_quantise_rows_bit_exact(device, port_oracle):
    from make_golden import int8_step_inputs
    inp = int8_step_inputs()
    for a, ias in ((inp["a"], inp["ias"]), (inp["tail"], inp["tail_ias"])):
        rows, K = a.shape
        q = torch.empty((rows, K), dtype=torch.int8, device="cuda")
        sc = torch.empty(rows, dtype=torch.float32, device="cuda")
        device.quantise_rows(_dev(a), rows, K, _dev(ias), q, sc)
        device.sync()
        want_q, want_sc = port_oracle.quantise_rows(a, ias)
        np.testing.assert_array_equal(q.cpu().numpy(), want_q)
        np.testing.assert_array_equal(sc.cpu().numpy(), want_sc)


@pytest.mark.parametrize("K", [12, 36, 200, 384, 1000, 1536, 3072, 4096, 5120, 8192, 8196])
@pytest.mark.parametrize("bf16", [False, True])
def test_quantise_rows_widths(device, port_oracle, K, bf16):
    """Every row width the quantiser dispatches on -- the row in one warp's
    registers (K % 4 == 0 up to 2048: 1 to 16 float4 per lane), in one CTA's
    (up to 8192: 4 or 8 float4 per thread), past-K lanes idle, or read twice
    by a warp (else) -- against the oracle, bit for bit, fp32 and bf16 rows,
    with an all-zero row and rows of very different magnitude."""
    rng = np.random.default_rng(K + 7 * bf16)
    rows = 37
    a = (rng.standard_normal((rows, K)) * rng.lognormal(0, 2, (rows, 1))).astype(np.float32)
    a[5] = 0
    x = torch.from_numpy(a).cuda()
    if bf16:
        x = x.to(torch.bfloat16)
        a = x.float().cpu().numpy()
    ias = (1.0 / rng.lognormal(0.0, 0.5, K)).astype(np.float32)
    q = torch.empty((rows, K), dtype=torch.int8, device="cuda")
    sc = torch.empty(rows, dtype=torch.float32, device="cuda")
    device.quantise_rows(x, rows, K, _dev(ias), q, sc)
    device.sync()
    want_q, want_sc = port_oracle.quantise_rows(a, ias)
    np.testing.assert_array_equal(q.cpu().numpy(), want_q)
    np.testing.assert_array_equal(sc.cpu().numpy(), want_sc)


@pytest.mark.parametrize("M,K,N", [(16, 512, 512), (1, 128, 8), (300, 1024, 4096),
                                   (257, 384, 1152), (1000, 4096, 1024), (77, 48, 40)])
@pytest.mark.parametrize("act", [0, 1])
def test_gemm_i8_dequant_bit_exact(device, port_oracle, M, K, N, act):
    """C = int8 A . int8 W in int32 on kind::i8, dequantised (and gelu8'd)
    in the epilogue, against the oracle's exact int32 product and its
    dequantise / dequant-gelu steps; K not a multiple of 128 and N not a
    multiple of 32 exercise the partial K-block and column chunk."""
    rng = np.random.default_rng(M + K + N + act)
    A = rng.integers(-127, 128, (M, K), dtype=np.int8)
    W = rng.integers(-127, 128, (K, N), dtype=np.int8)
    sa = rng.lognormal(-4.0, 0.5, M).astype(np.float32)
    ws = rng.lognormal(-6.0, 0.5, N).astype(np.float32)
    bias = (rng.standard_normal(N) * 0.02).astype(np.float32)
    h = device.stage_weight_i8(W)
    out = torch.empty((M, N), dtype=torch.float32, device="cuda")
    device.gemm_i8(h, _dev(A), _dev(sa), M, K, N, _dev(ws), out, bias=_dev(bias), act=act)
    device.sync()
    device.release_weight(h)
    c = port_oracle.gemm_i8(A, W)
    want = port_oracle.dequantise(c, sa, ws, bias)
    if act:
        want = port_oracle.gelu8(want)
    np.testing.assert_array_equal(out.cpu().numpy(), want)


def test_dequant_gelu_quant_composition_bit_exact(device, port_oracle):
    """The FFN-up step of the int8 path (dequant_act_quant with gelu8): the
    GPU's gemm_i8 with gelu8 followed by quantise_rows with the next
    divisor gives the oracle's int8 rows and row scales bit for bit, on the
    pinned step inputs' shapes and value ranges."""
    from make_golden import int8_step_inputs
    inp = int8_step_inputs()
    rng = np.random.default_rng(5)
    rows, K, N = 16, 1024, 512
    A = rng.integers(-127, 128, (rows, K), dtype=np.int8)
    W = rng.integers(-127, 128, (K, N), dtype=np.int8)
    h = device.stage_weight_i8(W)
    y = torch.empty((rows, N), dtype=torch.float32, device="cuda")
    device.gemm_i8(h, _dev(A), _dev(inp["sa"]), rows, K, N, _dev(inp["ws"]), y,
                   bias=_dev(inp["bias"]), act=1)
    q = torch.empty((rows, N), dtype=torch.int8, device="cuda")
    sc = torch.empty(rows, dtype=torch.float32, device="cuda")
    device.quantise_rows(y, rows, N, _dev(inp["ias_next"]), q, sc)
    device.sync()
    device.release_weight(h)
    c = port_oracle.gemm_i8(A, W)
    want_q, want_sc = port_oracle.dequant_gelu_quant(c, inp["sa"], inp["ws"], inp["bias"],
                                                     inp["ias_next"])
    np.testing.assert_array_equal(q.cpu().numpy(), want_q)
    np.testing.assert_array_equal(sc.cpu().numpy(), want_sc)


def test_gemm_i8_refusals(device):
    import nebw
    with pytest.raises(nebw.NebwError, match="K % 16"):
        device.stage_weight_i8(np.zeros((24, 8), np.int8))
    h = device.stage_weight_i8(np.zeros((32, 8), np.int8))
    a = torch.zeros((4, 32), dtype=torch.int8, device="cuda")
    s = torch.ones(8, dtype=torch.float32, device="cuda")
    out = torch.empty((4, 8), dtype=torch.float32, device="cuda")
    with pytest.raises(nebw.NebwError, match="mismatch"):
        device.gemm_i8(h, a, s, 4, 16, 8, s, out)
    with pytest.raises(nebw.NebwError, match="act"):
        device.gemm_i8(h, a, s, 4, 32, 8, s, out, act=2)
    device.release_weight(h)


# ---- the int8 encoder pass (NEBW_DATAPATH_I8) ------------------------------

def test_gemm_i8_bf16_output_bit_exact(device, port_oracle):
    """The QKV form of the int8 GEMM: the dequantised value narrowed RNE to
    bf16 -- the oracle's dequantise followed by its to_bf16, bit for bit."""
    import nebw
    rng = np.random.default_rng(31)
    M, K, N = 300, 384, 1152
    A = rng.integers(-127, 128, (M, K), dtype=np.int8)
    W = rng.integers(-127, 128, (K, N), dtype=np.int8)
    sa = rng.lognormal(-4.0, 0.5, M).astype(np.float32)
    ws = rng.lognormal(-6.0, 0.5, N).astype(np.float32)
    bias = (rng.standard_normal(N) * 0.02).astype(np.float32)
    h = device.stage_weight_i8(W)
    out = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    device.gemm_i8(h, _dev(A), _dev(sa), M, K, N, _dev(ws), out, bias=_dev(bias),
                   c_dtype=nebw.BF16)
    device.sync()
    device.release_weight(h)
    want = port_oracle.to_bf16(port_oracle.dequantise(port_oracle.gemm_i8(A, W), sa, ws, bias))
    np.testing.assert_array_equal(out.cpu().view(torch.int16).numpy().view(np.uint16), want)


def test_quantise_rows_bf16_input_bit_exact(device, port_oracle):
    """The attention-out step's quantiser reads the bf16 attention output,
    widened exactly: the oracle's quantiser on the widened values."""
    rng = np.random.default_rng(32)
    rows, K = 257, 1024
    x = torch.from_numpy((rng.standard_normal((rows, K)) * 0.3).astype(np.float32)).to(
        torch.bfloat16).cuda()
    x[3] = 0  # an all-zero row: scale 1, q 0
    ias = (1.0 / rng.lognormal(0.0, 0.5, K)).astype(np.float32)
    q = torch.empty((rows, K), dtype=torch.int8, device="cuda")
    sc = torch.empty(rows, dtype=torch.float32, device="cuda")
    device.quantise_rows(x, rows, K, _dev(ias), q, sc)
    device.sync()
    want_q, want_sc = port_oracle.quantise_rows(x.float().cpu().numpy(), ias)
    np.testing.assert_array_equal(q.cpu().numpy(), want_q)
    np.testing.assert_array_equal(sc.cpu().numpy(), want_sc)
    assert want_sc[3] == 1.0 and not want_q[3].any()


@pytest.mark.parametrize("H", [384, 1024])
def test_layernorm_quant(device, port_oracle, H):
    """add_norm_quant: x = LN(x + y) as the plain LayerNorm computes it, and
    the normalised rows quantised in the same kernel -- bit for bit the
    oracle's quantiser applied to the kernel's own fp32 rows; with q null
    only x is written."""
    rng = np.random.default_rng(33 + H)
    rows = 555
    x = rng.standard_normal((rows, H)).astype(np.float32)
    y = (rng.standard_normal((rows, H)) * 2).astype(np.float32)
    g = rng.standard_normal(H).astype(np.float32)
    b = rng.standard_normal(H).astype(np.float32)
    ias = (1.0 / rng.lognormal(0.0, 0.5, H)).astype(np.float32)
    x_d = _dev(x)
    q = torch.full((rows, H), 99, dtype=torch.int8, device="cuda")
    sc = torch.zeros(rows, dtype=torch.float32, device="cuda")
    device.layernorm_quant(x_d, _dev(g), _dev(b), rows, H, y=_dev(y), ias=_dev(ias), q=q,
                           scale=sc)
    device.sync()
    got = x_d.cpu().numpy()
    want = port_oracle.layer_norm(x + y, g, b)
    assert np.abs(got - want).max() <= 2e-5 * np.abs(want).max()
    want_q, want_sc = port_oracle.quantise_rows(got, ias)
    np.testing.assert_array_equal(q.cpu().numpy(), want_q)
    np.testing.assert_array_equal(sc.cpu().numpy(), want_sc)
    # plain LN form: no y, no quantised output (q untouched)
    x2 = _dev(x)
    q2 = torch.full((rows, H), 99, dtype=torch.int8, device="cuda")
    device.layernorm_quant(x2, _dev(g), _dev(b), rows, H)
    device.sync()
    assert np.abs(x2.cpu().numpy() - port_oracle.layer_norm(x, g, b)).max() <= \
        2e-5 * np.abs(want).max()
    assert bool((q2 == 99).all())


def _i8_container(tmp_path, key):
    import make_golden
    path = tmp_path / f"{key}_i8.npue"
    digest = make_golden.write_pretiled(path, key, "i8")
    return path, digest


@pytest.mark.parametrize("name", ["i8_array_c1", "i8_array_c2"])
def test_int8_pass_matches_reference_array_path(device, port_oracle, tmp_path, name):
    """The int8 datapath on the B200 (nebw_model_set_datapath I8) against the
    reference's own int8 array path -- BertEncoder::run with every GEMM on the
    array, its rows committed in tests/golden by make_golden.py -- and against
    the oracle's restatement of that path (pinned bit-exact to it), on the
    regenerated int8 container.  Every int8 step is bit-exact on its own (the
    tests above); the attention runs on the bf16 tensor cores (the
    reference's in fp32 on the host), and a quantiser turns its small
    differences into whole quantisation steps wherever a value lies near a
    rounding boundary, so the two passes agree to int8 rounding: measured
    cos 0.99996 / max-abs 1.5e-3 (MiniLM, 6 layers) and 0.99969 / 4.1e-3
    (bge-small, 12 layers, rows to 511 tokens) -- the bf16 datapath is as far
    from the reference's int8 path (0.99972).  Gate: cos >= 0.9995, max-abs
    <= 6e-3.  The int8 pass really quantises: it is not the bf16 datapath's
    result."""
    import make_golden
    import nebw
    from nebw import synth
    g = dict(np.load(REPO / "tests" / "golden" / f"{name}.npz"))
    key, _n = make_golden.I8_ARRAY[name]
    path, digest = _i8_container(tmp_path, key)
    assert digest == str(g["container_sha256"])
    m = nebw.Model.from_npue(device, path)
    try:
        bf16 = m.encode(g["ids"], g["lens"])
        m.set_datapath("i8")
        got = m.encode(g["ids"], g["lens"])
        again = m.encode(g["ids"], g["lens"])
    finally:
        m.close()
    assert np.isfinite(got).all()
    np.testing.assert_array_equal(got, again)
    cos, err = parity(got, g["embeddings"])
    cos_b, err_b = parity(bf16, g["embeddings"])
    print(f"{name}: int8 pass vs reference array path cos {cos:.7f} max-abs {err:.3e}; "
          f"bf16 pass vs it cos {cos_b:.7f} max-abs {err_b:.3e}")
    assert cos >= 0.9995 and err <= 6e-3, f"{name} vs reference: cos {cos:.7f}, max abs {err:.3e}"
    want = port_oracle.encode_i8(synth.config_weights(synth.CONFIGS[key]), path, g["ids"],
                                 g["mask"])
    np.testing.assert_array_equal(want, g["embeddings"])  # the oracle is the reference here
    assert not np.array_equal(got, bf16)


def test_int8_pass_bge_large_layers_vs_oracle(device, port_oracle, tmp_path):
    """bge-large's geometry (hidden 1024, FFN 4096: the FFN-down product runs
    on the CTA-pair int8 GEMM, the others on the single-CTA one), 2 layers,
    as an int8 container: the GPU's int8 pass against the oracle's int8
    array path (pinned bit-exact to the reference's) on 6 rows of the
    benchmark batch, the shortest and the longest among them."""
    import make_golden
    import nebw
    from nebw import synth
    from nebw.npue import write_bert_container
    cfg = synth.CONFIGS["bge-large"]
    w = synth.config_weights(cfg, layers=2)
    ids, mask, lens = synth.config_batch(cfg)
    rows = make_golden.sample_rows(lens, 6)
    path = tmp_path / "large_i8.npue"
    write_bert_container(path, w, max_seq_len=cfg.seq, gemm_layout="pretiled_bf16", a_dtype="i8",
                         tile=make_golden.PRETILED_TILE, mac=make_golden.PRETILED_MAC,
                         smooth_seed=make_golden.PRETILED_SMOOTH_SEED)
    m = nebw.Model.from_npue(device, path)
    try:
        m.set_datapath("i8")
        got = m.encode(ids[rows], lens[rows])
    finally:
        m.close()
    want = port_oracle.encode_i8(w, path, ids[rows], mask[rows])
    cos, err = parity(got, want)
    print(f"bge-large 2-layer int8 pass vs oracle: cos {cos:.7f} max-abs {err:.3e}")
    assert np.isfinite(got).all() and cos >= 0.9995 and err <= 6e-3, (cos, err)


def test_int8_pass_full_batch_and_order(device, tmp_path):
    """The whole MiniLM batch through the int8 datapath: every row finite, and
    each row independent of its batch neighbours (a permuted batch gives the
    same rows bit for bit, as every step is row-local or per sequence), also
    when the pass is replayed as a CUDA graph."""
    import nebw
    from nebw import synth
    cfg = synth.CONFIGS["minilm"]
    ids, _mask, lens = synth.config_batch(cfg)
    path, _ = _i8_container(tmp_path, "minilm")
    m = nebw.Model.from_npue(device, path)
    try:
        m.set_datapath("i8")
        full = m.encode(ids, lens)
        order = np.random.default_rng(3).permutation(len(lens))
        perm = m.encode(ids[order], lens[order])
        m.set_graphs(True)  # the int8 pass replayed as a CUDA graph: the same rows
        graphed = m.encode(ids[order], lens[order])
    finally:
        m.close()
    assert np.isfinite(full).all()
    np.testing.assert_array_equal(perm, full[order])
    np.testing.assert_array_equal(graphed, perm)


def test_int8_datapath_refusals(device, tmp_path):
    import nebw
    from nebw import synth
    w = synth.config_weights(synth.CONFIGS["minilm"], layers=2)
    m = nebw.Model.from_weights(device, w, max_seq_len=128)
    try:
        with pytest.raises(nebw.NebwError, match="int8 operands"):
            m.set_datapath("i8")
        with pytest.raises(nebw.NebwError, match="is \\[384, 384\\]"):
            m.set_int8_operand("layer.0.qkv", np.zeros((384, 384), np.int8),
                               np.ones(384, np.float32), np.ones(384, np.float32))
        with pytest.raises(nebw.NebwError, match="positive and finite"):
            m.set_int8_operand("layer.0.attn_out", np.zeros((384, 384), np.int8),
                               np.ones(384, np.float32), np.zeros(384, np.float32))
        with pytest.raises(nebw.NebwError, match="refused"):
            m.set_int8_operand("layer.7.qkv", np.zeros((384, 1152), np.int8),
                               np.ones(1152, np.float32), np.ones(384, np.float32))
    finally:
        m.close()
    path, _ = _i8_container(tmp_path, "minilm")
    m = nebw.Model.from_npue(device, path)
    try:
        m.set_datapath("i8")
        ids, _mask, lens = synth.config_batch(synth.CONFIGS["minilm"])
        i_d = torch.from_numpy(ids[:4]).cuda()
        l_d = torch.from_numpy(lens[:4].astype(np.int32)).cuda()
        out = torch.empty((4, m.hidden), device="cuda")
        S = ids.shape[1]

        def static():
            nebw._check(nebw.lib().nebw_encode_device_static(m.h, i_d.data_ptr(), l_d.data_ptr(),
                                                             4, S, out.data_ptr(), None))

        with pytest.raises(nebw.NebwError, match="int8 datapath"):
            static()
        m.set_datapath("bf16")
        static()
        device.sync()
    finally:
        m.close()
    gated = synth.config_weights(synth.CONFIGS["nomic-base"], layers=1)
    m = nebw.Model.from_weights(device, gated, max_seq_len=128)
    try:
        with pytest.raises(nebw.NebwError, match="plain BERT"):
            m.set_datapath("i8")
    finally:
        m.close()
