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

from conftest import REPO

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
