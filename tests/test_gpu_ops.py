"""Op-level parity of the CUDA kernels, through the C ABI, on a B200.

Integer/byte work (packing offsets, the bf16 RNE narrow, gelu8 in the
epilogue) is checked bit-exactly against the CPU oracle; floating-point
work against a float64 computation on the same bf16 operands with the
tolerance stated in each test.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns, round-to-nearest-even."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, np.uint16).astype(np.uint32) << 16).view(np.float32)


def dev_tensor(a: np.ndarray):
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16).copy()).cuda().view(torch.bfloat16)
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host_bits(t) -> np.ndarray:
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


GEMM_SHAPES = [
    (1, 64, 8), (37, 200, 24), (128, 384, 128), (300, 384, 1152), (1000, 384, 384),
    (257, 768, 2304), (513, 1024, 1024), (2048, 1024, 4096), (777, 4096, 1024),
]


@pytest.mark.parametrize("M,K,N", GEMM_SHAPES)
def test_gemm_fp32_out_matches_float64(device, M, K, N):
    rng = np.random.default_rng(M * 7 + K + N)
    A = bf16_bits(rng.standard_normal((M, K), np.float32))
    W = rng.standard_normal((K, N), np.float32) * 0.05
    bias = rng.standard_normal(N).astype(np.float32)
    h = device.stage_weight(W)
    Wb = bits_to_f32(bf16_bits(W)).astype(np.float64)
    ref = bits_to_f32(A).astype(np.float64) @ Wb + bias
    a_d = dev_tensor(A)
    c_d = torch.empty((M, N), dtype=torch.float32, device="cuda")
    device.gemm(h, a_d, M, K, N, c_d, bias=dev_tensor(bias), c_dtype=0)
    device.sync()
    got = c_d.cpu().numpy()
    # fp32 accumulation of K bf16 products against float64: |err| <= 1e-5 * sqrt(K) * scale
    scale = np.abs(ref).max()
    assert np.isfinite(got).all()
    assert np.abs(got - ref).max() <= 2e-6 * np.sqrt(K) * scale + 1e-6
    device.release_weight(h)


@pytest.mark.parametrize("M,K,N", [(37, 200, 24), (300, 384, 1152), (513, 1024, 4096)])
def test_gemm_epilogues_bit_exact(device, port_oracle, M, K, N):
    """bf16 narrow, gelu8 and residual epilogues reproduce, bit for bit, the
    oracle's to_bf16 / gelu8 / fp32 add applied to the fp32 epilogue's
    output (same accumulator, so the only difference can be the epilogue)."""
    rng = np.random.default_rng(K + N)
    A = bf16_bits(rng.standard_normal((M, K), np.float32))
    W = rng.standard_normal((K, N), np.float32) * 0.05
    bias = rng.standard_normal(N).astype(np.float32)
    resid = rng.standard_normal((M, N)).astype(np.float32)
    h = device.stage_weight(W)
    a_d, b_d = dev_tensor(A), dev_tensor(bias)
    f = torch.empty((M, N), dtype=torch.float32, device="cuda")
    device.gemm(h, a_d, M, K, N, f, bias=b_d, c_dtype=0)
    outs = {}
    for name, act in (("plain", 0), ("gelu8", 1)):
        o = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
        device.gemm(h, a_d, M, K, N, o, bias=b_d, act=act, c_dtype=1)
        outs[name] = o
    r = dev_tensor(resid)
    device.gemm(h, a_d, M, K, N, r, bias=b_d, residual=r, c_dtype=0)  # in place
    device.sync()
    f_h = f.cpu().numpy()
    np.testing.assert_array_equal(host_bits(outs["plain"]), port_oracle.to_bf16(f_h))
    np.testing.assert_array_equal(host_bits(outs["gelu8"]),
                                  port_oracle.to_bf16(port_oracle.gelu8(f_h)))
    np.testing.assert_array_equal(r.cpu().numpy(), f_h + resid)
    device.release_weight(h)


def test_gemm_erf_epilogue(device):
    rng = np.random.default_rng(5)
    M, K, N = 200, 384, 1536
    A = bf16_bits(rng.standard_normal((M, K), np.float32))
    W = rng.standard_normal((K, N), np.float32) * 0.05
    h = device.stage_weight(W)
    a_d = dev_tensor(A)
    f = torch.empty((M, N), dtype=torch.float32, device="cuda")
    o = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    device.gemm(h, a_d, M, K, N, f, c_dtype=0)
    device.gemm(h, a_d, M, K, N, o, act=2, c_dtype=1)
    device.sync()
    from math import erf
    x = f.cpu().numpy().astype(np.float64)
    ref = 0.5 * x * (1.0 + np.vectorize(erf)(x / np.sqrt(2.0)))
    got = bits_to_f32(host_bits(o)).astype(np.float64)
    # bf16 output: half an ulp of bf16 (2^-9 relative) plus erff's few-ulp error
    assert np.all(np.abs(got - ref) <= np.abs(ref) * 2.0 ** -8 + 1e-6)
    device.release_weight(h)


@pytest.mark.parametrize("H", [384, 768, 1024])
def test_layernorm(device, port_oracle, H):
    rng = np.random.default_rng(H)
    rows = 1000
    x = (rng.standard_normal((rows, H)) * 3 + 0.5).astype(np.float32)
    g = rng.standard_normal(H).astype(np.float32)
    b = rng.standard_normal(H).astype(np.float32)
    x_d = dev_tensor(x)
    a_d = torch.empty((rows, H), dtype=torch.bfloat16, device="cuda")
    device.layernorm(x_d, dev_tensor(g), dev_tensor(b), rows, H, a_bf16=a_d)
    device.sync()
    got = x_d.cpu().numpy()
    want = port_oracle.layer_norm(x, g, b)
    # fp32 two-pass LN, summation order differs from the oracle's eight lanes
    assert np.abs(got - want).max() <= 2e-5 * np.abs(want).max()
    np.testing.assert_array_equal(host_bits(a_d), port_oracle.to_bf16(got))


@pytest.mark.parametrize("y_bf16", [False, True])
def test_add_layernorm(device, port_oracle, y_bf16):
    """x = LN(x + y): y as an fp32 or a bf16 GEMM output, widened exactly."""
    rng = np.random.default_rng(11 + y_bf16)
    rows, H = 777, 1024
    x = rng.standard_normal((rows, H)).astype(np.float32)
    y = (rng.standard_normal((rows, H)) * 2).astype(np.float32)
    g = rng.standard_normal(H).astype(np.float32)
    b = rng.standard_normal(H).astype(np.float32)
    if y_bf16:
        y_d = torch.from_numpy(y).to(torch.bfloat16).cuda()
        y_host = y_d.float().cpu().numpy()
    else:
        y_d = dev_tensor(y)
        y_host = y
    x_d = dev_tensor(x)
    a_d = torch.empty((rows, H), dtype=torch.bfloat16, device="cuda")
    device.layernorm(x_d, dev_tensor(g), dev_tensor(b), rows, H, y=y_d, a_bf16=a_d)
    device.sync()
    got = x_d.cpu().numpy()
    want = port_oracle.layer_norm(y_host + x, g, b)
    assert np.abs(got - want).max() <= 2e-5 * np.abs(want).max()
    np.testing.assert_array_equal(host_bits(a_d), port_oracle.to_bf16(got))


def test_pack_offsets_bit_exact(device):
    rng = np.random.default_rng(3)
    for B in (1, 7, 1024, 5000):
        lens = rng.integers(1, 513, size=B).astype(np.int32)
        ld = dev_tensor(lens)
        lo = torch.empty(B, dtype=torch.int32, device="cuda")
        off = torch.empty(B + 1, dtype=torch.int32, device="cuda")
        device.pack_offsets(ld, B, 512, lo, off)
        device.sync()
        want = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
        np.testing.assert_array_equal(off.cpu().numpy(), want)
        np.testing.assert_array_equal(lo.cpu().numpy(), lens)


def test_pack_offsets_refuses_bad_length(device):
    import nebw
    lens = np.array([5, 0, 3], np.int32)
    lo = torch.empty(3, dtype=torch.int32, device="cuda")
    off = torch.empty(4, dtype=torch.int32, device="cuda")
    device.pack_offsets(dev_tensor(lens), 3, 8, lo, off)
    with pytest.raises(nebw.NebwError, match="length"):
        device.sync()
    device.sync()  # the error word was cleared


def test_bounded_wait_runs_out_and_reports(device):
    """The kernels' bounded mbarrier wait, made to run out: a probe waits 1 ms
    on a barrier nothing arrives on (no copy or product in flight), returns,
    records the wait-timeout code, and the next sync reports it by name; the
    context stays usable (a second probe and an op still run)."""
    import nebw
    device.sync()
    assert device.check_bounded_wait(1_000_000)
    with pytest.raises(nebw.NebwError, match="bounded device wait timed out") as e:
        device.sync()
    assert e.value.code == 5  # NEBW_EDEVICE
    device.sync()  # cleared
    assert device.check_bounded_wait(10_000)
    with pytest.raises(nebw.NebwError, match="timed out"):
        device.sync()
    x = torch.ones(256, device="cuda")
    y = torch.empty(256, dtype=torch.bfloat16, device="cuda")
    device.narrow_bf16(x, 256, y)
    device.sync()
    assert bool((y.float() == 1).all())
    with pytest.raises(nebw.NebwError, match="refused"):
        device.check_bounded_wait(10)


def _packed(lens):
    off = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    return off, int(off[-1])


@pytest.mark.parametrize("D,heads,kind", [(32, 12, 0), (64, 16, 0), (64, 16, 1), (64, 12, 1),
                                          (32, 12, 1), (32, 16, 1)])
def test_attention_matches_float64(device, D, heads, kind):
    """kind 0: mma.sync flash kernel; kind 1: tcgen05 kernel (head_dim 64
    with 128-byte swizzled head tiles, head_dim 32 with 64-byte ones)."""
    rng = np.random.default_rng(D + kind)
    lens = np.array([1, 8, 63, 64, 65, 127, 128, 129, 130, 512, 200, 257], np.int32)
    off, T = _packed(lens)
    H = D * heads
    qkv = bf16_bits(rng.standard_normal((T, 3 * H), np.float32) * 0.5)
    ctx = torch.zeros((T, H), dtype=torch.bfloat16, device="cuda")
    device.set_attention_kernel(kind)
    try:
        device.attention(dev_tensor(qkv), T, dev_tensor(off), dev_tensor(lens), len(lens), 512,
                         heads, D, ctx)
        device.sync()
    finally:
        device.set_attention_kernel(device.ATTN_TCGEN05)
    got = bits_to_f32(host_bits(ctx)).astype(np.float64)
    q = bits_to_f32(qkv).astype(np.float64)
    for b, L in enumerate(lens):
        r = slice(off[b], off[b] + L)
        for h in range(heads):
            Q = q[r, h * D:(h + 1) * D]
            Kt = q[r, H + h * D:H + (h + 1) * D]
            V = q[r, 2 * H + h * D:2 * H + (h + 1) * D]
            s = Q @ Kt.T
            p = np.exp(s - s.max(1, keepdims=True))
            p /= p.sum(1, keepdims=True)
            want = p @ V
            # P is rounded to bf16 for the PV product; output bf16
            err = np.abs(got[r, h * D:(h + 1) * D] - want).max()
            assert err <= 1.5e-2 * max(1.0, np.abs(want).max()), (b, h, err)


@pytest.mark.parametrize("D,heads", [(64, 4), (32, 4)])
def test_attention_running_max_rescale(device, D, heads):
    """The tcgen05 kernel takes p against a running row max that it raises
    (rescaling O in tensor memory and the row sums) only when a block's max
    grows past it by more than 2^8.  Scores that climb along the keys
    (s = 0.1 j: +6.4 per 64 keys, above the threshold's 5.55) raise it in
    nearly every block and in each half of a block; one sequence instead
    holds a single key 60 above the rest late in the row, so every earlier
    contribution is scaled by about 2^-86.  Against float64 on the same
    bf16 inputs."""
    rng = np.random.default_rng(17 + D)
    lens = np.array([130, 512, 70, 300, 200, 1], np.int32)
    off, T = _packed(lens)
    H = D * heads
    u = rng.standard_normal(D)
    u /= np.linalg.norm(u)
    qkv = np.zeros((T, 3 * H), np.float32)
    for b, L in enumerate(lens):
        r = slice(off[b], off[b] + L)
        j = np.arange(L, dtype=np.float64)
        score = np.where(j == 250, 60.0, 0.01 * j) if b == 3 else 0.1 * j
        for h in range(heads):
            qkv[r, h * D:(h + 1) * D] = u + 0.01 * rng.standard_normal((L, D))
            qkv[r, H + h * D:H + (h + 1) * D] = (score[:, None] * u +
                                                 0.01 * rng.standard_normal((L, D)))
            qkv[r, 2 * H + h * D:2 * H + (h + 1) * D] = 0.5 * rng.standard_normal((L, D))
    qkv = bf16_bits(qkv)
    ctx = torch.zeros((T, H), dtype=torch.bfloat16, device="cuda")
    device.attention(dev_tensor(qkv), T, dev_tensor(off), dev_tensor(lens), len(lens), 512,
                     heads, D, ctx)
    device.sync()
    got = bits_to_f32(host_bits(ctx)).astype(np.float64)
    q = bits_to_f32(qkv).astype(np.float64)
    assert np.isfinite(got).all()
    for b, L in enumerate(lens):
        r = slice(off[b], off[b] + L)
        for h in range(heads):
            Q = q[r, h * D:(h + 1) * D]
            Kt = q[r, H + h * D:H + (h + 1) * D]
            V = q[r, 2 * H + h * D:2 * H + (h + 1) * D]
            s = Q @ Kt.T
            p = np.exp(s - s.max(1, keepdims=True))
            p /= p.sum(1, keepdims=True)
            want = p @ V
            err = np.abs(got[r, h * D:(h + 1) * D] - want).max()
            assert err <= 1.5e-2 * max(1.0, np.abs(want).max()), (b, h, err)


@pytest.mark.parametrize("cls", [0, 1])
def test_pool_l2(device, port_oracle, cls):
    rng = np.random.default_rng(11 + cls)
    lens = np.array([1, 5, 128, 77, 3], np.int32)
    off, T = _packed(lens)
    H, S = 384, 128
    h = rng.standard_normal((T, H)).astype(np.float32)
    out = torch.empty((len(lens), H), dtype=torch.float32, device="cuda")
    device.pool_l2(dev_tensor(h), dev_tensor(off), dev_tensor(lens), len(lens), H,
                   1 if cls else 0, out)
    device.sync()
    padded = np.zeros((len(lens), S, H), np.float32)
    am = np.zeros((len(lens), S), np.float32)
    for b, L in enumerate(lens):
        padded[b, :L] = h[off[b]:off[b] + L]
        am[b, :L] = 1
    want = port_oracle.pool_rows(padded, am, S, cls)
    got = out.cpu().numpy()
    # double accumulation on both sides; only the L2 sum's order differs
    assert np.abs(got - want).max() <= 2e-7


def test_embed_ln(device, port_oracle):
    rng = np.random.default_rng(21)
    H, S, vocab = 384, 64, 1000
    word = rng.standard_normal((vocab, H)).astype(np.float32)
    pos = rng.standard_normal((S, H)).astype(np.float32)
    typ = rng.standard_normal((2, H)).astype(np.float32)
    g = np.ones(H, np.float32)
    b = np.zeros(H, np.float32)
    lens = np.array([64, 1, 17], np.int32)
    ids = rng.integers(0, vocab, size=(3, S)).astype(np.int32)
    off, T = _packed(lens)
    x = torch.empty((T, H), dtype=torch.float32, device="cuda")
    a = torch.empty((T, H), dtype=torch.bfloat16, device="cuda")
    device.embed_ln(dev_tensor(ids), dev_tensor(off), dev_tensor(lens), 3, S, dev_tensor(word),
                    vocab, dev_tensor(pos), dev_tensor(typ), dev_tensor(g), dev_tensor(b), H, x,
                    a_bf16=a)
    device.sync()
    rows = []
    for bb, L in enumerate(lens):
        for s in range(L):
            rows.append((word[ids[bb, s]] + pos[s]) + typ[0])
    want = port_oracle.layer_norm(np.array(rows, np.float32), g, b)
    got = x.cpu().numpy()
    assert np.abs(got - want).max() <= 2e-5 * np.abs(want).max()
    np.testing.assert_array_equal(host_bits(a), port_oracle.to_bf16(got))


def test_embed_refuses_bad_token(device):
    import nebw
    H, S, vocab = 128, 8, 10
    z = lambda *s: dev_tensor(np.zeros(s, np.float32))  # noqa: E731
    ids = np.full((1, S), 99, np.int32)
    lens = np.array([S], np.int32)
    off = np.array([0, S], np.int32)
    x = torch.empty((S, H), dtype=torch.float32, device="cuda")
    device.embed_ln(dev_tensor(ids), dev_tensor(off), dev_tensor(lens), 1, S, z(vocab, H), vocab,
                    z(S, H), z(2, H), dev_tensor(np.ones(H, np.float32)), z(H), H, x)
    with pytest.raises(nebw.NebwError, match="token id"):
        device.sync()


_SINGLE_CTA_CHILD = r"""
import sys
import numpy as np
import torch
import nebw

inp = np.load(sys.argv[1])
dev = nebw.Device(0, torch_stream=True)
res = {}
for key in sorted({k.rsplit('_', 1)[0] for k in inp.files}):
    A, W, b = inp[key + '_A'], inp[key + '_W'], inp[key + '_b']
    M, K = A.shape
    N = W.shape[1]
    h = dev.stage_weight(W)
    a = torch.from_numpy(A.view(np.int16).copy()).cuda().view(torch.bfloat16)
    bd = torch.from_numpy(b).cuda()
    for act, cd in ((0, 0), (0, 1), (1, 1), (2, 1)):
        c = torch.empty((M, N), dtype=torch.float32 if cd == 0 else torch.bfloat16, device='cuda')
        dev.gemm(h, a, M, K, N, c, bias=bd, act=act, c_dtype=cd)
        dev.sync()
        res[f'{key}_{act}_{cd}'] = c.float().cpu().numpy()
    dev.release_weight(h)
dev.close()
np.savez(sys.argv[2], **res)
"""


def test_gemm_single_cta_kernel_matches_pairs(device, tmp_path):
    """The single-CTA GEMM (128-row tiles; the path for GPUs that cannot
    place CTA pairs, forced here with NEBW_GEMM_CTAS=1 in a child process)
    against the CTA-pair path of this process, every epilogue: fp32 outputs
    within fp32 accumulation-order noise, bf16 outputs within one bf16 ulp."""
    import os
    import subprocess
    import sys
    from pathlib import Path

    rng = np.random.default_rng(23)
    shapes = [(37, 200, 24), (300, 384, 1152), (513, 1024, 4096)]
    inputs = {}
    for M, K, N in shapes:
        key = f"{M}x{K}x{N}"
        inputs[key + "_A"] = bf16_bits(rng.standard_normal((M, K), np.float32))
        inputs[key + "_W"] = rng.standard_normal((K, N), np.float32) * 0.05
        inputs[key + "_b"] = rng.standard_normal(N).astype(np.float32)
    np.savez(tmp_path / "in.npz", **inputs)
    repo = Path(__file__).resolve().parent.parent
    env = dict(os.environ, NEBW_GEMM_CTAS="1",
               PYTHONPATH=os.pathsep.join([str(repo / "npu-embeddings-xdna1_b200"), str(repo)]))
    subprocess.run([sys.executable, "-c", _SINGLE_CTA_CHILD, str(tmp_path / "in.npz"),
                    str(tmp_path / "out.npz")], env=env, check=True, timeout=300)
    single = np.load(tmp_path / "out.npz")
    for M, K, N in shapes:
        key = f"{M}x{K}x{N}"
        h = device.stage_weight(inputs[key + "_W"])
        a = dev_tensor(inputs[key + "_A"])
        bd = dev_tensor(inputs[key + "_b"])
        for act, cd in ((0, 0), (0, 1), (1, 1), (2, 1)):
            c = torch.empty((M, N), dtype=torch.float32 if cd == 0 else torch.bfloat16,
                            device="cuda")
            device.gemm(h, a, M, K, N, c, bias=bd, act=act, c_dtype=cd)
            device.sync()
            got = c.float().cpu().numpy().astype(np.float64)
            ref = single[f"{key}_{act}_{cd}"].astype(np.float64)
            assert np.isfinite(ref).all()
            if cd == 0:
                assert np.abs(got - ref).max() <= 1e-5 * np.abs(ref).max() + 1e-6, (key, act)
            else:
                assert np.all(np.abs(got - ref) <= np.abs(ref) * 2.0 ** -7 + 1e-6), (key, act)
        device.release_weight(h)
