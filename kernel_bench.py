"""Single-kernel timing through the C ABI, for tuning and for profiler runs
(the commands behind the profiles/ summaries; not part of the library).

    python kernel_bench.py gemm --M 16384 --K 1024 --N 4096 --epi gelu8
    python kernel_bench.py attention --B 64 --len 512 --heads 16 --hd 64
    python kernel_bench.py layernorm --M 131072 --H 1024
    python kernel_bench.py encoder --config bge-large --layers 1

Each case runs a few
warm-up launches and then times --iters launches with CUDA events on the
launching stream, printing one JSON line with the per-launch time and the
achieved TFLOP/s or GB/s.  Operand buffers are sized so that, across the
rotation of --copies buffers, the working set exceeds the 126 MB L2.
"""

from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import numpy as np

sys.path.insert(0, str(Path(__file__).resolve().parent / "npu-embeddings-xdna1_b200"))


def _bits(a):
    import torch
    return torch.from_numpy(a.view(np.int16).copy()).cuda().view(torch.bfloat16)


def bench_gemm(dev, M, K, N, epi, iters, copies):
    import torch
    rng = np.random.default_rng(0)
    w = (rng.standard_normal((K, N), np.float32) * 0.02).astype(np.float32)
    h = dev.stage_weight(w)
    bias = torch.randn(N, device="cuda")
    As = [torch.randn(M, K, device="cuda").to(torch.bfloat16) for _ in range(copies)]
    f32 = epi in ("f32", "resid")
    Cs = [torch.empty(M, N, device="cuda", dtype=torch.float32 if f32 else torch.bfloat16)
          for _ in range(copies)]
    act = {"gelu8": 1, "erf": 2}.get(epi, 0)

    def run(i):
        c = Cs[i % copies]
        dev.gemm(h, As[i % copies], M, K, N, c, bias=bias, residual=c if epi == "resid" else None,
                 act=act, c_dtype=0 if f32 else 1, stream=torch.cuda.current_stream())

    for i in range(3):
        run(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(iters):
        run(i)
    e1.record()
    torch.cuda.synchronize()
    dev.sync()
    ms = e0.elapsed_time(e1) / iters
    fl = 2.0 * M * N * K
    return {"kernel": "gemm_tc", "M": M, "K": K, "N": N, "epi": epi, "ms": ms,
            "tflops": fl / ms / 1e9}


def bench_attention(dev, B, L, heads, hd, iters, copies):
    import torch
    H = heads * hd
    lens = np.full(B, L, np.int32)
    off = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    T = int(off[-1])
    qkv = [(torch.randn(T, 3 * H, device="cuda") * 0.5).to(torch.bfloat16) for _ in range(copies)]
    ctx = torch.empty(T, H, device="cuda", dtype=torch.bfloat16)
    off_d = torch.from_numpy(off).cuda()
    len_d = torch.from_numpy(lens).cuda()

    def run(i):
        dev.attention(qkv[i % copies], T, off_d, len_d, B, L, heads, hd, ctx,
                      stream=torch.cuda.current_stream())

    for i in range(3):
        run(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(iters):
        run(i)
    e1.record()
    torch.cuda.synchronize()
    dev.sync()
    ms = e0.elapsed_time(e1) / iters
    fl = 4.0 * B * L * L * H
    return {"kernel": "attention", "B": B, "len": L, "heads": heads, "hd": hd, "ms": ms,
            "tflops": fl / ms / 1e9}


def bench_layernorm(dev, M, H, iters, copies):
    """The encoder's add + LayerNorm: x = LN(x + y) with y the bf16 GEMM
    output, x kept fp32 and the next GEMM's bf16 operand written: 12 bytes
    an element."""
    import torch
    xs = [torch.randn(M, H, device="cuda") for _ in range(copies)]
    ys = [torch.randn(M, H, device="cuda").to(torch.bfloat16) for _ in range(copies)]
    a = torch.empty(M, H, device="cuda", dtype=torch.bfloat16)
    g = torch.ones(H, device="cuda")
    b = torch.zeros(H, device="cuda")

    def run(i):
        dev.layernorm(xs[i % copies], g, b, M, H, y=ys[i % copies], a_bf16=a,
                      stream=torch.cuda.current_stream())

    for i in range(3):
        run(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(iters):
        run(i)
    e1.record()
    torch.cuda.synchronize()
    dev.sync()
    ms = e0.elapsed_time(e1) / iters
    by = M * H * (4 + 2 + 4 + 2)
    return {"kernel": "layernorm", "M": M, "H": H, "ms": ms, "gbs": by / ms / 1e6}


def bench_pool(dev, config, cls, iters):
    """Pooling + L2 over a configuration's packed batch (fp32 hidden rows
    [T, H]): mean reads every row (T x H x 4 bytes), CLS one row a sequence."""
    import torch
    from nebw import synth
    cfg = synth.CONFIGS[config]
    _, _, lens = synth.config_batch(cfg)
    lens = lens.astype(np.int32)
    off = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    T, B, H = int(off[-1]), len(lens), cfg.arch.hidden
    h = torch.randn(T, H, device="cuda")
    off_d = torch.from_numpy(off).cuda()
    len_d = torch.from_numpy(lens).cuda()
    out = torch.empty(B, H, device="cuda")

    def run():
        dev.pool_l2(h, off_d, len_d, B, H, int(cls), out, stream=torch.cuda.current_stream())

    for _ in range(3):
        run()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        run()
    e1.record()
    torch.cuda.synchronize()
    dev.sync()
    ms = e0.elapsed_time(e1) / iters
    by = (B if cls else T) * H * 4 + B * H * 4
    return {"kernel": "pool_l2", "config": config, "cls": bool(cls), "T": T, "B": B, "H": H,
            "ms": ms, "gbs": by / ms / 1e6}


def bench_narrow(dev, M, iters, copies):
    """The standalone fp32 -> bf16 RNE narrow over M elements: 6 bytes each."""
    import torch
    xs = [torch.randn(M, device="cuda") for _ in range(copies)]
    y = torch.empty(M, device="cuda", dtype=torch.bfloat16)

    def run(i):
        dev.narrow_bf16(xs[i % copies], M, y, stream=torch.cuda.current_stream())

    for i in range(3):
        run(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(iters):
        run(i)
    e1.record()
    torch.cuda.synchronize()
    dev.sync()
    ms = e0.elapsed_time(e1) / iters
    return {"kernel": "narrow_bf16", "M": M, "ms": ms, "gbs": M * 6 / ms / 1e6}


def bench_gemm_i8(dev, M, K, N, epi, iters, copies):
    """The int8 GEMM (tcgen05 kind::i8) with the dequantise epilogue: epi
    "f32" fp32 out, "gelu8" dequantise + gelu8, fp32 out, "bf16" bf16 RNE out
    (the int8 encoder pass's QKV form)."""
    import torch
    import nebw
    rng = np.random.default_rng(0)
    h = dev.stage_weight_i8(rng.integers(-127, 128, (K, N), dtype=np.int8))
    ws = torch.rand(N, device="cuda") * 1e-3
    bias = torch.randn(N, device="cuda") * 0.02
    As = [torch.randint(-127, 128, (M, K), dtype=torch.int8, device="cuda") for _ in range(copies)]
    sa = torch.rand(M, device="cuda") * 1e-2
    bf16 = epi == "bf16"
    Cs = [torch.empty(M, N, device="cuda", dtype=torch.bfloat16 if bf16 else torch.float32)
          for _ in range(copies)]
    act = 1 if epi == "gelu8" else 0

    def run(i):
        dev.gemm_i8(h, As[i % copies], sa, M, K, N, ws, Cs[i % copies], bias=bias, act=act,
                    stream=torch.cuda.current_stream(), c_dtype=nebw.BF16 if bf16 else nebw.F32)

    for i in range(3):
        run(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(iters):
        run(i)
    e1.record()
    torch.cuda.synchronize()
    dev.sync()
    ms = e0.elapsed_time(e1) / iters
    ops = 2.0 * M * N * K
    return {"kernel": "gemm_i8", "M": M, "K": K, "N": N, "epi": epi, "ms": ms,
            "tops": ops / (ms / 1e3) / 1e12}


def bench_encoder(dev, config, layers, iters, datapath="bf16", graphs=False, batch=0):
    """Whole passes of a benchmark configuration's batch through a model of
    `layers` layers (the production launch sequence, attention work list
    included), with per-kernel device times from the model's profiler.
    datapath "i8": the same weights written as an int8 pre-tiled container
    (the reference's --dtype i8 form) and run on the int8 datapath.  graphs:
    the passes replayed as CUDA graphs (timed without the per-kernel
    profiler, which launches directly).  batch > 0: the first `batch`
    sequences only (8 GPUs' share of the batch is batch / 8)."""
    import tempfile
    import torch
    import nebw
    from nebw import synth
    cfg = synth.CONFIGS[config]
    ids, _, lens = synth.config_batch(cfg)
    if batch > 0:
        ids, lens = ids[:batch], lens[:batch]
    n = len(lens)
    w = synth.config_weights(cfg, layers=layers if layers > 0 else None)
    if datapath == "i8":
        from nebw.npue import write_bert_container
        with tempfile.TemporaryDirectory() as td:
            path = f"{td}/i8.npue"
            write_bert_container(path, w, max_seq_len=cfg.seq, gemm_layout="pretiled_bf16",
                                 a_dtype="i8", tile=(64, 64), mac=(8, 8), smooth_seed=1)
            m = nebw.Model.from_npue(dev, path)
        m.set_datapath("i8")
    else:
        m = nebw.Model.from_weights(dev, w, max_seq_len=cfg.seq)
    ids_d = torch.from_numpy(np.ascontiguousarray(ids)).cuda()
    lens_d = torch.from_numpy(lens.astype(np.int32)).cuda()
    out = torch.empty(n, m.hidden, device="cuda")
    st = torch.cuda.current_stream()
    m.set_graphs(graphs)

    def run():
        m.encode_into(ids_d, lens_d, out, n, cfg.seq, stream=st)

    for _ in range(3):
        run()
    torch.cuda.synchronize()
    if not graphs:
        m.profile(True)
        m.profile_collect()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        run()
    e1.record()
    torch.cuda.synchronize()
    dev.sync()
    per = {}
    if not graphs:
        per = {k: round(ms / iters, 4) for k, (c, ms) in m.profile_collect().items() if c}
        m.profile(False)
    m.close()
    return {"kernel": "encoder", "config": config, "layers": w.layers, "batch": n,
            "datapath": datapath, "graphs": graphs, "ms": e0.elapsed_time(e1) / iters,
            "kernels_ms": per}


def bench_latency(dev, config, layers, B, seq, iters):
    """Per-request wall time of the host-buffer entry point (nebw_encode: ids
    and lengths copied in, the pass, embeddings copied out) for requests of B
    sequences padded to `seq`, lengths drawn from the configuration's batch,
    with the pass launched kernel by kernel and replayed as a CUDA graph."""
    import time
    import nebw
    from nebw import synth
    cfg = synth.CONFIGS[config]
    ids, _, lens = synth.config_batch(cfg)
    ids = np.ascontiguousarray(ids[:, :seq])
    lens = np.minimum(lens, seq).astype(np.int32)
    w = synth.config_weights(cfg, layers=layers if layers > 0 else None)  # <= 0: every layer
    m = nebw.Model.from_weights(dev, w, max_seq_len=cfg.seq)
    out = {}
    try:
        for graphs in (False, True):
            m.set_graphs(graphs)
            reqs = [(ids[i * B:(i + 1) * B], lens[i * B:(i + 1) * B])
                    for i in range(len(lens) // B)]
            for r in reqs[:3]:
                m.encode(*r)
            t0 = time.perf_counter()
            for i in range(iters):
                m.encode(*reqs[i % len(reqs)])
            out["graphs" if graphs else "direct"] = (time.perf_counter() - t0) / iters * 1e3
    finally:
        m.close()
    return {"kernel": "latency", "config": config, "layers": w.layers, "B": B, "seq": seq,
            "ms_per_request": out}


def main(argv=None):
    import nebw
    ap = argparse.ArgumentParser()
    ap.add_argument("op", choices=["gemm", "gemm_i8", "attention", "layernorm", "encoder",
                                   "latency", "pool", "narrow"])
    ap.add_argument("--cls", type=int, default=0, help="pool: 1 CLS row, 0 masked mean")
    ap.add_argument("--graphs", type=int, default=0, help="encoder: replay the pass as a CUDA graph")
    ap.add_argument("--batch", type=int, default=0, help="encoder: first N sequences (0: all)")
    ap.add_argument("--config", default="bge-large")
    ap.add_argument("--layers", type=int, default=1)
    ap.add_argument("--M", type=int, default=16384)
    ap.add_argument("--K", type=int, default=1024)
    ap.add_argument("--N", type=int, default=4096)
    ap.add_argument("--H", type=int, default=1024)
    ap.add_argument("--B", type=int, default=64)
    ap.add_argument("--len", type=int, default=512)
    ap.add_argument("--heads", type=int, default=16)
    ap.add_argument("--hd", type=int, default=64)
    ap.add_argument("--epi", default="bf16", choices=["bf16", "gelu8", "erf", "f32", "resid"])
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--copies", type=int, default=2)
    ap.add_argument("--attn-kind", type=int, default=1, help="0 mma.sync, 1 tcgen05")
    ap.add_argument("--datapath", default="bf16", choices=["bf16", "i8"],
                    help="encoder: bf16 weights, or an int8 container on the int8 datapath")
    a = ap.parse_args(argv)
    dev = nebw.Device(0, torch_stream=True)
    dev.set_attention_kernel(a.attn_kind)
    if a.op == "gemm":
        r = bench_gemm(dev, a.M, a.K, a.N, a.epi, a.iters, a.copies)
    elif a.op == "gemm_i8":
        r = bench_gemm_i8(dev, a.M, a.K, a.N, a.epi, a.iters, a.copies)
    elif a.op == "attention":
        r = bench_attention(dev, a.B, a.len, a.heads, a.hd, a.iters, a.copies)
    elif a.op == "layernorm":
        r = bench_layernorm(dev, a.M, a.H, a.iters, a.copies)
    elif a.op == "pool":
        r = bench_pool(dev, a.config, a.cls, a.iters)
    elif a.op == "narrow":
        r = bench_narrow(dev, a.M, a.iters, a.copies)
    elif a.op == "latency":
        r = bench_latency(dev, a.config, a.layers, a.B, a.len, a.iters)
    else:
        r = bench_encoder(dev, a.config, a.layers, a.iters, a.datapath, bool(a.graphs), a.batch)
    print(json.dumps(r), flush=True)
    dev.close()


if __name__ == "__main__":
    main()
