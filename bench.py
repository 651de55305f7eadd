#!/usr/bin/env python
"""Benchmark: embeddings/s of the BERT-encoder hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config bge-large]
    python -m torch.distributed.run --nproc-per-node N ... bench.py --gpus N ...
    python bench.py --impl reference ...     # the reference's own CPU path

Workload: bge-large architecture (24 layers, hidden
1024, 16 heads, FFN 4096), random-init N(0, 0.02), a batch of 1024 sequences
padded to 512 with log-normal lengths (median 96, sigma 0.8, clipped to
[8, 512]), CLS pooling + L2.  One step = one encoder pass over the whole
batch.  At N GPUs the batch is sharded by a length-balanced plan (one weight
replica per GPU, no collective on the data path) and the [1024, 1024] fp32
embeddings are gathered to rank 0 with NCCL; the total batch is fixed, so
scaling is strong.

Reported, on one JSON line from rank 0:
  value       embeddings/s with inputs resident in HBM (CUDA events on the
              launching stream, max over ranks)
  e2e         the same through the public C ABI with host buffers: H2D of the
              ids and lengths, the pass, the gather, D2H of the embeddings
  roofline    the GEMM family (tcgen05 kernel): algorithmic FLOPs / measured
              device time per launch, against MEASURED_PEAKS.json
  kernels     per-kernel-kind device time, share and roofline
  cpu_baseline  the reference's own host-CPU path (oracle/_ref, built from
              the reference tree) -- or the oracle port where it is absent --
              on a bounded sample of the same batch, on this host's cores
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
PKG = REPO / "npu-embeddings-xdna1_b200"
sys.path.insert(0, str(PKG))
sys.path.insert(0, str(REPO))

from nebw import synth  # noqa: E402

METRIC = "embeddings/sec at bge-large seq512"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
PROFILE_TRAFFIC = REPO / "profiles" / "traffic.json"


# ---------------------------------------------------------------------------
# workload arithmetic
# ---------------------------------------------------------------------------

def gemm_flops_per_token(a: synth.Arch) -> float:
    """QKV + attention-out + FFN-up (2F wide for the gated families) + FFN-down."""
    H, F = a.hidden, a.ffn
    FW = 2 * F if a.gated else F
    return 2.0 * a.layers * (3 * H * H + H * H + H * FW + F * H)


def metric_for(cfg) -> str:
    """The headline metric (bge-large) or the same metric named for another
    configuration."""
    return METRIC if cfg.key == "bge-large" else f"embeddings/sec at {cfg.key} seq{cfg.seq}"


def attn_flops(a: synth.Arch, lens) -> float:
    lens = np.asarray(lens, np.float64)
    return float(a.layers * 4.0 * (lens ** 2).sum() * a.hidden)


def seq_flops(a: synth.Arch, lens) -> np.ndarray:
    lens = np.asarray(lens, np.float64)
    return gemm_flops_per_token(a) * lens + a.layers * 4.0 * lens ** 2 * a.hidden



def load_peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {k: float(d[k]) for k in FALLBACK_PEAKS if k in d}, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


# ---------------------------------------------------------------------------
# clocks
# ---------------------------------------------------------------------------

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus):
        self.gpus = set(gpus)
        self.rows = []
        self.proc = None
        self.t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.t = threading.Thread(target=self._read, daemon=True)
        self.t.start()

    def _read(self):
        for line in self.proc.stdout:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9:
                self.rows.append(parts)

    def stop(self):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.t:
            self.t.join(timeout=5)

    def summary(self):
        rows = [r for r in self.rows if r[0].isdigit() and int(r[0]) in self.gpus]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i] == "Active"})
        pw = [float(r[3]) for r in rows if r[3].replace(".", "").isdigit()]
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "power_w_max": max(pw) if pw else None, "samples": len(rows)}


# ---------------------------------------------------------------------------
# ranks (N > 1): the data path is libnebw's own NCCL communicator
# ---------------------------------------------------------------------------

class Ranks:
    """One process per GPU.  torch.distributed runs over gloo, on the host
    only: barriers, the max of the per-rank timings, and handing rank 0's
    communicator id to the others.  The sharded pass and the gather of the
    embeddings go through libnebw (nebw_comm_init_rank,
    nebw_encode_shard_gather / nebw_encode_sharded over NCCL)."""

    def __init__(self, dev, world: int, rank: int):
        import torch.distributed as dist

        import nebw
        self.world, self.rank, self.dist = world, rank, dist
        self.comm = None
        if world > 1:
            from datetime import timedelta
            dist.init_process_group("gloo", timeout=timedelta(seconds=300))
            box = [nebw.comm_unique_id() if rank == 0 else None]
            dist.broadcast_object_list(box, src=0)
            self.comm = nebw.Comm.init_rank(dev, world, rank, box[0], timeout_s=120.0)

    def barrier(self):
        import torch
        if self.comm is not None:
            self.comm.sync(stream=torch.cuda.current_stream())
        if self.world > 1:
            self.dist.barrier()
        torch.cuda.synchronize()

    def max(self, x: float) -> float:
        import torch
        t = torch.tensor([x], dtype=torch.float64)
        if self.world > 1:
            self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def all_gather(self, row):
        import torch
        t = torch.tensor([row], dtype=torch.float64)
        if self.world == 1:
            return [t]
        out = [torch.zeros_like(t) for _ in range(self.world)]
        self.dist.all_gather(out, t)
        return out

    def close(self):
        if self.comm is not None:
            self.comm.close()
            self.comm = None
        if self.world > 1:
            self.dist.barrier()
            self.dist.destroy_process_group()


def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform
    return platform.processor() or "unknown"


# ---------------------------------------------------------------------------
# the CPU arms
# ---------------------------------------------------------------------------

def cpu_reference_setup(cfg: synth.Config, w, workdir):
    """(runner, kind, threads): runner(ids, mask) -> embeddings."""
    from oracle.oracle import REF_LIB, PortOracle, RefOracle, host_threads
    threads = host_threads()
    if REF_LIB.exists():
        from nebw.npue import write_bert_container
        path = Path(workdir) / "bench_ref.npue"
        write_bert_container(path, w, max_seq_len=cfg.seq)
        sess = RefOracle().session(path, cfg.seq, threads)
        return (lambda ids, mask: sess.run(ids, mask, w.hidden)), "reference", threads
    port = PortOracle()
    return (lambda ids, mask: port.encode(w, ids, mask, threads=threads)), "port", threads


def pick_sample(lens, n):
    """n row indices spread over the batch, including the longest and the
    shortest row (the host path pads every row to seq, so cost is flat)."""
    idx = {int(np.argmax(lens)), int(np.argmin(lens))}
    for i in np.linspace(0, len(lens) - 1, num=max(n, 2)).astype(int):
        if len(idx) >= n:
            break
        idx.add(int(i))
    return np.array(sorted(idx))[:n]


CPU_METHOD = ("the reference's own host path (one lane, every host thread), one request of "
              "p sequences at a time, each padded to the configuration's seq as the reference "
              "pads every request; p = ceil(8 * threads / seq) so that its 8-row GEMM blocks "
              "occupy every thread; one untimed request first, then the timed sequences; "
              "sequences/s = timed sequences / their wall time")


def cpu_per_request(cfg, threads: int) -> int:
    """p: sequences per reference request -- enough 8-row GEMM blocks
    (conv_host.hpp:154-160) to occupy every host thread."""
    return int(max(1, min(cfg.batch, -(-threads * 8 // cfg.seq))))


def cpu_host_facts(threads: int) -> dict:
    return {"cores": threads, "nproc": os.cpu_count(), "cpu_model": cpu_model(),
            "method": CPU_METHOD}


def run_cpu_baseline(cfg, w, ids, mask, lens, n_timed: int = 8):
    """The CPU baseline beside the GPU line: CPU_METHOD with n_timed >= 8
    sequences spread over the batch (the longest and shortest included)."""
    with tempfile.TemporaryDirectory() as td:
        run, kind, threads = cpu_reference_setup(cfg, w, td)
        p = cpu_per_request(cfg, threads)
        sample = pick_sample(lens, max(n_timed, p))
        t0 = time.perf_counter()
        run(ids[sample[:p]], mask[sample[:p]])  # untimed: builds the reference's weight cache
        t_warm = time.perf_counter() - t0
        t0 = time.perf_counter()
        for i in range(0, len(sample), p):
            r = sample[i:i + p]
            run(ids[r], mask[r])
        el = time.perf_counter() - t0
    return {"value": len(sample) / el, "unit": "embeddings/s", "kind": kind,
            **cpu_host_facts(threads),
            "sample": f"{len(sample)} sequences of the {cfg.batch}-row batch in requests of {p}, "
                      f"each padded to seq {cfg.seq}; {el:.1f} s timed after a {t_warm:.1f} s "
                      f"untimed request",
            "full_batch_s_extrapolated": cfg.batch * el / len(sample)}


def reference_arm(args, cfg):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    w = synth.config_weights(cfg)
    ids, mask, lens = synth.config_batch(cfg)
    with tempfile.TemporaryDirectory() as td:
        run, kind, threads = cpu_reference_setup(cfg, w, td)
        # one reference request of p sequences per step (CPU_METHOD)
        per_step = cpu_per_request(cfg, threads)
        order = pick_sample(lens, min(len(lens), per_step * (args.warmup + args.steps)))

        def rows(i):
            return np.array([order[(i * per_step + k) % len(order)] for k in range(per_step)])

        for i in range(args.warmup):
            r = rows(i)
            run(ids[r], mask[r])
        t0 = time.perf_counter()
        for i in range(args.steps):
            r = rows(args.warmup + i)
            run(ids[r], mask[r])
        el = time.perf_counter() - t0
    value = args.steps * per_step / el
    line = {
        "impl": "reference", "metric": metric_for(cfg), "value": value, "unit": "embeddings/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * el / args.steps, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"{cfg.key}: batch {cfg.batch} x seq {cfg.seq}, "
                               f"{cfg.arch.layers}L/{cfg.arch.hidden}H, lengths {cfg.lengths}",
                   "global_batch": cfg.batch, "seq_len": cfg.seq, "parallelism": "host threads",
                   "step": f"{per_step} sequence(s) of the batch per step (bounded sample)"},
        "cpu_baseline": {"value": value, "unit": "embeddings/s", "kind": kind,
                         **cpu_host_facts(threads),
                         "sample": f"{args.warmup} untimed + {args.steps} timed requests of "
                                   f"{per_step} sequence(s) of the batch, padded to {cfg.seq} "
                                   f"({args.steps * per_step} timed sequences)"},
        "e2e": {"value": value, "unit": "embeddings/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# the GPU arm
# ---------------------------------------------------------------------------

def gpu_arm(args, cfg):
    import torch

    import nebw

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE {world}")
    torch.cuda.set_device(local)

    arch = cfg.arch
    w = synth.config_weights(cfg)
    ids, mask, lens = synth.config_batch(cfg)
    B, S, H = cfg.batch, cfg.seq, arch.hidden
    dev = nebw.Device(local)
    ranks = Ranks(dev, world, rank)
    owner, counts = nebw.shard_plan(lens, world)
    mine = np.nonzero(owner == rank)[0]
    b_r = len(mine)
    T_r = int(lens[mine].sum())

    dev.set_attention_kernel(dev.ATTN_TCGEN05 if args.attention == "tcgen05" else dev.ATTN_MMA)
    model = nebw.Model.from_weights(dev, w, max_seq_len=S)
    launches_per_step = model.launch_count(S) + (1 if world > 1 and rank == 0 else 0)
    stream = torch.cuda.current_stream()

    ids_h = torch.from_numpy(np.ascontiguousarray(ids[mine])).pin_memory()
    lens_h = torch.from_numpy(np.ascontiguousarray(lens[mine])).pin_memory()
    ids_d = ids_h.cuda()
    lens_d = lens_h.cuda()
    out_d = torch.zeros((B if rank == 0 else b_r, H), dtype=torch.float32, device="cuda")
    order_d = torch.from_numpy(nebw.shard_order(owner, world)).cuda() if rank == 0 else None
    out_h = np.empty((B, H), np.float32)

    def step():
        if world == 1:
            model.encode_into(ids_d, lens_d, out_d, b_r, S, stream=stream)
        else:  # this rank's shard, then the gather to rank 0 in request order
            ranks.comm.encode_shard_gather(model, ids_d, lens_d, b_r, S, counts, order_d,
                                           out_d if rank == 0 else None, stream=stream)

    # ---- device-resident throughput --------------------------------------
    # each pass replayed as a CUDA graph (nebw_model_set_graphs: the same
    # kernels, one launch; bit-identical rows) unless --no-graphs
    model.set_graphs(args.graphs)
    for _ in range(args.warmup):
        step()
    ranks.barrier()
    sampler = ClockSampler(range(world)) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.6)
    ranks.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    ranks.barrier()
    if sampler:
        sampler.stop()
    ms = e0.elapsed_time(e1)
    dev.sync()
    ms_max = ranks.max(ms)
    # the per-kernel split: the same steps again with a CUDA event before
    # every kernel (the profiler launches the kernels one by one)
    model.profile(True)
    model.profile_collect()
    ranks.barrier()
    for _ in range(args.steps):
        step()
    ranks.barrier()
    model.profile(False)
    prof = model.profile_collect()
    dev.sync()

    # ---- end to end through the public API with host buffers ------------
    # N = 1: nebw_encode (H2D of ids and lengths, the pass, D2H); N > 1:
    # nebw_encode_sharded (every rank is handed the whole batch, copies its
    # shard in, encodes, gathers to rank 0, which copies [B, H] out)
    def step_e2e():
        if world == 1:
            model.encode_into(ids, lens, out_h, B, S, host=True)
            return out_h
        return ranks.comm.encode_sharded(model, ids, lens, out_h if rank == 0 else None)

    for _ in range(max(1, args.warmup)):
        res = step_e2e()
    ranks.barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        res = step_e2e()
    ranks.barrier()
    e2e_s = ranks.max(time.perf_counter() - t0)

    # N > 1: rank 0 re-encodes a fixed subset of rows -- most of them owned
    # by other ranks -- on its own GPU alone; rows are independent passes, so
    # the gathered rows must match bit for bit
    rows_match = None
    if world > 1 and rank == 0:
        sub = np.unique(np.concatenate([np.linspace(0, B - 1, 48).astype(int),
                                        [int(np.argmax(lens)), int(np.argmin(lens))]]))
        alone = model.encode(ids[sub], lens[sub])
        rows_match = {"value": bool(np.array_equal(alone, res[sub])), "rows": int(len(sub)),
                      "rows_on_other_ranks": int((owner[sub] != 0).sum())}

    # per-rank profile -> the slowest rank's numbers are the ones reported
    all_prof = ranks.all_gather([prof[k][1] for k in model.KERNEL_KINDS])
    all_tok = ranks.all_gather([float(T_r), float((lens[mine].astype(np.float64) ** 2).sum())])

    ok = res is not None and bool(np.isfinite(res).all()) if rank == 0 else True

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = run_cpu_baseline(cfg, w, ids, mask, lens)

    if rank == 0:
        peaks, peak_src = load_peaks()
        slow = int(np.argmax([p.sum().item() for p in all_prof]))
        pms = dict(zip(model.KERNEL_KINDS, all_prof[slow][0].tolist()))
        T_s, L2_s = all_tok[slow][0].tolist()
        steps = args.steps
        Hf, F, L = float(H), float(arch.ffn), arch.layers
        FW = 2.0 * F if arch.gated else F  # FFN-up width ([up | gate] for the gated families)
        gemm_fl = {"gemm_qkv": 2 * T_s * Hf * 3 * Hf * L, "gemm_ao": 2 * T_s * Hf * Hf * L,
                   "gemm_up": 2 * T_s * Hf * FW * L, "gemm_down": 2 * T_s * F * Hf * L}
        gemm_ms = sum(pms[k] for k in gemm_fl) / steps
        gemm_tflops = sum(gemm_fl.values()) / (gemm_ms / 1e3) / 1e12
        peak_t = peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"])
        total_prof_ms = sum(pms.values()) / steps
        kernels = {}
        for k in model.KERNEL_KINDS:
            kernels[k] = {"ms_per_step": pms[k] / steps,
                          "share": pms[k] / steps / total_prof_ms if total_prof_ms else None}
        for k, fl in gemm_fl.items():
            kernels[k]["tflops"] = fl / (pms[k] / steps / 1e3) / 1e12
            kernels[k]["frac_of_peak"] = kernels[k]["tflops"] / peak_t
        att_fl = 4.0 * L2_s * Hf * L
        kernels["attention"]["tflops"] = att_fl / (pms["attention"] / steps / 1e3) / 1e12
        kernels["attention"]["frac_of_peak"] = kernels["attention"]["tflops"] / peak_t
        # read x (fp32) and y (bf16), write x (fp32) and the bf16 copy: 12 B/element,
        # 2 per layer
        ln_bytes = T_s * Hf * (4 + 2 + 4 + 2) * 2 * L
        kernels["layernorm"]["gbs"] = ln_bytes / (pms["layernorm"] / steps / 1e3) / 1e9
        kernels["layernorm"]["frac_of_peak"] = kernels["layernorm"]["gbs"] / peaks["hbm_gbs"]
        # the dominant kernel: the FFN-up GEMM (T x 1024 -> 4096, bias + gelu8, bf16 out)
        up_ms = pms["gemm_up"] / (L * steps)
        up_flops = 2.0 * T_s * Hf * FW
        up_bytes = T_s * Hf * 2 + Hf * FW * 2 + T_s * FW * 2  # A + W + C, algorithmic
        traffic = None
        if PROFILE_TRAFFIC.exists() and cfg.key == "bge-large":
            # one ncu capture of this kernel at M = m_cap, scaled to M = T: the
            # activation and output bytes grow with M, the weight bytes do not
            tr = json.loads(PROFILE_TRAFFIC.read_text())["gemm_up"]
            s = T_s / tr["m"]
            traffic = (tr["weight_bytes"] + (tr["dram_read"] - tr["weight_bytes"]) * s
                       + tr["dram_write"] * s)
        n_gemm_launches = 4 * L * steps
        value = B * steps / (ms_max / 1e3)
        e2e = B * steps / e2e_s
        all_flops = float(seq_flops(arch, lens).sum())
        line = {
            "metric": metric_for(cfg), "value": value, "unit": "embeddings/s", "n_gpus": world,
            "steps": steps, "warmup": args.warmup, "ms_per_step": ms_max / steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": f"{cfg.key}: {arch.name} architecture ({arch.layers}L, hidden "
                                   f"{arch.hidden}, {arch.heads} heads, FFN {arch.ffn}"
                                   + (f", {arch.gated} over a {2 * arch.ffn}-wide FFN-up, rotary "
                                      "positions" if arch.gated else "")
                                   + f"), random-init N(0,0.02); batch {B} x seq {S}, lengths "
                                   f"{cfg.lengths} clipped [8,{S}]; "
                                   f"{'CLS' if cfg.cls_pool else 'mean'} pooling + L2",
                       "global_batch": B, "seq_len": S, "real_tokens": int(lens.sum()),
                       "parallelism": f"dp{world} (libnebw: length-balanced shards, "
                                      "NCCL gather to rank 0)" if world > 1 else "single GPU",
                       "l2": "no flush: every step streams the 0.6 GB bf16 weights and GBs of "
                             "activations, far above the 126 MB L2",
                       "graphs": bool(args.graphs),
                       "timing": ("timed steps replay each pass as a CUDA graph "
                                  "(nebw_model_set_graphs)" if args.graphs else
                                  "timed steps launch kernel by kernel") +
                                 "; the per-kernel split and the roofline figures come from a "
                                 "second run of the same steps with a CUDA event on the "
                                 "launching stream before every kernel"},
            "e2e": {"value": e2e, "unit": "embeddings/s",
                    "h2d_bytes_per_step": int(B * S * 4 + B * 4),
                    "d2h_bytes_per_step": int(B * H * 4),
                    "api": "nebw_encode" if world == 1 else "nebw_encode_sharded (every rank)",
                    "timer": "wall clock, synchronous per step, max over ranks"},
            "gpu_launches": int(launches_per_step * steps * world),
            "roofline": {"kernel": (f"gemm_tc<256, {arch.gated}> FFN-up (T x {H} -> {int(FW)}, "
                                    f"{arch.gated} epilogue -> {int(F)})" if arch.gated else
                                    f"gemm_tc<256, gelu8> FFN-up (T x {H} -> {int(F)})")
                                   + ", the largest share",
                         "bound": "tensor", "achieved": up_flops / (up_ms / 1e3) / 1e12,
                         "peak": peak_t, "unit": "TFLOP/s",
                         "frac": up_flops / (up_ms / 1e3) / 1e12 / peak_t,
                         "peak_source": f"{peak_src} bf16 dense, sustained (timed inside a long step)",
                         "traffic": traffic, "algorithmic_bytes": up_bytes,
                         "flops_per_launch": up_flops, "ms_per_launch": up_ms,
                         "launches": L * steps},
            "roofline_gemm_family": {"kernel": "gemm_tc QKV/AO/UP/DOWN, launch-weighted",
                                     "achieved": gemm_tflops, "peak": peak_t, "unit": "TFLOP/s",
                                     "frac": gemm_tflops / peak_t, "launches": n_gemm_launches,
                                     "flops_per_step": sum(gemm_fl.values())},
            "end_to_end_frac": {"real_token_tflops": all_flops / (ms_max / steps / 1e3) / 1e12,
                                "frac": all_flops / (ms_max / steps / 1e3) / 1e12 / (peak_t * world),
                                "padded_equivalent_tflops": float(seq_flops(arch, np.full(B, S)).sum())
                                / (ms_max / steps / 1e3) / 1e12},
            "kernels": kernels,
            "outputs_finite": ok,
        }
        if world > 1:
            line["collective"] = {
                "what": "gather of the pooled [b_r, H] fp32 rows to rank 0 (ncclSend / ncclRecv "
                        "in one group) + a request-order scatter kernel on rank 0, inside "
                        "nebw_encode_shard_gather",
                "bytes_per_step": int(B * H * 4), "nranks": world,
                "counts": [int(c) for c in counts]}
            line["rows_match_single_gpu"] = rows_match["value"]
            line["rows_match_detail"] = rows_match
        if sampler:
            line["clocks"] = sampler.summary()
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)

    model.close()
    ranks.close()
    dev.close()
    return 0


# ---------------------------------------------------------------------------
# configuration 5: vit-base-patch16-224 (a secondary workload, --config vit-base)
# ---------------------------------------------------------------------------

METRIC_VIT = "images/sec at vit-base-patch16-224 (CLS row)"


def vit_flops_per_image(a: synth.VitArch) -> float:
    """Patch GEMM + L x (the four GEMMs over n_pos rows + QK^T and PV)."""
    H, F, S = a.hidden, a.ffn, a.n_pos
    return (2.0 * a.n_patches * a.channels * a.patch_size ** 2 * H
            + a.layers * (2.0 * S * (4 * H * H + 2 * H * F) + 4.0 * S * S * H))


def vit_cpu_setup(cfg, w, workdir):
    """(runner, kind, threads): runner(images) -> CLS rows."""
    from oracle.oracle import REF_LIB, PortOracle, RefOracle, host_threads
    threads = host_threads()
    if REF_LIB.exists():
        from nebw.npue import write_vit_container
        path = Path(workdir) / "bench_ref_vit.npue"
        write_vit_container(path, w)
        sess = RefOracle().vit_session(path, threads)
        return (lambda imgs: sess.run(imgs, w.hidden)), "reference", threads
    port = PortOracle()
    return (lambda imgs: port.vit_encode(w, imgs, threads=threads)), "port", threads


def vit_cpu_baseline(cfg, w, images, budget_s=15.0):
    with tempfile.TemporaryDirectory() as td:
        run, kind, threads = vit_cpu_setup(cfg, w, td)
        t0 = time.perf_counter()
        run(images[:1])
        t1 = time.perf_counter() - t0
        t0 = time.perf_counter()
        run(images[1:2])
        per = time.perf_counter() - t0
        n = int(max(1, min(16, budget_s // max(per, 1e-3))))
        t0 = time.perf_counter()
        run(images[2:2 + n])
        el = time.perf_counter() - t0 + per
    return {"value": (n + 1) / el, "unit": "images/s", "kind": kind, **cpu_host_facts(threads),
            "sample": f"{n + 1} images of the {cfg.batch}-image batch, {el:.1f} s timed after a "
                      f"{t1:.1f} s warm-up (one image at a time, as VitEncoder::run takes them)",
            "full_batch_s_extrapolated": cfg.batch * el / (n + 1)}


def vit_reference_arm(args, cfg):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    w = synth.vit_config_weights(cfg)
    per_step = 2
    images = synth.vit_config_images(cfg, n=per_step * (args.warmup + args.steps))
    with tempfile.TemporaryDirectory() as td:
        run, kind, threads = vit_cpu_setup(cfg, w, td)
        for i in range(args.warmup):
            run(images[i * per_step:(i + 1) * per_step])
        t0 = time.perf_counter()
        for i in range(args.steps):
            j = args.warmup + i
            run(images[j * per_step:(j + 1) * per_step])
        el = time.perf_counter() - t0
    value = args.steps * per_step / el
    print(json.dumps({
        "impl": "reference", "metric": METRIC_VIT, "value": value, "unit": "images/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * el / args.steps, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"{cfg.key}: batch {cfg.batch} images 3x224x224",
                   "global_batch": cfg.batch, "parallelism": "host threads",
                   "step": f"{per_step} images of the batch per step (bounded sample)"},
        "cpu_baseline": {"value": value, "unit": "images/s", "kind": kind, **cpu_host_facts(threads),
                         "sample": f"{args.warmup} warm + {args.steps} timed steps of "
                                   f"{per_step} images"},
        "e2e": {"value": value, "unit": "images/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }), flush=True)
    return 0


def vit_arm(args, cfg):
    import torch

    import nebw

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE {world}")
    torch.cuda.set_device(local)
    arch = cfg.arch
    B, H = cfg.batch, arch.hidden
    w = synth.vit_config_weights(cfg)
    images = synth.vit_config_images(cfg)
    # every image costs the same: contiguous equal shards, gathered in order
    per = -(-B // world)
    bounds = [(min(B, r * per), min(B, (r + 1) * per)) for r in range(world)]
    counts = np.array([hi - lo for lo, hi in bounds], np.int32)
    lo, hi = bounds[rank]
    n_r = hi - lo
    dev = nebw.Device(local)
    ranks = Ranks(dev, world, rank)
    dev.set_attention_kernel(dev.ATTN_TCGEN05 if args.attention == "tcgen05" else dev.ATTN_MMA)
    model = nebw.VitModel.from_weights(dev, w)
    launches_per_step = model.launch_count()
    stream = torch.cuda.current_stream()
    img_h = torch.from_numpy(np.ascontiguousarray(images[lo:hi])).pin_memory()
    img_d = img_h.cuda()
    out_d = torch.zeros((max(n_r, 1), H), dtype=torch.float32, device="cuda")
    gather_d = torch.zeros((B, H), dtype=torch.float32, device="cuda") if rank == 0 else None
    out_h = torch.empty((B, H), dtype=torch.float32).pin_memory()

    def step():
        model.encode_into(img_d, out_d, n_r, stream=stream)
        if world > 1:  # libnebw's NCCL gather of the CLS rows, rank order = image order
            ranks.comm.gather_rows(out_d, counts, H, gather_d, 0, stream=stream)

    for _ in range(args.warmup):
        step()
    ranks.barrier()
    sampler = ClockSampler(range(world)) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.6)
    model.profile(True)
    ranks.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    ranks.barrier()
    if sampler:
        sampler.stop()
    model.profile(False)
    prof = model.profile_collect()
    ms_max = ranks.max(e0.elapsed_time(e1))

    def step_e2e():
        if world == 1:
            model.encode_into(img_h, out_h, n_r, host=True)   # nebw_vit_encode: H2D, pass, D2H
            return out_h[:n_r].numpy()
        img_d.copy_(img_h, non_blocking=True)
        model.encode_into(img_d, out_d, n_r, stream=stream)
        ranks.comm.gather_rows(out_d, counts, H, gather_d, 0, stream=stream)
        if rank == 0:
            out_h.copy_(gather_d, non_blocking=True)
        ranks.comm.sync(stream=stream)
        return out_h.numpy() if rank == 0 else None

    for _ in range(max(1, args.warmup)):
        res = step_e2e()
    ranks.barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        res = step_e2e()
    ranks.barrier()
    e2e_s = ranks.max(time.perf_counter() - t0)
    all_prof = ranks.all_gather([prof[k][1] for k in model.KERNEL_KINDS])
    ok = bool(np.isfinite(res).all()) if rank == 0 else True
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = vit_cpu_baseline(cfg, w, images)

    if rank == 0:
        peaks, peak_src = load_peaks()
        peak_t = peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"])
        slow = int(np.argmax([p.sum().item() for p in all_prof]))
        pms = dict(zip(model.KERNEL_KINDS, all_prof[slow][0].tolist()))
        steps = args.steps
        R = float(n_r * arch.n_pos)
        Hf, F, L = float(H), float(arch.ffn), arch.layers
        gemm_fl = {"gemm_qkv": 2 * R * Hf * 3 * Hf * L, "gemm_ao": 2 * R * Hf * Hf * L,
                   "gemm_up": 2 * R * Hf * F * L, "gemm_down": 2 * R * F * Hf * L}
        total_ms = sum(pms.values()) / steps
        kernels = {k: {"ms_per_step": pms[k] / steps,
                       "share": pms[k] / steps / total_ms if total_ms else None}
                   for k in model.KERNEL_KINDS}
        for k, fl in gemm_fl.items():
            kernels[k]["tflops"] = fl / (pms[k] / steps / 1e3) / 1e12
            kernels[k]["frac_of_peak"] = kernels[k]["tflops"] / peak_t
        att_fl = 4.0 * n_r * arch.n_pos ** 2 * Hf * L
        kernels["attention"]["tflops"] = att_fl / (pms["attention"] / steps / 1e3) / 1e12
        kernels["attention"]["frac_of_peak"] = kernels["attention"]["tflops"] / peak_t
        # the first LN1 reads x and writes the bf16 operand (6 B/element); every
        # later site reads x and y, writes x and the operand (12 B/element)
        ln_bytes = R * Hf * (6 + 12 * (2 * L - 1))
        kernels["layernorm"]["gbs"] = ln_bytes / (pms["layernorm"] / steps / 1e3) / 1e9
        kernels["layernorm"]["frac_of_peak"] = kernels["layernorm"]["gbs"] / peaks["hbm_gbs"]
        up_ms = pms["gemm_up"] / (L * steps)
        up_flops = 2.0 * R * Hf * F
        up_traffic = None
        if PROFILE_TRAFFIC.exists():
            tr = json.loads(PROFILE_TRAFFIC.read_text()).get("vit_gemm_up")
            if tr:  # one ncu capture at M = m rows, scaled to M = R as for bge-large
                sc = R / tr["m"]
                up_traffic = (tr["weight_bytes"] + (tr["dram_read"] - tr["weight_bytes"]) * sc
                              + tr["dram_write"] * sc)
        # the profiler's kinds under their ViT names: im2col is timed as the
        # packing step, the patch GEMM + [cls; pe] + pos + LN1 of layer 0 as
        # the embedding step
        kernels["im2col"] = kernels.pop("pack")
        kernels["patch_embed_ln"] = kernels.pop("embed_ln")
        gemm_ms = sum(pms[k] for k in gemm_fl) / steps
        per_img = vit_flops_per_image(arch)
        line = {
            "metric": METRIC_VIT, "value": B * steps / (ms_max / 1e3), "unit": "images/s",
            "n_gpus": world, "steps": steps, "warmup": args.warmup,
            "ms_per_step": ms_max / steps, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": f"{cfg.key}: {arch.name} architecture ({arch.layers}L, hidden "
                                   f"{H}, {arch.heads} heads, FFN {arch.ffn}, pre-LN, 16x16 patch "
                                   f"embedding, {arch.n_pos} positions), random-init N(0,0.02); "
                                   f"batch {B} images 3x224x224 fp32 uniform [-1,1]; CLS row",
                       "global_batch": B, "seq_len": arch.n_pos,
                       "parallelism": f"dp{world} (equal image shards, libnebw NCCL gather "
                                      "to rank 0)" if world > 1 else "single GPU",
                       "l2": "no flush: every step streams 1.2 GB of images and GBs of "
                             "activations, far above the 126 MB L2"},
            "e2e": {"value": B * steps / e2e_s, "unit": "images/s",
                    "h2d_bytes_per_step": int(n_r * arch.channels * arch.image_size ** 2 * 4),
                    "d2h_bytes_per_step": int(B * H * 4),
                    "timer": "wall clock, synchronous per step, max over ranks"},
            "gpu_launches": int(launches_per_step * steps * world),
            "roofline": {"kernel": "gemm_tc<256, gelu-erf> FFN-up (R x 768 -> 3072)",
                         "bound": "tensor", "achieved": up_flops / (up_ms / 1e3) / 1e12,
                         "peak": peak_t, "unit": "TFLOP/s",
                         "frac": up_flops / (up_ms / 1e3) / 1e12 / peak_t,
                         "peak_source": f"{peak_src} bf16 dense, sustained",
                         "traffic": up_traffic, "algorithmic_bytes": R * Hf * 2 + Hf * F * 2 + R * F * 2,
                         "flops_per_launch": up_flops, "ms_per_launch": up_ms},
            "roofline_gemm_family": {"achieved": sum(gemm_fl.values()) / (gemm_ms / 1e3) / 1e12,
                                     "peak": peak_t, "unit": "TFLOP/s",
                                     "frac": sum(gemm_fl.values()) / (gemm_ms / 1e3) / 1e12 / peak_t},
            "end_to_end_frac": {"tflops": B * per_img / (ms_max / steps / 1e3) / 1e12,
                                "frac": B * per_img / (ms_max / steps / 1e3) / 1e12 / (peak_t * world)},
            "kernels": kernels,
            "outputs_finite": ok,
        }
        if world > 1:
            line["collective"] = {
                "what": "gather of the [n_r, H] fp32 CLS rows to rank 0 (ncclSend / ncclRecv "
                        "in one group, nebw_gather_rows)",
                "bytes_per_step": int(B * H * 4), "nranks": world,
                "counts": [int(c) for c in counts]}
        if sampler:
            line["clocks"] = sampler.summary()
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)

    model.close()
    ranks.close()
    dev.close()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["nebw", "reference"], default="nebw")
    ap.add_argument("--config", default="bge-large",
                    choices=sorted(synth.CONFIGS) + sorted(synth.VIT_CONFIGS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--graphs", action=argparse.BooleanOptionalAction, default=True,
                    help="replay each pass as a CUDA graph (BERT configurations)")
    ap.add_argument("--attention", choices=["mma", "tcgen05"], default="tcgen05",
                    help="attention kernel for head_dim 64")
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.config in synth.VIT_CONFIGS:
        cfg = synth.VIT_CONFIGS[args.config]
        return vit_reference_arm(args, cfg) if args.impl == "reference" else vit_arm(args, cfg)
    cfg = synth.CONFIGS[args.config]
    if args.impl == "reference":
        return reference_arm(args, cfg)
    return gpu_arm(args, cfg)


if __name__ == "__main__":
    sys.exit(main())
