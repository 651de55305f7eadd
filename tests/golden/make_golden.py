"""Generate the golden fixtures in this directory from the reference itself.

    python tests/golden/make_golden.py            (needs oracle/_ref built)

Each fixture is the output of the reference's OWN host-CPU encoder path --
runtime/src/encoders/bert_encoder.cpp + pool.cpp + model.cpp compiled from the
reference tree (oracle/Makefile `ref`) and driven through
EmbedService::chunk's call sequence (oracle/ref_driver.cpp) -- on seeded
synthetic weights and tokens of a benchmark configuration.  The weights are
not stored: they are regenerated from the recorded seed by nebw.synth, and a
fingerprint of them is stored so a drift in the generator is caught.

Fixtures (rows sampled from each configuration's synthetic batch: the
shortest and longest rows, the first and last row index, and rows spread
evenly over the sorted lengths, so the tail of a skewed length distribution
is sampled as well as its median):
  minilm_c1.npz      all-MiniLM-L6-v2 arch, the full 32 x 128 batch, mean pool
  bge_small_c2.npz   bge-small arch, 32 rows at seq 512, CLS pool
  bge_base_c3.npz    bge-base arch, 32 rows at seq 512, CLS pool
  bge_large_c4.npz   bge-large arch, 32 rows at seq 512, CLS pool
  nomic_c6.npz       nomic-embed-text-v1.5 shape (container arch
                     nomic_bert_rope_swiglu: RoPE theta 1000, SwiGLU, no
                     biases), 16 rows at seq 512, mean pool
  gte_c7.npz         gte-base-en-v1.5 shape (container arch
                     gte_new_rope_geglu: RoPE frequencies as data, erf GeGLU),
                     16 rows at seq 512, mean pool
  vit_base_c5.npz    vit-base-patch16-224 arch, the first 16 images of the
                     configuration's batch, the CLS row after the final
                     LayerNorm -- the reference's VitEncoder::run
                     (runtime/src/vit/encoder.cpp) via oracle/ref_vit_driver.cpp.
                     The images are regenerated from the recorded seed (their
                     SHA-256 is stored), not stored.
  pretiled_bf16_c1.npz, pretiled_i8_c1.npz
                     MiniLM's configuration written by nebw.npue in the
                     reference's pre-tiled form (block panels, bf16, or int8
                     with .wscale / .asmooth), 8 rows through the reference's
                     host path on that container (host_b.hpp untiles it);
                     the container is regenerated (its SHA-256 is stored).
  i8_array_c1.npz, i8_array_c2.npz
                     MiniLM (8 rows) and bge-small (4 rows) through the
                     reference's int8 ARRAY path on the int8 container above:
                     BertEncoder::run with every GEMM on the array (int8 host
                     quantisation, the int32 product, dequantisation, the fused
                     add_norm_quant / dequant_act_quant epilogues), each
                     dispatch the exact int32 product computed by the oracle's
                     stand-in design; container SHA-256 stored.
  vit_pretiled_bf16_c5.npz, vit_pretiled_i8_c5.npz
                     vit-base written by nebw.npue with pre-tiled encoder
                     operands (bf16, or int8 with .wscale / .asmooth), the
                     CLS rows of 2 images through the reference's ViT host
                     path on that container; container SHA-256 stored.
  int8_steps.npz     the int8 datapath's host steps (host_kernels.hpp:
                     quantise_a_int8, dequantise_c with an int32 C,
                     dequant_act_quant with gelu8) on int8_step_inputs(), via
                     oracle/ref_i8_driver.cpp; the inputs are regenerated
                     (their SHA-256 is stored), the outputs stored.

    python tests/golden/make_golden.py vit_base_c5     (one fixture)
"""

from __future__ import annotations

import hashlib
import sys
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO / "npu-embeddings-xdna1_b200"))
sys.path.insert(0, str(REPO))

from nebw import synth  # noqa: E402

FIXTURES = {
    "minilm_c1": ("minilm", None),
    "bge_small_c2": ("bge-small", 32),
    "bge_base_c3": ("bge-base", 32),
    "bge_large_c4": ("bge-large", 32),
    "nomic_c6": ("nomic-base", 16),
    "gte_c7": ("gte-base", 16),
}


def weights_fingerprint(w) -> str:
    h = hashlib.sha256()
    for name, arr in w.tensors():
        a = np.ascontiguousarray(arr)
        h.update(name.encode())
        h.update(a.reshape(-1)[:64].tobytes())
        h.update(a.reshape(-1)[-64:].tobytes())
    return h.hexdigest()


def sample_rows(lens, n):
    """n row indices: the shortest and longest rows, row 0 and row B-1, then
    rows at evenly spaced positions of the length-sorted order (a stable
    sort, so the pick is deterministic), topped up from a seeded
    permutation if equal picks collide."""
    if n is None:
        return np.arange(len(lens))
    lens = np.asarray(lens)
    pick = {int(np.argmin(lens)), int(np.argmax(lens)), 0, len(lens) - 1}
    by_len = np.argsort(lens, kind="stable")
    for q in np.linspace(0, len(lens) - 1, n):
        if len(pick) >= n:
            break
        pick.add(int(by_len[int(round(q))]))
    for i in np.random.default_rng(7).permutation(len(lens)):
        if len(pick) >= n:
            break
        pick.add(int(i))
    return np.array(sorted(pick))


VIT_FIXTURES = {"vit_base_c5": ("vit-base", 16)}


INT8_SEED = 20261401


def int8_step_inputs(seed: int = INT8_SEED) -> dict:
    """Seeded inputs for the int8 steps: activation rows with per-column
    SmoothQuant divisors (an all-zero row, a row of exact rounding ties, a
    row with one outlier), int32 accumulators from a real int8 product plus a
    row of values large enough to round when widened to float, and the row /
    column scales and biases of a dequantisation.  N and K are multiples of 8
    except for the `tail` rows (K = 37), which exercise the scalar tail."""
    rng = np.random.default_rng(seed)
    rows, K, N = 16, 512, 512
    a = (rng.standard_normal((rows, K)) * rng.lognormal(0.0, 1.0, K)).astype(np.float32)
    a[0] = 0.0
    a[1] = 0.0
    a[1, 0] = 127.0
    a[1, 1:9] = [0.5, 1.5, 2.5, -0.5, -1.5, -2.5, 126.5, -126.5]
    a[2, 7] = 4.0e3
    ias = (1.0 / rng.lognormal(0.0, 0.5, K)).astype(np.float32)
    ias[:9] = 1.0
    aq = rng.integers(-127, 128, (rows, 1024), dtype=np.int8)
    wq = rng.integers(-127, 128, (1024, N), dtype=np.int8)
    c = (aq.astype(np.int64) @ wq.astype(np.int64)).astype(np.int32)
    c[3] = rng.integers(-(2**31 - 1), 2**31 - 1, N, dtype=np.int64).astype(np.int32)
    sa = (rng.lognormal(-4.0, 0.5, rows)).astype(np.float32)
    ws = (rng.lognormal(-6.0, 0.5, N)).astype(np.float32)
    bias = (rng.standard_normal(N) * 0.02).astype(np.float32)
    ias_next = (1.0 / rng.lognormal(0.0, 0.5, N)).astype(np.float32)
    tail = (rng.standard_normal((5, 37)) * 3).astype(np.float32)
    tail_ias = (1.0 / rng.lognormal(0.0, 0.5, 37)).astype(np.float32)
    return dict(a=a, ias=ias, c=c, sa=sa, ws=ws, bias=bias, ias_next=ias_next, tail=tail,
                tail_ias=tail_ias)


def int8_inputs_sha256(inp: dict) -> str:
    h = hashlib.sha256()
    for k in sorted(inp):
        h.update(k.encode())
        h.update(np.ascontiguousarray(inp[k]).tobytes())
    return h.hexdigest()


def int8_step_outputs(o, inp: dict) -> dict:
    """The four int8 steps of `o` (a PortOracle or RefOracle) on `inp`."""
    q, sc = o.quantise_rows(inp["a"], inp["ias"])
    tq, tsc = o.quantise_rows(inp["tail"], inp["tail_ias"])
    y = o.dequantise(inp["c"], inp["sa"], inp["ws"], inp["bias"])
    gq, gsn = o.dequant_gelu_quant(inp["c"], inp["sa"], inp["ws"], inp["bias"], inp["ias_next"])
    return dict(q=q, scale=sc, tail_q=tq, tail_scale=tsc, dequant=y, gelu_q=gq, gelu_scale=gsn)


def make_int8(ref):
    inp = int8_step_inputs()
    out = int8_step_outputs(ref, inp)
    np.savez_compressed(
        HERE / "int8_steps.npz", seed=np.int64(INT8_SEED), inputs_sha256=int8_inputs_sha256(inp),
        provenance="reference host_kernels.hpp int8 steps (-O2 -march=x86-64-v3) via "
                   "oracle/ref_i8_driver.cpp", **out)
    print("int8_steps: written")


PRETILED = {"pretiled_bf16_c1": ("minilm", "bf16"), "pretiled_i8_c1": ("minilm", "i8")}
PRETILED_TILE, PRETILED_MAC, PRETILED_SMOOTH_SEED = (64, 64), (8, 8), 20261501


def write_pretiled(path, key: str, a_dtype: str) -> str:
    """The configuration's seeded weights as a pre-tiled container at `path`;
    returns its SHA-256."""
    from nebw.npue import write_bert_container
    cfg = synth.CONFIGS[key]
    write_bert_container(path, synth.config_weights(cfg), max_seq_len=cfg.seq,
                         gemm_layout="pretiled_bf16", a_dtype=a_dtype, tile=PRETILED_TILE,
                         mac=PRETILED_MAC, smooth_seed=PRETILED_SMOOTH_SEED)
    return hashlib.sha256(Path(path).read_bytes()).hexdigest()


def make_pretiled(ref, name, key, a_dtype):
    import tempfile
    cfg = synth.CONFIGS[key]
    ids, mask, lens = synth.config_batch(cfg)
    rows = sample_rows(lens, 8)
    with tempfile.TemporaryDirectory(dir=HERE) as td:
        path = Path(td) / "c.npue"
        digest = write_pretiled(path, key, a_dtype)
        out = ref.encode_container(path, cfg.seq, ids[rows], mask[rows], hidden_size=cfg.arch.hidden)
    np.savez_compressed(
        HERE / f"{name}.npz", config=key, a_dtype=a_dtype, container_sha256=digest,
        rows=rows.astype(np.int32), ids=ids[rows], mask=mask[rows],
        lens=lens[rows].astype(np.int32), embeddings=out,
        provenance="reference host-CPU path on a pre-tiled container (host_b.hpp untile, "
                   "int8 dequantised by .wscale with A divided by .asmooth) via "
                   "oracle/ref_driver.cpp")
    print(f"{name}: {len(rows)} rows")


I8_ARRAY = {"i8_array_c1": ("minilm", 8), "i8_array_c2": ("bge-small", 4)}


def make_i8_array(ref, name, key, n):
    """The reference's int8 ARRAY path (BertEncoder::run with the GEMMs on the
    array: int8 host steps around exact int32 products) on the configuration's
    int8 pre-tiled container, the one make_pretiled writes."""
    import tempfile
    cfg = synth.CONFIGS[key]
    ids, mask, lens = synth.config_batch(cfg)
    rows = sample_rows(lens, n)
    t0 = time.time()
    with tempfile.TemporaryDirectory(dir=HERE) as td:
        path = Path(td) / "c.npue"
        digest = write_pretiled(path, key, "i8")
        out = ref.encode_container(path, cfg.seq, ids[rows], mask[rows],
                                   hidden_size=cfg.arch.hidden, array=True)
    np.savez_compressed(
        HERE / f"{name}.npz", config=key, a_dtype="i8", container_sha256=digest,
        rows=rows.astype(np.int32), ids=ids[rows], mask=mask[rows],
        lens=lens[rows].astype(np.int32), embeddings=out,
        provenance="reference int8 array path (BertEncoder::run with --npu-ops gemm and the "
                   "fused epilogues; each dispatch the exact int32 product, oracle/ref_stub.cpp "
                   "array emulation) via oracle/ref_driver.cpp nebw_ref_encode_array")
    print(f"{name}: {len(rows)} rows in {time.time() - t0:.1f} s")


VIT_PRETILED = {"vit_pretiled_bf16_c5": ("vit-base", "bf16"),
                "vit_pretiled_i8_c5": ("vit-base", "i8")}


def write_vit_pretiled(path, key: str, a_dtype: str) -> str:
    from nebw.npue import write_vit_container
    cfg = synth.VIT_CONFIGS[key]
    write_vit_container(path, synth.vit_config_weights(cfg), gemm_layout="pretiled_bf16",
                        a_dtype=a_dtype, tile=PRETILED_TILE, mac=PRETILED_MAC,
                        smooth_seed=PRETILED_SMOOTH_SEED)
    return hashlib.sha256(Path(path).read_bytes()).hexdigest()


def make_vit_pretiled(ref, name, key, a_dtype, n=2):
    import tempfile
    cfg = synth.VIT_CONFIGS[key]
    w = synth.vit_config_weights(cfg)
    images = synth.vit_config_images(cfg, n=n)
    with tempfile.TemporaryDirectory(dir=HERE) as td:
        path = Path(td) / "v.npue"
        digest = write_vit_pretiled(path, key, a_dtype)
        out = ref.vit_encode_container(path, images, hidden_size=w.arch.hidden,
                                       n_pos=w.arch.n_pos)
    np.savez_compressed(
        HERE / f"{name}.npz", config=key, a_dtype=a_dtype, container_sha256=digest,
        n_images=np.int32(n), image_sha256=hashlib.sha256(images.tobytes()).hexdigest(),
        embeddings=out,
        provenance="reference host-CPU ViT path on a pre-tiled container (host_b.hpp untile, "
                   "int8 dequantised by .wscale with A scaled by 1/asmooth) via "
                   "oracle/ref_vit_driver.cpp")
    print(f"{name}: {n} images")


def make_vit(ref, name, key, n):
    cfg = synth.VIT_CONFIGS[key]
    w = synth.vit_config_weights(cfg)
    images = synth.vit_config_images(cfg, n=n)
    t0 = time.time()
    out = ref.vit_encode(w, images)
    print(f"{name}: {n} images in {time.time() - t0:.1f} s")
    np.savez_compressed(
        HERE / f"{name}.npz", config=key, n_images=np.int32(n),
        image_seed=20261301 + cfg.index, image_sha256=hashlib.sha256(images.tobytes()).hexdigest(),
        embeddings=out, weight_seed=20261201 + cfg.index,
        weights_fingerprint=weights_fingerprint(w),
        provenance="reference host-CPU ViT path (vit/encoder.cpp, whisper/npu_ops.cpp, -O2 "
                   "-march=x86-64-v3) via oracle/ref_vit_driver.cpp")


def main():
    from oracle.oracle import RefOracle
    ref = RefOracle()
    only = set(sys.argv[1:])
    if not only or "int8_steps" in only:
        make_int8(ref)
    for name, (key, a_dtype) in PRETILED.items():
        if not only or name in only:
            make_pretiled(ref, name, key, a_dtype)
    for name, (key, n) in I8_ARRAY.items():
        if not only or name in only:
            make_i8_array(ref, name, key, n)
    for name, (key, a_dtype) in VIT_PRETILED.items():
        if not only or name in only:
            make_vit_pretiled(ref, name, key, a_dtype)
    for name, (key, n) in VIT_FIXTURES.items():
        if not only or name in only:
            make_vit(ref, name, key, n)
    for name, (key, n) in FIXTURES.items():
        if only and name not in only:
            continue
        cfg = synth.CONFIGS[key]
        w = synth.config_weights(cfg)
        ids, mask, lens = synth.config_batch(cfg)
        rows = sample_rows(lens, n)
        t0 = time.time()
        out = ref.encode(w, ids[rows], mask[rows])
        print(f"{name}: {len(rows)} rows in {time.time() - t0:.1f} s")
        np.savez_compressed(
            HERE / f"{name}.npz", config=key, rows=rows.astype(np.int32),
            ids=ids[rows], mask=mask[rows], lens=lens[rows].astype(np.int32), embeddings=out,
            weight_seed=20261201 + cfg.index, token_seed=20261301 + cfg.index,
            weights_fingerprint=weights_fingerprint(w),
            provenance="reference host-CPU path (bert_encoder.cpp/pool.cpp/model.cpp, -O2 "
                       "-march=x86-64-v3) via oracle/ref_driver.cpp")


if __name__ == "__main__":
    main()
