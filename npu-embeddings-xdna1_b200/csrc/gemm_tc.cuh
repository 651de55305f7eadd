// The unified bf16 GEMM of the encoder (QKV, attention-out, FFN-up,
// FFN-down) on the sm_100a tensor cores.
//
//   C[M, N] = epilogue( A[M, K] . W[N, K]^T )        A, W bf16; accumulate fp32
//
// This replaces the reference's gemm_rtp design set (AIE MMAC over
// pre-tiled B panels, tools/lib/gemm_pretiled.py:1-60, dispatched from
// BertEncoder::gemm, runtime/src/encoders/bert_encoder.cpp:741-924) and its
// host twin hostconv::gemm_nt (runtime/include/common/conv_host.hpp:150-181),
// with the elementwise passes that follow a GEMM in BertEncoder::run folded
// into the epilogue:
//   + bias                      (gemm_nt adds it last, conv_host.hpp:177)
//   + gelu8 / erf GELU          (gelu_cpu, bert_encoder.cpp:532-580;
//                                gelu_erf_exact, app_state.hpp:116-120)
//   + residual, fp32 out        (add_into, bert_encoder.cpp:1183-1194)
//   fp32 -> bf16 RNE narrow     (kernels/narrow_f32_bf16.cc; to_bf16,
//                                host_kernels.hpp:157-161)
//
// Design (one CTA per SM, persistent over 128 x BN output tiles):
//   warp 0      TMA producer: A and W tiles of 64 K-elements, 128-byte
//               swizzled, into a STAGES-deep ring of shared-memory stages
//   warp 1      allocates TMEM, issues tcgen05.mma (M=128, N=BN, K=16) from
//               one thread, commits each stage back to the producer and each
//               finished tile to the epilogue
//   warps 2-9   epilogue: tcgen05.ld the accumulator (one row per thread,
//               two warps per 32-lane quarter, half the columns each),
//               bias / activation / residual in fp32, store
// The accumulator is double-buffered in TMEM (2 x BN columns), so the
// epilogue of tile i overlaps the MMAs of tile i+1.
//
// M may be read from device memory at kernel start (the packed token count
// of a varlen batch), so a whole encoder pass needs no host round trip.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cstdint>

#include "ptx.cuh"

namespace nebw {

enum GemmEpi : int {
  kEpiBf16 = 0,       // out bf16 = acc + bias
  kEpiBf16Gelu8 = 1,  // out bf16 = gelu8(acc + bias)
  kEpiBf16Erf = 2,    // out bf16 = erf-gelu(acc + bias)
  kEpiF32 = 3,        // out f32  = acc + bias
  kEpiF32Resid = 4,   // out f32  = (acc + bias) + resid   (resid may alias out)
  // Gated FFN-up over a weight whose N columns are interleaved in groups of
  // 64 = [32 up | 32 gate] (the same 32 output columns): out bf16 [M, N/2],
  // out[:, 32g + i] = (up + bias) * act(gate + bias).  CTA-pair kernel only.
  kEpiBf16SwiGLU = 5,  // act = SiLU
  kEpiBf16GeGLU = 6,   // act = erf GELU
  // QKV with rotary positions: columns < rope_cols (Q and K) rotated per
  // head_dim-64 head by the row's position (row_pos) before the narrow, V
  // columns plain.  CTA-pair kernel only.
  kEpiBf16Rope = 7,
  // int8 operands (tcgen05 kind::i8, s32 accumulators, 128-int8 K-blocks:
  // the same 128-byte rows), dequantised in the epilogue as
  // app::dequantise_c does, y = fma(float(acc) * sa[row], ws[col], bias[col]);
  // rows past the live count are written as 0.  CTA-pair kernel only.
  kEpiI8F32 = 8,    // out f32  = y
  kEpiI8Gelu8 = 9,  // out f32  = gelu8(y)
  kEpiI8Bf16 = 10,  // out bf16 = y
};

__host__ __device__ constexpr bool epi_int8(int e) { return e >= kEpiI8F32 && e <= kEpiI8Bf16; }

struct GemmArgs {
  int M;             // row bound (the A tensor map's row extent)
  const int *M_dev;  // if set, the live row count is min(*M_dev, M)
  int N, K;
  const float *bias;   // [N] or null
  const float *resid;  // [M, N] fp32 for kEpiF32Resid
  void *out;           // [M, N], bf16 or fp32 by epilogue
  int *err;            // device error word
  // kEpiBf16Rope: position of each packed row in its sequence, the cos / sin
  // tables [rope_rows, 64], the rotated column count (2 * hidden)
  const int *row_pos;
  const float *rope_cos, *rope_sin;
  int rope_rows, rope_cols;
  // int8 epilogues: A's row scales [M] and W's column scales [N]
  const float *sa, *ws;
};

constexpr int kGemmBM = 128;
constexpr int kGemmBK = 64;
constexpr int kGemmThreads = 320;  // 2 control warps + 8 epilogue warps

template <int BN>
struct GemmShape {
  static_assert(BN == 128 || BN == 256, "BN must be 128 or 256");
  static constexpr int kStages = BN == 256 ? 4 : 6;
  static constexpr int kABytes = kGemmBM * kGemmBK * 2;  // 16 KB
  static constexpr int kBBytes = BN * kGemmBK * 2;       // 16 or 32 KB
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTmemCols = 2 * BN;               // 256 or 512
  static constexpr int kBarBytes = 256;
  static constexpr int kSmemBytes = 1024 /*align slack*/ + kStages * kStageBytes + kBarBytes;
};

// ---- activation functions of the epilogue ------------------------------------

// gelu8: max(v,0) + P(min(|v|,4)), the reference's degree-8 polynomial with
// its own coefficients (host_kernels.hpp:322-352), Horner with fused
// multiply-adds exactly as its AVX2 form evaluates it.
__device__ __forceinline__ float gelu8(float v) {
  const float u = fminf(fabsf(v), 4.0f);
  float pl = fmaf(-7.2340282171e-05f, u, 1.8179518005e-03f);
  pl = fmaf(pl, u, -1.7707383379e-02f);
  pl = fmaf(pl, u, 8.4577147641e-02f);
  pl = fmaf(pl, u, -1.9228671834e-01f);
  pl = fmaf(pl, u, 9.8431124458e-02f);
  pl = fmaf(pl, u, 3.6137852062e-01f);
  pl = fmaf(pl, u, -4.9454128936e-01f);
  pl = fmaf(pl, u, -1.3007010117e-04f);
  return fmaxf(v, 0.0f) + pl;
}

// gelu8 on two values at once with sm_100's packed fp32 arithmetic
// (fma_x2 / add_x2): each lane is the same IEEE operation as the scalar form
// above, so the results are bit-identical at half the FMA-pipe instructions.
__device__ __forceinline__ void gelu8_x2(float &a, float &b) {
  const uint64_t u = pk2(fminf(fabsf(a), 4.0f), fminf(fabsf(b), 4.0f));
  uint64_t pl = fma_x2(pk2(-7.2340282171e-05f, -7.2340282171e-05f), u,
                       pk2(1.8179518005e-03f, 1.8179518005e-03f));
  pl = fma_x2(pl, u, pk2(-1.7707383379e-02f, -1.7707383379e-02f));
  pl = fma_x2(pl, u, pk2(8.4577147641e-02f, 8.4577147641e-02f));
  pl = fma_x2(pl, u, pk2(-1.9228671834e-01f, -1.9228671834e-01f));
  pl = fma_x2(pl, u, pk2(9.8431124458e-02f, 9.8431124458e-02f));
  pl = fma_x2(pl, u, pk2(3.6137852062e-01f, 3.6137852062e-01f));
  pl = fma_x2(pl, u, pk2(-4.9454128936e-01f, -4.9454128936e-01f));
  pl = fma_x2(pl, u, pk2(-1.3007010117e-04f, -1.3007010117e-04f));
  unpk2(add_x2(pk2(fmaxf(a, 0.0f), fmaxf(b, 0.0f)), pl), a, b);
}

// Erf GELU, x * Phi(x) = 0.5 x (1 + erf(x / sqrt 2)), with erf from
// Abramowitz & Stegun, Handbook of Mathematical Functions, formula 7.1.28
// (Hastings): for t >= 0, erf(t) = 1 - (1 + a1 t + ... + a6 t^6)^-16 with
// |error| <= 3e-7.  erf is odd, so x erf(x / sqrt 2) = |x| erf(|x| / sqrt 2)
// and
//   x Phi(x) = max(x, 0) - |x| q,   q = 0.5 (1 - erf(|x| / sqrt 2)) = 0.5 / s^16
// with s = 1 + P(|x| / sqrt 2): one reciprocal on the SFU and one fused
// multiply-add per value, no compare or select.  Measured against erf in
// double over [-12, 12] in fp32: absolute error of the GELU <= 7e-7, far
// below the bf16 rounding of the output (relative 2^-9).  s^16 overflows to
// inf for |x| > ~35, where 1/s^16 = 0 and the result is max(x, 0).
// The reference computes erf in double (app::gelu_erf_exact,
// app_state.hpp:116-120).
__device__ __forceinline__ float gelu_erf(float v) {
  const float t = fabsf(v) * 0.70710678118654752440f;
  float p = fmaf(4.30638e-05f, t, 2.765672e-04f);
  p = fmaf(p, t, 1.520143e-04f);
  p = fmaf(p, t, 9.2705272e-03f);
  p = fmaf(p, t, 4.22820123e-02f);
  p = fmaf(p, t, 7.05230784e-02f);
  float sp = fmaf(p, t, 1.0f);
  sp = sp * sp;
  sp = sp * sp;
  sp = sp * sp;
  sp = sp * sp;
  return fmaf(fabsf(v) * rcp_approx(sp), -0.5f, fmaxf(v, 0.0f));
}

// The same on two values with packed fp32 (fma_x2 / mul_x2).
__device__ __forceinline__ void gelu_erf_x2(float &a, float &b) {
  const uint64_t ax = pk2(fabsf(a), fabsf(b));
  const uint64_t t = mul_x2(ax, pk2(0.70710678118654752440f, 0.70710678118654752440f));
  uint64_t p = fma_x2(pk2(4.30638e-05f, 4.30638e-05f), t, pk2(2.765672e-04f, 2.765672e-04f));
  p = fma_x2(p, t, pk2(1.520143e-04f, 1.520143e-04f));
  p = fma_x2(p, t, pk2(9.2705272e-03f, 9.2705272e-03f));
  p = fma_x2(p, t, pk2(4.22820123e-02f, 4.22820123e-02f));
  p = fma_x2(p, t, pk2(7.05230784e-02f, 7.05230784e-02f));
  uint64_t sp = fma_x2(p, t, pk2(1.0f, 1.0f));
  sp = mul_x2(sp, sp);
  sp = mul_x2(sp, sp);
  sp = mul_x2(sp, sp);
  sp = mul_x2(sp, sp);
  float s0, s1;
  unpk2(sp, s0, s1);
  const uint64_t aq = mul_x2(ax, pk2(rcp_approx(s0), rcp_approx(s1)));  // 2 |x| q
  unpk2(fma_x2(aq, pk2(-0.5f, -0.5f), pk2(fmaxf(a, 0.0f), fmaxf(b, 0.0f))), a, b);
}

// SiLU on the SFU: x / (1 + 2^(-x log2 e)), the exponent floored at -120 as
// swiglu_cpu floors it (bert_encoder.cpp:582-627); ex2.approx and a fast
// divide, far below the bf16 rounding of the gated product.
__device__ __forceinline__ float silu_fast(float x) {
  const float a = fmaxf(-x * 1.4426950408889634f, -120.0f);
  return __fdividef(x, 1.0f + ex2_approx(a));
}

template <int EPI>
__device__ __forceinline__ float epi_act(float v) {
  if constexpr (EPI == kEpiBf16Gelu8) return gelu8(v);
  else if constexpr (EPI == kEpiBf16Erf) return gelu_erf(v);
  else return v;
}

// Store 32 accumulator columns [col0, col0+32) of one output row.
template <int EPI>
__device__ __forceinline__ void epi_store32(const GemmArgs &p, int row, int col0,
                                            const uint32_t (&r)[32]) {
  const int N = p.N;
  const int ncols = min(32, N - col0);  // N % 8 == 0, so ncols % 8 == 0
  float v[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
  if (p.bias) {
    const float4 *b4 = reinterpret_cast<const float4 *>(p.bias + col0);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (i * 4 < ncols) {
        const float4 b = __ldg(b4 + i);
        v[4 * i + 0] += b.x;
        v[4 * i + 1] += b.y;
        v[4 * i + 2] += b.z;
        v[4 * i + 3] += b.w;
      }
    }
  }
  const size_t base = static_cast<size_t>(row) * N + col0;
  if constexpr (EPI == kEpiF32 || EPI == kEpiF32Resid) {
    float *o = static_cast<float *>(p.out) + base;
    if constexpr (EPI == kEpiF32Resid) {
      const float4 *r4 = reinterpret_cast<const float4 *>(p.resid + base);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (i * 4 < ncols) {
          const float4 x = r4[i];
          v[4 * i + 0] += x.x;
          v[4 * i + 1] += x.y;
          v[4 * i + 2] += x.z;
          v[4 * i + 3] += x.w;
        }
      }
    }
    float4 *o4 = reinterpret_cast<float4 *>(o);
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (i * 4 < ncols) o4[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
  } else {
    uint4 *o4 = reinterpret_cast<uint4 *>(static_cast<__nv_bfloat16 *>(p.out) + base);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (i * 8 < ncols) {
        uint4 w;
        w.x = pack_bf16x2(epi_act<EPI>(v[8 * i + 0]), epi_act<EPI>(v[8 * i + 1]));
        w.y = pack_bf16x2(epi_act<EPI>(v[8 * i + 2]), epi_act<EPI>(v[8 * i + 3]));
        w.z = pack_bf16x2(epi_act<EPI>(v[8 * i + 4]), epi_act<EPI>(v[8 * i + 5]));
        w.w = pack_bf16x2(epi_act<EPI>(v[8 * i + 6]), epi_act<EPI>(v[8 * i + 7]));
        o4[i] = w;
      }
    }
  }
}

template <int BN, int EPI>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                   const GemmArgs p) {
  using S = GemmShape<BN>;
  constexpr int kStages = S::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t *sA = smem;
  uint8_t *sW = smem + kStages * S::kABytes;
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + kStages * S::kStageBytes);
  uint64_t *empty = full + kStages;
  uint64_t *tfull = empty + kStages;   // [2] accumulator ready for the epilogue
  uint64_t *tempty = tfull + 2;        // [2] accumulator drained by the epilogue
  uint64_t *drain = tempty + 2;        // [1] MMA-side drain at exit
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  int M = p.M;
  if (p.M_dev) M = min(M, __ldg(p.M_dev));
  const int m_blocks = (M + kGemmBM - 1) / kGemmBM;
  const int n_blocks = (p.N + BN - 1) / BN;
  const int num_tiles = m_blocks * n_blocks;
  const int num_kb = (p.K + kGemmBK - 1) / kGemmBK;

  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmW);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 8);  // one arrival per epilogue warp
    }
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, S::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, last_phase = 0;  // per stage: ever issued, parity of last issue
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int mb = tile / n_blocks, nb = tile % n_blocks;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, p.err)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], S::kStageBytes);
          tma_load_2d(sA + stage * S::kABytes, &tmA, &full[stage], kb * kGemmBK, mb * kGemmBM);
          tma_load_2d(sW + stage * S::kBBytes, &tmW, &full[stage], kb * kGemmBK, nb * BN);
          issued_mask |= 1u << stage;
          last_phase = (last_phase & ~(1u << stage)) | (phase << stage);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Drain: every stage this thread loaded has landed before the CTA may
      // exit (normally already true -- the MMA thread waited on each).
      for (int s = 0; s < kStages; ++s)
        if (issued_mask & (1u << s)) mbar_wait(&full[s], (last_phase >> s) & 1u, p.err);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    // The whole warp walks the schedule and waits (so that the loop state
    // and the descriptors are warp-uniform); one elected lane issues.
    {
      constexpr uint32_t idesc = idesc_bf16_f32(kGemmBM, BN);
      const bool elect = elect_one_sync();
      auto wait_all = [&](uint64_t *bar, uint32_t parity) -> bool {
        return __all_sync(0xffffffffu, mbar_wait(bar, parity, p.err));
      };
      int stage = 0;
      uint32_t phase = 0;
      bool issued_any = false, ok = true;
      int local = 0;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!wait_all(&tempty[acc], acc_phase ^ 1u)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!wait_all(&full[stage], phase)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t da = sdesc_kmajor_sw128(smem_u32(sA + stage * S::kABytes));
          const uint64_t dw = sdesc_kmajor_sw128(smem_u32(sW + stage * S::kBBytes));
          if (elect) {
#pragma unroll
            for (int k = 0; k < kGemmBK / 16; ++k)  // +32 B per 16 elements of K
              umma_bf16(d_tmem, da + k * 2, dw + k * 2, idesc, (kb | k) != 0 ? 1u : 0u);
            umma_commit(&empty[stage]);  // stage reusable once these MMAs retire
          }
          __syncwarp();
          issued_any = true;
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (ok && elect) umma_commit(&tfull[acc]);
        __syncwarp();
      }
      // Drain: all MMAs this warp issued have retired before TMEM is freed.
      if (issued_any) {
        if (elect) umma_commit(drain);
        __syncwarp();
        wait_all(drain, 0);
      }
    }
  } else {
    // ---------------- epilogue (warps 2..9) ----------------
    // Two warps per TMEM lane quarter (a warp may only read lanes
    // [32*(warp%4), +32)); each takes half of the tile's columns.  TMEM loads
    // are double-buffered: chunk c+1 is in flight while chunk c is stored.
    constexpr int kHalf = BN / 2;
    constexpr int kChunks = kHalf / 32;
    const int quarter = warp & 3;
    const int col_half = ((warp - 2) >> 2) * kHalf;
    const int row_in_tile = quarter * 32 + lane;
    int local = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      // warp-uniform outcome: the tcgen05.ld below is warp-collective
      if (!__all_sync(0xffffffffu, mbar_wait(&tfull[acc], acc_phase, p.err))) break;
      tc_fence_after();
      const int mb = tile / n_blocks, nb = tile % n_blocks;
      const int row = mb * kGemmBM + row_in_tile;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                             static_cast<uint32_t>(acc * BN + col_half);
      uint32_t ra[32], rb[32];
      tmem_ld_32x32b_x32(t_row, ra);
      tmem_wait_ld_regs(ra);
#pragma unroll
      for (int c = 0; c < kChunks; ++c) {
        uint32_t(&cur)[32] = (c & 1) ? rb : ra;
        uint32_t(&nxt)[32] = (c & 1) ? ra : rb;
        if (c + 1 < kChunks) tmem_ld_32x32b_x32(t_row + (c + 1) * 32, nxt);
        if (c + 1 == kChunks) {
          // every TMEM read of this tile has completed: hand the buffer back
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tempty[acc]);
        }
        const int col0 = nb * BN + col_half + c * 32;
        if (row < M && col0 < p.N) epi_store32<EPI>(p, row, col0, cur);
        if (c + 1 < kChunks) tmem_wait_ld_regs(nxt);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, S::kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// The same GEMM on CTA pairs (tcgen05 cta_group::2): tiles of 256 x BN per
// pair.  Each CTA of a pair loads its 128 rows of A and its BN/2 rows of W;
// the pair leader issues M=256 UMMAs that read both CTAs' shared memory and
// accumulate rows 0-127 in the leader's TMEM and rows 128-255 in the peer's.
// Per FLOP, each SM moves half the operand bytes of the single-CTA tile, and
// the smaller per-CTA stage allows a deeper ring (6 or 8 stages).
//
// Synchronisation, per stage s and accumulator buffer a:
//   full[s]   leader only: the leader's producer arrives with the pair's
//             transaction bytes; both CTAs' TMA loads complete on it
//   empty[s]  both CTAs: the leader's MMA commit, multicast to the pair
//   tfull[a]  both CTAs: the leader's commit after a tile's last k-block
//   tempty[a] leader only: one arrival per epilogue warp of both CTAs (16)
// No TMA load uses multicast; the only multicast is tcgen05.commit's.
// ---------------------------------------------------------------------------

template <int BN>
struct GemmPairShape {
  static_assert(BN == 128 || BN == 256, "BN must be 128 or 256");
  static constexpr int kHalfN = BN / 2;                  // W rows loaded per CTA
  static constexpr int kABytes = kGemmBM * kGemmBK * 2;  // 16 KB
  static constexpr int kBBytes = kHalfN * kGemmBK * 2;   // 16 or 8 KB
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = (160 * 1024) / kStageBytes;  // 5 or 6
  static constexpr int kTmemCols = 2 * BN;
  // epilogue staging: per epilogue warp two 32 x 32 fp32 (or bf16) chunks
  static constexpr int kChunkBytes = 32 * 32 * 4;
  static constexpr int kStagingBytes = 8 * 2 * kChunkBytes;  // 64 KB
  static constexpr int kBarBytes = 256;
  static constexpr int kSmemBytes =
      1024 + kStages * kStageBytes + kStagingBytes + kBarBytes;
};

// Write 32 accumulator columns of this thread's row, after bias and the
// activation, into a 32-row chunk staged in shared memory in the swizzled
// layout of the output tensor map's 32 x 32 box: fp32 rows are 128 bytes
// (128-byte swizzle: 16-byte piece p of row r sits at p ^ (r % 8)), bf16
// rows are 64 bytes (64-byte swizzle: p ^ ((r / 2) % 4)).  Either way a
// warp's 32 row-writes of one piece land in all 32 banks, four deep.
template <int EPI>
__device__ __forceinline__ void epi_stage32(const GemmArgs &p, int col0, const uint32_t (&r)[32],
                                            uint8_t *chunk, int lane) {
  const int ncols = min(32, p.N - col0);
  float v[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
  if (p.bias) {
    const float4 *b4 = reinterpret_cast<const float4 *>(p.bias + col0);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (i * 4 < ncols) {
        const float4 b = __ldg(b4 + i);
        unpk2(add_x2(pk2(v[4 * i + 0], v[4 * i + 1]), pk2(b.x, b.y)), v[4 * i + 0], v[4 * i + 1]);
        unpk2(add_x2(pk2(v[4 * i + 2], v[4 * i + 3]), pk2(b.z, b.w)), v[4 * i + 2], v[4 * i + 3]);
      }
    }
  }
  if constexpr (EPI == kEpiF32) {
    uint8_t *row = chunk + lane * 128;
    const int sw = lane & 7;
#pragma unroll
    for (int q = 0; q < 8; ++q)
      *reinterpret_cast<float4 *>(row + ((q ^ sw) << 4)) =
          make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
  } else {
    uint32_t pk[16];
    if constexpr (EPI == kEpiBf16Gelu8) {
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        gelu8_x2(v[2 * i], v[2 * i + 1]);
        pk[i] = pack_bf16x2(v[2 * i], v[2 * i + 1]);
      }
    } else if constexpr (EPI == kEpiBf16Erf) {
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        gelu_erf_x2(v[2 * i], v[2 * i + 1]);
        pk[i] = pack_bf16x2(v[2 * i], v[2 * i + 1]);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i)
        pk[i] = pack_bf16x2(epi_act<EPI>(v[2 * i]), epi_act<EPI>(v[2 * i + 1]));
    }
    uint8_t *row = chunk + lane * 64;
    const int sw = (lane >> 1) & 3;
#pragma unroll
    for (int q = 0; q < 4; ++q)
      *reinterpret_cast<uint4 *>(row + ((q ^ sw) << 4)) =
          make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
  }
}

// The int8 epilogue: dequantise (and gelu8) the 32 int32 accumulator columns
// [col0, col0 + 32) of this thread's row -- app::dequantise_c's
// y = fma(float(c) * sa, ws[col], bias[col]) -- into its row of a 32-row
// chunk staged in shared memory, in the output map's swizzle: fp32 rows of 128 bytes (16-byte piece q at q ^ (r % 8)),
// or bf16 RNE rows of 64 bytes (q ^ ((r / 2) % 4)).  Columns past N and rows
// past the live count are staged as 0 (the bulk store clips columns past the
// map's N; rows past the live count but inside the buffer are written, and a
// zero row is what the encoder's later readers of those rows expect).
template <bool GELU, bool BF16>
__device__ __forceinline__ void i8_stage32(int N, const float *ws, const float *bias, float sa,
                                           bool live_row, int col0, const uint32_t (&r)[32],
                                           uint8_t *chunk, int lane) {
  const int ncols = live_row ? min(32, N - col0) : 0;  // N % 8 == 0
  const float4 *w4 = reinterpret_cast<const float4 *>(ws + col0);
  const float4 *b4 = reinterpret_cast<const float4 *>(bias + col0);
  // two columns at a time on the packed fp32 pipe: the same IEEE product and
  // fused multiply-add per value as the scalar form, half the instructions
  const uint64_t sa2 = pk2(sa, sa);
  float y[32];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if (i * 4 < ncols) {
      const float4 w = __ldg(w4 + i);
      const float4 b = bias ? __ldg(b4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
      const float c0 = __int2float_rn(static_cast<int>(r[4 * i + 0]));
      const float c1 = __int2float_rn(static_cast<int>(r[4 * i + 1]));
      const float c2 = __int2float_rn(static_cast<int>(r[4 * i + 2]));
      const float c3 = __int2float_rn(static_cast<int>(r[4 * i + 3]));
      unpk2(fma_x2(mul_x2(pk2(c0, c1), sa2), pk2(w.x, w.y), pk2(b.x, b.y)), y[4 * i + 0],
            y[4 * i + 1]);
      unpk2(fma_x2(mul_x2(pk2(c2, c3), sa2), pk2(w.z, w.w), pk2(b.z, b.w)), y[4 * i + 2],
            y[4 * i + 3]);
      if constexpr (GELU) {
        gelu8_x2(y[4 * i + 0], y[4 * i + 1]);
        gelu8_x2(y[4 * i + 2], y[4 * i + 3]);
      }
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e) y[4 * i + e] = 0.0f;
    }
  }
  if constexpr (BF16) {
    uint8_t *rowp = chunk + lane * 64;
    const int sw = (lane >> 1) & 3;
#pragma unroll
    for (int q = 0; q < 4; ++q)
      *reinterpret_cast<uint4 *>(rowp + ((q ^ sw) << 4)) =
          make_uint4(pack_bf16x2(y[8 * q], y[8 * q + 1]), pack_bf16x2(y[8 * q + 2], y[8 * q + 3]),
                     pack_bf16x2(y[8 * q + 4], y[8 * q + 5]),
                     pack_bf16x2(y[8 * q + 6], y[8 * q + 7]));
  } else {
    uint8_t *rowp = chunk + lane * 128;
    const int sw = lane & 7;
#pragma unroll
    for (int q = 0; q < 8; ++q)
      *reinterpret_cast<float4 *>(rowp + ((q ^ sw) << 4)) =
          make_float4(y[4 * q], y[4 * q + 1], y[4 * q + 2], y[4 * q + 3]);
  }
}

// Gated epilogue: the up chunk (GEMM columns col0 .. col0+31) and the gate
// chunk (col0+32 .. col0+63) of this thread's row -> 32 bf16 outputs
// up * act(gate), biases added first, staged as one bf16 32 x 32 chunk in
// the output map's 64-byte swizzle.
template <int EPI>
__device__ __forceinline__ void epi_stage_glu(const GemmArgs &p, int col0,
                                              const uint32_t (&ru)[32],
                                              const uint32_t (&rg)[32], uint8_t *chunk,
                                              int lane) {
  uint32_t pk[16];
  const float4 *bu = p.bias ? reinterpret_cast<const float4 *>(p.bias + col0) : nullptr;
  const float4 *bg = p.bias ? reinterpret_cast<const float4 *>(p.bias + col0 + 32) : nullptr;
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    float u[4] = {__uint_as_float(ru[4 * q]), __uint_as_float(ru[4 * q + 1]),
                  __uint_as_float(ru[4 * q + 2]), __uint_as_float(ru[4 * q + 3])};
    float g[4] = {__uint_as_float(rg[4 * q]), __uint_as_float(rg[4 * q + 1]),
                  __uint_as_float(rg[4 * q + 2]), __uint_as_float(rg[4 * q + 3])};
    if (bu) {
      const float4 b1 = __ldg(bu + q), b2 = __ldg(bg + q);
      u[0] += b1.x; u[1] += b1.y; u[2] += b1.z; u[3] += b1.w;
      g[0] += b2.x; g[1] += b2.y; g[2] += b2.z; g[3] += b2.w;
    }
    float o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if constexpr (EPI == kEpiBf16SwiGLU) o[i] = u[i] * silu_fast(g[i]);
      else o[i] = u[i] * gelu_erf(g[i]);
    }
    pk[2 * q] = pack_bf16x2(o[0], o[1]);
    pk[2 * q + 1] = pack_bf16x2(o[2], o[3]);
  }
  uint8_t *row = chunk + lane * 64;
  const int sw = (lane >> 1) & 3;
#pragma unroll
  for (int q = 0; q < 4; ++q)
    *reinterpret_cast<uint4 *>(row + ((q ^ sw) << 4)) =
        make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
}

// Rotary epilogue for one head of Q or K: chunk x1 (dims 0..31, GEMM
// columns col0 ..) and x2 (dims 32..63, col0 + 32 ..) of this thread's row,
// biases added, rotated by the row's position (o1 = fma(-x2, s, x1 c), o2 =
// fma(x1, s, x2 c), the reference build's evaluation order), narrowed and
// staged as two bf16 32 x 32 chunks.  The position is clamped to the table,
// so a row past the live count reads a valid entry (its output is never
// used).
__device__ __forceinline__ void epi_stage_rope(const GemmArgs &p, int col0, int row, int live_rows,
                                               const uint32_t (&r1)[32], const uint32_t (&r2)[32],
                                               uint8_t *chunk1, uint8_t *chunk2, int lane) {
  int pos = row < live_rows ? __ldg(p.row_pos + row) : 0;
  pos = min(max(pos, 0), p.rope_rows - 1);
  const float4 *cs = reinterpret_cast<const float4 *>(p.rope_cos + static_cast<int64_t>(pos) * 64);
  const float4 *sn = reinterpret_cast<const float4 *>(p.rope_sin + static_cast<int64_t>(pos) * 64);
  const float4 *b1 = p.bias ? reinterpret_cast<const float4 *>(p.bias + col0) : nullptr;
  const float4 *b2 = p.bias ? reinterpret_cast<const float4 *>(p.bias + col0 + 32) : nullptr;
  uint32_t pk1[16], pk2a[16];
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const float4 c = __ldg(cs + q), sv = __ldg(sn + q);
    float x1[4] = {__uint_as_float(r1[4 * q]), __uint_as_float(r1[4 * q + 1]),
                   __uint_as_float(r1[4 * q + 2]), __uint_as_float(r1[4 * q + 3])};
    float x2[4] = {__uint_as_float(r2[4 * q]), __uint_as_float(r2[4 * q + 1]),
                   __uint_as_float(r2[4 * q + 2]), __uint_as_float(r2[4 * q + 3])};
    if (b1) {
      const float4 u = __ldg(b1 + q), w = __ldg(b2 + q);
      x1[0] += u.x; x1[1] += u.y; x1[2] += u.z; x1[3] += u.w;
      x2[0] += w.x; x2[1] += w.y; x2[2] += w.z; x2[3] += w.w;
    }
    const float cc[4] = {c.x, c.y, c.z, c.w}, ss[4] = {sv.x, sv.y, sv.z, sv.w};
    float o1[4], o2[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      o1[i] = __fmaf_rn(-x2[i], ss[i], __fmul_rn(x1[i], cc[i]));
      o2[i] = __fmaf_rn(x1[i], ss[i], __fmul_rn(x2[i], cc[i]));
    }
    pk1[2 * q] = pack_bf16x2(o1[0], o1[1]);
    pk1[2 * q + 1] = pack_bf16x2(o1[2], o1[3]);
    pk2a[2 * q] = pack_bf16x2(o2[0], o2[1]);
    pk2a[2 * q + 1] = pack_bf16x2(o2[2], o2[3]);
  }
  const int sw = (lane >> 1) & 3;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    *reinterpret_cast<uint4 *>(chunk1 + lane * 64 + ((q ^ sw) << 4)) =
        make_uint4(pk1[4 * q], pk1[4 * q + 1], pk1[4 * q + 2], pk1[4 * q + 3]);
    *reinterpret_cast<uint4 *>(chunk2 + lane * 64 + ((q ^ sw) << 4)) =
        make_uint4(pk2a[4 * q], pk2a[4 * q + 1], pk2a[4 * q + 2], pk2a[4 * q + 3]);
  }
}

template <int BN, int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kGemmThreads, 1)
    gemm_tc_pair_kernel(const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmW,
                        const __grid_constant__ CUtensorMap tmC, const GemmArgs p) {
  using S = GemmPairShape<BN>;
  constexpr int kStages = S::kStages;
  constexpr int kPairM = 2 * kGemmBM;
  constexpr bool kTmaStore = EPI != kEpiF32Resid;
  constexpr bool kInt8 = epi_int8(EPI);
  // elements per 128-byte K-block: 64 bf16 or 128 int8 (the same tiles)
  constexpr int kBK = kInt8 ? 2 * kGemmBK : kGemmBK;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t *sA = smem;
  uint8_t *sW = smem + kStages * S::kABytes;
  uint8_t *staging = smem + kStages * S::kStageBytes;
  uint64_t *full = reinterpret_cast<uint64_t *>(staging + S::kStagingBytes);
  uint64_t *empty = full + kStages;
  uint64_t *tfull = empty + kStages;
  uint64_t *tempty = tfull + 2;
  uint64_t *drain = tempty + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0 = leader, 1 = peer
  const bool leader = rank == 0;

  int M = p.M;
  if (p.M_dev) M = min(M, __ldg(p.M_dev));
  const int m_blocks = (M + kPairM - 1) / kPairM;
  const int n_blocks = (p.N + BN - 1) / BN;
  const int num_tiles = m_blocks * n_blocks;
  const int num_kb = (p.K + kBK - 1) / kBK;
  const int pair = blockIdx.x >> 1, num_pairs = gridDim.x >> 1;

  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmW);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 16);  // 8 epilogue warps x 2 CTAs
    }
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, S::kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised, TMEM allocated
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs) ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = pair; tile < num_tiles && ok; tile += num_pairs) {
        const int mb = tile / n_blocks, nb = tile % n_blocks;
        const int a_row = mb * kPairM + static_cast<int>(rank) * kGemmBM;
        const int w_row = nb * BN + static_cast<int>(rank) * S::kHalfN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, p.err)) {
            ok = false;
            break;
          }
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * S::kStageBytes);
          const uint32_t bar = map_to_cta(smem_u32(&full[stage]), 0);
          tma_load_2d_pair(sA + stage * S::kABytes, &tmA, bar, kb * kBK, a_row);
          tma_load_2d_pair(sW + stage * S::kBBytes, &tmW, bar, kb * kBK, w_row);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Tail: wait until the leader's MMAs have released every stage, so all
      // loads this CTA issued have landed and all multicast commits aimed at
      // this CTA's empty barriers have arrived before it may exit.
      for (int i = 0; i < kStages && ok; ++i) {
        if (!mbar_wait(&empty[stage], phase ^ 1u, p.err)) break;
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (leader only) ----------------
    // The whole warp walks the schedule and waits (so that the loop state
    // and the descriptors are warp-uniform); one elected lane issues.
    if (leader) {
      constexpr uint32_t idesc = kInt8 ? idesc_s8_s32(kPairM, BN) : idesc_bf16_f32(kPairM, BN);
      const bool elect = elect_one_sync();
      auto wait_all = [&](uint64_t *bar, uint32_t parity) -> bool {
        return __all_sync(0xffffffffu, mbar_wait(bar, parity, p.err));
      };
      int stage = 0;
      uint32_t phase = 0;
      bool issued_any = false, ok = true;
      int local = 0;
      for (int tile = pair; tile < num_tiles && ok; tile += num_pairs, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!wait_all(&tempty[acc], acc_phase ^ 1u)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!wait_all(&full[stage], phase)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t da = sdesc_kmajor_sw128(smem_u32(sA + stage * S::kABytes));
          const uint64_t dw = sdesc_kmajor_sw128(smem_u32(sW + stage * S::kBBytes));
          if (elect) {
            // four MMAs per 128-byte K-block, +32 B each (16 bf16 or 32 int8 of K)
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              if constexpr (kInt8)
                umma_s8_pair(d_tmem, da + k * 2, dw + k * 2, idesc, (kb | k) != 0 ? 1u : 0u);
              else
                umma_bf16_pair(d_tmem, da + k * 2, dw + k * 2, idesc, (kb | k) != 0 ? 1u : 0u);
            }
            umma_commit_pair(&empty[stage], 0x3);
          }
          __syncwarp();
          issued_any = true;
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (ok && elect) umma_commit_pair(&tfull[acc], 0x3);
        __syncwarp();
      }
      if (issued_any) {
        if (elect) umma_commit_pair(drain, 0x1);
        __syncwarp();
        wait_all(drain, 0);
      }
    }
  } else {
    // ---------------- epilogue (warps 2..9 of both CTAs) ----------------
    constexpr int kHalf = BN / 2;
    constexpr int kChunks = kHalf / 32;
    const int quarter = warp & 3;
    const int col_half = ((warp - 2) >> 2) * kHalf;
    const int row_base = static_cast<int>(rank) * kGemmBM + quarter * 32;  // this warp's 32 rows
    uint8_t *my_staging = staging + (warp - 2) * 2 * S::kChunkBytes;
    // a warp's 8 KB of staging holds two fp32 or four bf16 32 x 32 chunks:
    // that many stores may still be reading it while the next is written
    constexpr bool kF32Out =
        EPI == kEpiF32 || EPI == kEpiF32Resid || EPI == kEpiI8F32 || EPI == kEpiI8Gelu8;
    constexpr int kOutChunk = kF32Out ? S::kChunkBytes : S::kChunkBytes / 2;
    constexpr int kSlots = 2 * S::kChunkBytes / kOutChunk;
    int nstore = 0;  // bulk stores this warp has issued (lane 0)
    int local = 0;
    for (int tile = pair; tile < num_tiles; tile += num_pairs, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(&tfull[acc], acc_phase, p.err))) break;
      tc_fence_after();
      const int mb = tile / n_blocks, nb = tile % n_blocks;
      const int row0 = mb * kPairM + row_base;
      const int row = row0 + lane;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                             static_cast<uint32_t>(acc * BN + col_half);
      uint32_t ra[32], rb[32];
      if constexpr (EPI == kEpiBf16SwiGLU || EPI == kEpiBf16GeGLU) {
        // chunk pairs: 2k = up, 2k + 1 = gate of the same 32 output columns
#pragma unroll
        for (int c = 0; c < kChunks; c += 2) {
          tmem_ld_32x32b_x32(t_row + c * 32, ra);
          tmem_ld_32x32b_x32(t_row + (c + 1) * 32, rb);
          tmem_wait_ld_regs(ra);
          tmem_wait_ld_regs(rb);
          if (c + 2 == kChunks) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(map_to_cta(smem_u32(&tempty[acc]), 0));
          }
          const int col0 = nb * BN + col_half + c * 32;  // GEMM column of the up chunk
          if (row0 < M && col0 < p.N) {  // warp-uniform
            uint8_t *chunk = my_staging + (nstore % kSlots) * kOutChunk;
            if (lane == 0) bulk_wait_group_read<kSlots - 1>();
            __syncwarp();
            epi_stage_glu<EPI>(p, col0, ra, rb, chunk, lane);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              tma_store_2d(&tmC, chunk, col0 / 2, row0);  // output column (col0 / 64) * 32
              bulk_commit_group();
            }
            ++nstore;
          }
        }
        continue;
      }
      if constexpr (EPI == kEpiBf16Rope) {
        // chunk pairs: the two halves (dims 0..31, 32..63) of one head
#pragma unroll
        for (int c = 0; c < kChunks; c += 2) {
          tmem_ld_32x32b_x32(t_row + c * 32, ra);
          tmem_ld_32x32b_x32(t_row + (c + 1) * 32, rb);
          tmem_wait_ld_regs(ra);
          tmem_wait_ld_regs(rb);
          if (c + 2 == kChunks) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(map_to_cta(smem_u32(&tempty[acc]), 0));
          }
          const int col0 = nb * BN + col_half + c * 32;
          if (row0 < M && col0 < p.N) {  // warp-uniform
            uint8_t *c1 = my_staging + (nstore % kSlots) * kOutChunk;
            uint8_t *c2 = my_staging + ((nstore + 1) % kSlots) * kOutChunk;
            if (lane == 0) bulk_wait_group_read<kSlots - 2>();  // both slots free
            __syncwarp();
            if (col0 < p.rope_cols) {
              epi_stage_rope(p, col0, row, M, ra, rb, c1, c2, lane);
            } else {
              epi_stage32<kEpiBf16>(p, col0, ra, c1, lane);
              epi_stage32<kEpiBf16>(p, col0 + 32, rb, c2, lane);
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              tma_store_2d(&tmC, c1, col0, row0);
              bulk_commit_group();
              tma_store_2d(&tmC, c2, col0 + 32, row0);
              bulk_commit_group();
            }
            nstore += 2;
          }
        }
        continue;
      }
      tmem_ld_32x32b_x32(t_row, ra);
      tmem_wait_ld_regs(ra);
#pragma unroll
      for (int c = 0; c < kChunks; ++c) {
        uint32_t(&cur)[32] = (c & 1) ? rb : ra;
        uint32_t(&nxt)[32] = (c & 1) ? ra : rb;
        if (c + 1 < kChunks) tmem_ld_32x32b_x32(t_row + (c + 1) * 32, nxt);
        if (c + 1 == kChunks) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(map_to_cta(smem_u32(&tempty[acc]), 0));
        }
        const int col0 = nb * BN + col_half + c * 32;
        if constexpr (kTmaStore) {
          if (row0 < M && col0 < p.N) {  // warp-uniform
            uint8_t *chunk = my_staging + (nstore % kSlots) * kOutChunk;
            // the store that last read `chunk` is done
            if (lane == 0) bulk_wait_group_read<kSlots - 1>();
            __syncwarp();
            if constexpr (kInt8)
              i8_stage32<EPI == kEpiI8Gelu8, EPI == kEpiI8Bf16>(
                  p.N, p.ws, p.bias, row < M ? __ldg(p.sa + row) : 0.0f, row < M, col0, cur,
                  chunk, lane);
            else
              epi_stage32<EPI>(p, col0, cur, chunk, lane);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              tma_store_2d(&tmC, chunk, col0, row0);
              bulk_commit_group();
            }
            ++nstore;
          }
        } else {
          if (row < M && col0 < p.N) epi_store32<EPI>(p, row, col0, cur);
        }
        if (c + 1 < kChunks) tmem_wait_ld_regs(nxt);
      }
    }
    if (kTmaStore && lane == 0) bulk_wait_group_all();
  }

  tc_fence_before();
  cluster_sync();  // no CTA leaves while its pair may still signal it
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, S::kTmemCols);
  }
}

}  // namespace nebw
