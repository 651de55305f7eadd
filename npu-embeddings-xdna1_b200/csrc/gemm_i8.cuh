// The int8 datapath of the reference's `--dtype i8` containers on the
// sm_100a tensor cores.
//
// The reference's array path quantises each GEMM input per row to int8 with
// its SmoothQuant divisor folded in, multiplies int8 x int8 into int32 on the
// NPU, and dequantises C on the host (app::quantise_a_int8,
// app::dequantise_c, app::dequant_act_quant; runtime/include/common/
// host_kernels.hpp:263-614).  Here:
//
//   quantise_rows_kernel   q = rne(clamp(x * ias * (1 / sc), +-127)),
//                          sc = max|x * ias| / 127 (1 when the row is 0);
//                          one warp per row
//   gemm_i8_kernel         C = A_q . W_q^T in int32 on tcgen05.mma kind::i8
//                          (exact), dequantised in the epilogue as
//                          y = fma(float(C) * sa[row], ws[col], bias[col]),
//                          optionally gelu8(y) (dequant_act_quant's act),
//                          fp32 out -- or bf16 RNE of y for the encoder's
//                          QKV product, which the tensor-core attention reads
//
// The integer product is exact and every floating-point step is the
// reference's single IEEE operation in its order (int -> float round to
// nearest even, the product, one fused multiply-add; the divisions are
// IEEE), so both kernels reproduce the reference's steps bit for bit.  The
// FFN-up step dequant_act_quant is gemm_i8 with gelu8 followed by
// quantise_rows with the next GEMM's divisor.
//
// The GEMM is the single-CTA structure of gemm_tc_kernel (TMA producer warp,
// one MMA-issuing warp, eight epilogue warps, a double-buffered TMEM
// accumulator) with 128-byte K-blocks: 128 int8 per row instead of 64 bf16,
// the same swizzled tiles, four K=32 MMAs per block.  The epilogue stages
// each warp's 32 x 32 output chunks in shared memory, in the output tensor
// map's swizzle, and writes them with TMA bulk-tensor stores (whole-row
// segments, not one 16-byte piece per row per instruction), so an fp32
// output of many columns is written at the HBM rate.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cstdint>

#include "gemm_tc.cuh"
#include "ptx.cuh"

namespace nebw {

constexpr int kGemmI8BK = 128;  // int8 elements per K-block (one 128-byte row)

template <int BN>
struct GemmI8Shape {
  static_assert(BN == 128 || BN == 256, "BN must be 128 or 256");
  static constexpr int kABytes = kGemmBM * kGemmI8BK;  // 16 KB
  static constexpr int kBBytes = BN * kGemmI8BK;       // 16 or 32 KB
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = BN == 256 ? 3 : 5;
  static constexpr int kTmemCols = 2 * BN;
  // epilogue staging: per epilogue warp two fp32 (or four bf16) 32 x 32 chunks
  static constexpr int kChunkBytes = 32 * 32 * 4;
  static constexpr int kStagingBytes = 8 * 2 * kChunkBytes;  // 64 KB
  static constexpr int kBarBytes = 256;
  static constexpr int kSmemBytes = 1024 + kStages * kStageBytes + kStagingBytes + kBarBytes;
  static_assert(kSmemBytes <= 232448, "shared memory per CTA");
};

struct GemmI8Args {
  int M, N, K;
  const int *M_dev;   // if set, the live row count is min(*M_dev, M)
  const float *sa;    // [M] row scales of A (quantise_rows' sc)
  const float *ws;    // [N] column scales of W
  const float *bias;  // [N] or null (then 0)
  float *out;         // [M, N] fp32, or
  __nv_bfloat16 *out_bf16;  // [M, N] bf16 RNE of the dequantised value (out null)
  int *err;
};

__device__ __forceinline__ float widen(float v) { return v; }
__device__ __forceinline__ float widen(__nv_bfloat16 v) { return __bfloat162float(v); }

// One row per warp: quantise_a_int8 (host_kernels.hpp:263-315).  The row
// maximum is order-independent, so the warp reduction gives the reference's
// value exactly; sc = mx / 127 and inv = 1 / sc are IEEE divisions.  x is
// fp32, or bf16 widened exactly (the attention's output); rows past
// *rows_dev (when set) are left alone.
template <typename XT>
__global__ void __launch_bounds__(256)
    quantise_rows_kernel(const XT *__restrict__ x, int rows, const int *__restrict__ rows_dev,
                         int K, const float *__restrict__ ias, int8_t *__restrict__ q,
                         float *__restrict__ scale) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (rows_dev) rows = min(rows, __ldg(rows_dev));
  if (row >= rows) return;
  const XT *xr = x + static_cast<int64_t>(row) * K;
  float mx = 0.0f;
  for (int j = lane; j < K; j += 32) mx = fmaxf(mx, fabsf(widen(xr[j]) * __ldg(ias + j)));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  const float sc = mx > 0.0f ? mx / 127.0f : 1.0f;
  const float inv = 1.0f / sc;
  if (lane == 0) scale[row] = sc;
  int8_t *qr = q + static_cast<int64_t>(row) * K;
  for (int j = lane; j < K; j += 32) {
    const float t = fminf(fmaxf((widen(xr[j]) * __ldg(ias + j)) * inv, -127.0f), 127.0f);
    qr[j] = static_cast<int8_t>(__float2int_rn(t));
  }
}

// The same quantisation with the row held in registers, so that it is read
// from memory once (the form above reads it twice, once for its maximum):
// here one CTA of 256 threads per row, NV float4 (or 4 x bf16) per thread,
// for rows too wide for one warp's registers.  K % 4 == 0, K <= 1024 * NV.
constexpr int kQuantThreads = 256;

__device__ __forceinline__ float4 load_widen4(const float *p) {
  return *reinterpret_cast<const float4 *>(p);
}
__device__ __forceinline__ float4 load_widen4(const __nv_bfloat16 *p) {
  const uint2 u = *reinterpret_cast<const uint2 *>(p);
  return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u),
                     __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xffff0000u));
}

template <typename XT, int NV>
__global__ void __launch_bounds__(kQuantThreads)
    quantise_rows_cta_kernel(const XT *__restrict__ x, int rows, const int *__restrict__ rows_dev,
                             int K, const float *__restrict__ ias, int8_t *__restrict__ q,
                             float *__restrict__ scale) {
  __shared__ float red[kQuantThreads / 32];
  const int row = blockIdx.x, t = threadIdx.x;
  if (rows_dev) rows = min(rows, __ldg(rows_dev));
  if (row >= rows) return;  // CTA-uniform
  const XT *xr = x + static_cast<int64_t>(row) * K;
  float4 v[NV];
  float mx = 0.0f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = (i * kQuantThreads + t) * 4;
    if (c < K) {
      const float4 a = load_widen4(xr + c);
      const float4 s = __ldg(reinterpret_cast<const float4 *>(ias + c));
      v[i] = make_float4(a.x * s.x, a.y * s.y, a.z * s.z, a.w * s.w);  // x * ias, rounded once
      mx = fmaxf(fmaxf(mx, fabsf(v[i].x)), fabsf(v[i].y));
      mx = fmaxf(fmaxf(mx, fabsf(v[i].z)), fabsf(v[i].w));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((t & 31) == 0) red[t >> 5] = mx;
  __syncthreads();
  mx = red[0];
#pragma unroll
  for (int w = 1; w < kQuantThreads / 32; ++w) mx = fmaxf(mx, red[w]);
  const float sc = mx > 0.0f ? mx / 127.0f : 1.0f;
  const float inv = 1.0f / sc;
  if (t == 0) scale[row] = sc;
  int8_t *qr = q + static_cast<int64_t>(row) * K;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = (i * kQuantThreads + t) * 4;
    if (c < K) {
      const float e[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
      uint32_t pk = 0;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float tq = fminf(fmaxf(e[k] * inv, -127.0f), 127.0f);
        pk |= (static_cast<uint32_t>(__float2int_rn(tq)) & 0xffu) << (8 * k);
      }
      *reinterpret_cast<uint32_t *>(qr + c) = pk;
    }
  }
}

// The same with a warp per row and the row in its registers (NV float4, or
// 4 x bf16, per lane): the form for rows of up to 128 * NV values, eight rows
// per CTA.  K % 4 == 0, K <= 128 * NV.
template <typename XT, int NV>
__global__ void __launch_bounds__(256)
    quantise_rows_warp_kernel(const XT *__restrict__ x, int rows, const int *__restrict__ rows_dev,
                              int K, const float *__restrict__ ias, int8_t *__restrict__ q,
                              float *__restrict__ scale) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (rows_dev) rows = min(rows, __ldg(rows_dev));
  if (row >= rows) return;  // warp-uniform
  const XT *xr = x + static_cast<int64_t>(row) * K;
  float4 v[NV];
  float mx = 0.0f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = (i * 32 + lane) * 4;
    if (c < K) {
      const float4 a = load_widen4(xr + c);
      const float4 s = __ldg(reinterpret_cast<const float4 *>(ias + c));
      v[i] = make_float4(a.x * s.x, a.y * s.y, a.z * s.z, a.w * s.w);  // x * ias, rounded once
      mx = fmaxf(fmaxf(mx, fabsf(v[i].x)), fabsf(v[i].y));
      mx = fmaxf(fmaxf(mx, fabsf(v[i].z)), fabsf(v[i].w));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  const float sc = mx > 0.0f ? mx / 127.0f : 1.0f;
  const float inv = 1.0f / sc;
  if (lane == 0) scale[row] = sc;
  int8_t *qr = q + static_cast<int64_t>(row) * K;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = (i * 32 + lane) * 4;
    if (c < K) {
      const float e[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
      uint32_t pk = 0;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float tq = fminf(fmaxf(e[k] * inv, -127.0f), 127.0f);
        pk |= (static_cast<uint32_t>(__float2int_rn(tq)) & 0xffu) << (8 * k);
      }
      *reinterpret_cast<uint32_t *>(qr + c) = pk;
    }
  }
}

// C[M, N] = dequant(A_q[M, K] . W_q[N, K]^T): A and W int8, K-major, read by
// TMA in 128 x 128-byte (A) and BN x 128-byte (W) swizzled boxes; C written
// through tmC (32 x 32 boxes: fp32 with the 128-byte swizzle, or bf16 with
// the 64-byte one, as BF16 says).  One CTA per SM, persistent over 128 x BN
// tiles.  Every wait is bounded.
template <int BN, bool GELU, bool BF16>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_i8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                   const __grid_constant__ CUtensorMap tmC, const GemmI8Args p) {
  using S = GemmI8Shape<BN>;
  constexpr int kStages = S::kStages;
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
  int M = p.M;
  if (p.M_dev) M = min(M, __ldg(p.M_dev));
  const int m_blocks = (M + kGemmBM - 1) / kGemmBM;
  const int n_blocks = (p.N + BN - 1) / BN;
  const int num_tiles = m_blocks * n_blocks;
  const int num_kb = (p.K + kGemmI8BK - 1) / kGemmI8BK;

  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmC);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 8);
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
      uint32_t issued_mask = 0, last_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int mb = tile / n_blocks, nb = tile % n_blocks;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, p.err)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], S::kStageBytes);
          tma_load_2d(sA + stage * S::kABytes, &tmA, &full[stage], kb * kGemmI8BK, mb * kGemmBM);
          tma_load_2d(sW + stage * S::kBBytes, &tmW, &full[stage], kb * kGemmI8BK, nb * BN);
          issued_mask |= 1u << stage;
          last_phase = (last_phase & ~(1u << stage)) | (phase << stage);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      for (int s = 0; s < kStages; ++s)
        if (issued_mask & (1u << s)) mbar_wait(&full[s], (last_phase >> s) & 1u, p.err);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer: four K=32 int8 MMAs per 128-byte block ----
    constexpr uint32_t idesc = idesc_s8_s32(kGemmBM, BN);
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
          for (int k = 0; k < kGemmI8BK / 32; ++k)  // +32 B per 32 int8 of K
            umma_s8(d_tmem, da + k * 2, dw + k * 2, idesc, (kb | k) != 0 ? 1u : 0u);
          umma_commit(&empty[stage]);
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
    if (issued_any) {
      if (elect) umma_commit(drain);
      __syncwarp();
      wait_all(drain, 0);
    }
  } else {
    // ---------------- epilogue (warps 2..9): int32 rows out of TMEM ----------
    constexpr int kHalf = BN / 2;
    constexpr int kChunks = kHalf / 32;
    const int quarter = warp & 3;
    const int col_half = ((warp - 2) >> 2) * kHalf;
    const int row_in_tile = quarter * 32 + lane;
    uint8_t *my_staging = staging + (warp - 2) * 2 * S::kChunkBytes;
    // a warp's 8 KB of staging holds two fp32 or four bf16 32 x 32 chunks:
    // that many stores may still be reading it while the next is written
    constexpr int kOutChunk = BF16 ? S::kChunkBytes / 2 : S::kChunkBytes;
    constexpr int kSlots = 2 * S::kChunkBytes / kOutChunk;
    int nstore = 0;  // bulk stores this warp has issued (lane 0)
    int local = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(&tfull[acc], acc_phase, p.err))) break;
      tc_fence_after();
      const int mb = tile / n_blocks, nb = tile % n_blocks;
      const int row0 = mb * kGemmBM + quarter * 32;  // this warp's 32 rows
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
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tempty[acc]);
        }
        const int col0 = nb * BN + col_half + c * 32;
        if (row0 < M && col0 < p.N) {  // warp-uniform
          uint8_t *chunk = my_staging + (nstore % kSlots) * kOutChunk;
          // the store that last read `chunk` is done
          if (lane == 0) bulk_wait_group_read<kSlots - 1>();
          __syncwarp();
          i8_stage32<GELU, BF16>(p.N, p.ws, p.bias, row < M ? __ldg(p.sa + row) : 0.0f, row < M,
                                 col0, cur, chunk, lane);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmC, chunk, col0, row0);
            bulk_commit_group();
          }
          ++nstore;
        }
        if (c + 1 < kChunks) tmem_wait_ld_regs(nxt);
      }
    }
    if (lane == 0) bulk_wait_group_all();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, S::kTmemCols);
  }
}

}  // namespace nebw
