// Fused masked attention on the 5th-generation tensor cores (head_dim 64).
//
// One CTA per (128-query tile, head, sequence).  For a sequence of length L
// (nk = ceil(L / 128) key blocks, Lc = 128 * nk keys computed):
//
//   TMA     Q [128 x 64], K [Lc x 64], V [Lc x 64] bf16 tiles of the packed
//           Q|K|V rows, 128-byte swizzled (one mbarrier)
//   UMMA    S = Q K^T   (M=128, N=256/128, K=16 steps) into TMEM columns
//           [0, Lc) -- Q is pre-scaled by 1/sqrt(64) (the packer's fold)
//   CUDA    V is transposed in shared memory into the K-major layout the
//           PV product reads, keys >= L written as zero (while S runs)
//   CUDA    exact softmax per query row (the full row is in TMEM): two
//           warpgroups split the key columns, pass 1 the row max, pass 2
//           p = exp2((s - max) log2 e) with keys >= L masked to 0, the row
//           sum, and P as bf16 into shared memory (swizzled K-major, over
//           the now-dead K and V tiles)
//   UMMA    O = P V     (M=128, N=64, K=16 steps) into TMEM columns [0, 64)
//   CUDA    ctx = O / rowsum, bf16, for query rows < L
//
// Replaces qk_impl / softmax_cpu / av_impl (runtime/src/encoders/
// bert_encoder.cpp:995-1135, :481-530): the reference's padded keys get
// weight <= 2^-120 / sum through its -1e30 mask and exp2 floor; here they
// get exactly 0.
//
// Work lists: the encoder pass sorts sequences into length buckets on the
// device (L <= 128, <= 256, <= 512) and launches this kernel once per bucket
// with LP = the bucket's bound, so that short sequences run with a small
// shared-memory and TMEM footprint (3-4 CTAs per SM) and only the longest
// need a whole SM.  With work == nullptr the sequence index is the CTA's z.
//
// Every wait is bounded (kWaitTimeoutNs); on timeout the CTA records an
// error, drains what it issued with bounded waits, frees TMEM and returns.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cstdint>

#include "ptx.cuh"

namespace nebw {

constexpr int kAttnTcThreads = 256;  // two warpgroups
constexpr int kAttnTcD = 64;

template <int LP>
struct AttnTcShape {
  static_assert(LP == 128 || LP == 256 || LP == 512, "bucket bound must be 128, 256 or 512");
  static constexpr int kQBytes = 128 * 128;  // 128 rows x 64 bf16
  static constexpr int kKBytes = LP * 128;   // LP keys x 64 bf16
  static constexpr int kVBytes = LP * 128;   // V staging, same shape
  static constexpr int kVtBytes = LP * 128;  // 64 d-rows x LP keys
  // P (128 rows x LP keys bf16 = kKBytes + kVBytes) overlays K and V.
  static constexpr int kRedBytes = 4 * 128 * 4;
  static constexpr int kBarBytes = 64;
  static constexpr int kSmemBytes =
      1024 + kQBytes + kKBytes + kVBytes + kVtBytes + kRedBytes + kBarBytes;
  static constexpr uint32_t kTmemCols = LP;  // S: one fp32 column per key
};

__device__ __forceinline__ void attn_named_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kAttnTcThreads) : "memory");
}

template <int LP>
__global__ void __launch_bounds__(kAttnTcThreads, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tmQKV, const int *__restrict__ seq_off,
                        const int *__restrict__ seq_len, const int *__restrict__ work,
                        const int *__restrict__ work_count, int H, __nv_bfloat16 *__restrict__ ctx,
                        int *err) {
  using S = AttnTcShape<LP>;
  const int item = blockIdx.z;
  if (work_count && item >= __ldg(work_count)) return;
  const int b = work ? __ldg(work + item) : item;
  const int h = blockIdx.y;
  const int L = __ldg(seq_len + b);
  const int q0 = blockIdx.x * 128;
  if (q0 >= L) return;
  const int base = __ldg(seq_off + b);
  const int nk = min((L + 127) >> 7, LP / 128);
  const int Lc = nk * 128;

  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t *sQ = smem;
  uint8_t *sK = sQ + S::kQBytes;
  uint8_t *sV = sK + S::kKBytes;
  uint8_t *sVt = sV + S::kVBytes;
  uint8_t *sP = sK;  // overlays K and V once both are consumed
  float *red = reinterpret_cast<float *>(sVt + S::kVtBytes);  // [4][128]
  uint64_t *bars = reinterpret_cast<uint64_t *>(red + 4 * 128);
  uint64_t *bar_ld = bars, *bar_s = bars + 1, *bar_o = bars + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 4);

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int wg = warp >> 2;                  // warpgroup: key-column half
  const int r = (warp & 3) * 32 + lane;      // this thread's TMEM lane = query row in tile

  if (tid == 0) {
    tma_prefetch_desc(&tmQKV);
    mbar_init(bar_ld, 1);
    mbar_init(bar_s, 1);
    mbar_init(bar_o, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, S::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // ---- loads ----
  if (tid == 0) {
    mbar_arrive_expect_tx(bar_ld, S::kQBytes + nk * 2 * 128 * 128);
    tma_load_2d(sQ, &tmQKV, bar_ld, h * kAttnTcD, base + q0);
    for (int kb = 0; kb < nk; ++kb) {
      tma_load_2d(sK + kb * 16384, &tmQKV, bar_ld, H + h * kAttnTcD, base + kb * 128);
      tma_load_2d(sV + kb * 16384, &tmQKV, bar_ld, 2 * H + h * kAttnTcD, base + kb * 128);
    }
  }
  bool ok = mbar_wait(bar_ld, 0, err);

  // ---- S = Q K^T ----
  bool issued = false;
  if (tid == 0 && ok) {
    tc_fence_after();
    const uint32_t q_addr = smem_u32(sQ);
    for (int jb = 0; jb < nk; jb += 2) {
      const bool wide = jb + 1 < nk;
      const uint32_t idesc = wide ? idesc_bf16_f32(128, 256) : idesc_bf16_f32(128, 128);
      const uint32_t k_addr = smem_u32(sK + jb * 16384);
#pragma unroll
      for (int k = 0; k < kAttnTcD / 16; ++k)
        umma_bf16(tmem + static_cast<uint32_t>(jb * 128), sdesc_kmajor_sw128(q_addr + k * 32),
                  sdesc_kmajor_sw128(k_addr + k * 32), idesc, k > 0 ? 1u : 0u);
    }
    umma_commit(bar_s);
    issued = true;
  }

  // ---- V^T (overlaps the S product) ----
  // item = (key octet jo, d octet dq): 8 keys x 8 dims transposed in registers
  if (ok) {
    for (int it = tid; it < Lc; it += kAttnTcThreads) {
      const int jo = it >> 3, dq = it & 7;
      const int j0 = jo * 8;
      uint32_t w[8][4];
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const int j = j0 + kk;
        const uint4 x = *reinterpret_cast<const uint4 *>(sV + j * 128 + ((dq ^ (j & 7)) << 4));
        const bool valid = j < L;
        w[kk][0] = valid ? x.x : 0u;
        w[kk][1] = valid ? x.y : 0u;
        w[kk][2] = valid ? x.z : 0u;
        w[kk][3] = valid ? x.w : 0u;
      }
      uint8_t *blk = sVt + (j0 >> 6) * 8192;
      const int piece = (j0 & 63) >> 3;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int d = dq * 8 + 2 * q + e;
          const uint32_t sel = e ? 0x7632u : 0x5410u;
          uint4 o;
          o.x = __byte_perm(w[0][q], w[1][q], sel);
          o.y = __byte_perm(w[2][q], w[3][q], sel);
          o.z = __byte_perm(w[4][q], w[5][q], sel);
          o.w = __byte_perm(w[6][q], w[7][q], sel);
          *reinterpret_cast<uint4 *>(blk + d * 128 + ((piece ^ (d & 7)) << 4)) = o;
        }
      }
    }
  }
  __syncthreads();  // V staging consumed, V^T written

  ok = __syncthreads_and(ok ? mbar_wait(bar_s, 0, err) : 0);
  tc_fence_after();

  constexpr float kLog2e = 1.4426950408889634f;
  const int c_lo = wg * (Lc >> 6), c_hi = c_lo + (Lc >> 6);  // 32-column chunks of this warpgroup
  const uint32_t t_row = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
  float inv_sum = 0.f;
  if (ok) {
    // pass 1: row max over keys < L
    float mx = -INFINITY;
    for (int c = c_lo; c < c_hi; ++c) {
      uint32_t v[32];
      tmem_ld_32x32b_x32(t_row + c * 32, v);
      tmem_wait_ld_regs(v);
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (c * 32 + i < L) mx = fmaxf(mx, __uint_as_float(v[i]));
    }
    red[wg * 128 + r] = mx;
    attn_named_sync();
    const float m = fmaxf(red[r], red[128 + r]);
    const float m2 = m * kLog2e;
    // pass 2: p, row sum, P (bf16) into the swizzled K-major A tile
    float sum = 0.f;
    for (int c = c_lo; c < c_hi; ++c) {
      uint32_t v[32];
      tmem_ld_32x32b_x32(t_row + c * 32, v);
      tmem_wait_ld_regs(v);
      uint32_t pk[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int j = c * 32 + 2 * i;
        const float p0 = j < L ? exp2f(fmaf(__uint_as_float(v[2 * i]), kLog2e, -m2)) : 0.f;
        const float p1 = j + 1 < L ? exp2f(fmaf(__uint_as_float(v[2 * i + 1]), kLog2e, -m2)) : 0.f;
        sum += p0 + p1;
        pk[i] = pack_bf16x2(p0, p1);
      }
      uint8_t *row = sP + (c >> 1) * 16384 + r * 128;
      const int p0 = (c & 1) * 4;
#pragma unroll
      for (int q = 0; q < 4; ++q)
        *reinterpret_cast<uint4 *>(row + (((p0 + q) ^ (r & 7)) << 4)) =
            make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
    }
    red[256 + wg * 128 + r] = sum;
  }
  tc_fence_before();
  fence_proxy_async_smem();
  __syncthreads();
  if (ok) inv_sum = 1.0f / (red[256 + r] + red[384 + r]);

  // ---- O = P V ----
  bool issued_o = false;
  if (tid == 0 && ok) {
    tc_fence_after();
    const uint32_t idesc = idesc_bf16_f32(128, kAttnTcD);
    const uint32_t p_addr = smem_u32(sP), vt_addr = smem_u32(sVt);
    for (int s = 0; s < Lc / 16; ++s) {
      const int kb = s >> 2, ks = s & 3;
      umma_bf16(tmem, sdesc_kmajor_sw128(p_addr + kb * 16384 + ks * 32),
                sdesc_kmajor_sw128(vt_addr + kb * 8192 + ks * 32), idesc, s > 0 ? 1u : 0u);
    }
    umma_commit(bar_o);
    issued_o = true;
  }
  ok = __syncthreads_and(ok ? mbar_wait(bar_o, 0, err) : 0);
  tc_fence_after();

  if (ok) {
    uint32_t v[32];
    tmem_ld_32x32b_x32(t_row + wg * 32, v);
    tmem_wait_ld_regs(v);
    const int q = q0 + r;
    if (q < L) {
      uint4 *dst = reinterpret_cast<uint4 *>(ctx + static_cast<int64_t>(base + q) * H + h * kAttnTcD +
                                             wg * 32);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint4 o;
        o.x = pack_bf16x2(__uint_as_float(v[8 * i + 0]) * inv_sum, __uint_as_float(v[8 * i + 1]) * inv_sum);
        o.y = pack_bf16x2(__uint_as_float(v[8 * i + 2]) * inv_sum, __uint_as_float(v[8 * i + 3]) * inv_sum);
        o.z = pack_bf16x2(__uint_as_float(v[8 * i + 4]) * inv_sum, __uint_as_float(v[8 * i + 5]) * inv_sum);
        o.w = pack_bf16x2(__uint_as_float(v[8 * i + 6]) * inv_sum, __uint_as_float(v[8 * i + 7]) * inv_sum);
        dst[i] = o;
      }
    }
  }

  // Teardown: whatever this CTA issued has completed before TMEM is freed
  // (already true on the normal path; bounded waits on the error path).
  if (tid == 0 && !ok) {
    mbar_wait(bar_ld, 0, err);
    if (issued) mbar_wait(bar_s, 0, err);
    if (issued_o) mbar_wait(bar_o, 0, err);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, S::kTmemCols);
  }
}

// Length buckets for the attention launches: list[k] holds the sequences
// with L in (bound[k-1], bound[k]], bound = {128, 256, 512}; count[k] their
// number.  One CTA, B <= 65535.
__global__ void __launch_bounds__(1024)
    attn_bucket_kernel(const int *__restrict__ seq_len, int B, int *__restrict__ lists,
                       int *__restrict__ counts) {
  __shared__ int cnt[3];
  if (threadIdx.x < 3) cnt[threadIdx.x] = 0;
  __syncthreads();
  for (int b = threadIdx.x; b < B; b += blockDim.x) {
    const int L = seq_len[b];
    const int k = L <= 128 ? 0 : (L <= 256 ? 1 : 2);
    const int slot = atomicAdd(&cnt[k], 1);
    lists[k * B + slot] = b;
  }
  __syncthreads();
  if (threadIdx.x < 3) counts[threadIdx.x] = cnt[threadIdx.x];
}

}  // namespace nebw
