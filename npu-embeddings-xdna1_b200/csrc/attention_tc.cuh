// Fused masked attention on the 5th-generation tensor cores, head_dim D of
// 64 (bge-base/large, ViT-base) or 32 (MiniLM, bge-small).
//
// Persistent CTAs over (sequence, 128-query tile, head) work items,
// flash-style over key blocks of up to 64 with an online softmax,
// warp-specialised so that loads, tensor-core products and the softmax of
// different key blocks (and of consecutive items) overlap:
//
//   warp 0      TMA: the Q tile once per item through a 2-slot ring (the
//               next item's Q lands while this one runs), then K_j and V_j
//               (64-key tiles) of the packed Q|K|V rows (128-byte swizzled
//               for D 64, 64-byte for D 32) in issue order through a 3-slot
//               ring
//   warp 1      tcgen05.mma from one elected lane (the whole warp walks the
//               schedule, so loop state and descriptors stay warp-uniform),
//               software-pipelined inside an
//               item so that the softmax of key block j can start before
//               P_j-1 V_j-1 runs (an item's last P V is issued as soon as its
//               P is written):
//                 S_j  = Q K_j^T  (M=128, N = the block's valid keys rounded
//                                  up to 16, K=16 x D/16)  -> TMEM [0, 64)
//                 O += P_j-1 V_j-1 (M=128, N=D, K = 16 x that block's
//                                  N/16; V read MN-major)  -> TMEM [64, 64+D)
//   warps 2-5   one query row per thread (its TMEM lane); a warp whose 32
//               rows all lie past the sequence only keeps the barrier
//               protocol.  S_j is read from TMEM once, into registers; row
//               max over its valid keys; p = 2^(s log2 e - m log2 e) on the
//               SFU (packed fp32 FMAs for the argument and the running sum),
//               P_j as bf16 into shared memory (swizzled K-major, the UMMA A
//               layout).  O accumulates in TMEM; the max m that p is taken
//               against is raised (and O and the sum rescaled in place) only
//               when a row's max grows past it by more than a factor 2^8,
//               so p <= 2^8 and O is rarely touched before the end, where
//               ctx = O / sum as bf16, staged through shared memory into
//               whole 2D-byte row slices per store
//
// Only the valid keys of a block are multiplied and exponentiated (in
// 16-key groups), so short sequences -- most of an embedding batch -- cost
// what their length needs rather than a full 128 x 64 tile.
//
// 72 KB (D 64) or 44 KB (D 32) of shared memory, 128 TMEM columns and 96
// registers per thread per CTA (three CTAs of 18 warps put five warps on one
// SM sub-partition, whose 16K registers allow 96 a thread), so three CTAs
// share an SM (three softmax warps per SM sub-partition) and one's softmax
// overlaps the others' waits on loads and products; the 64-key block is what
// makes the third CTA fit.  Q is pre-scaled by 1/sqrt(D) (the packer's fold,
// tools/pack/pack_npue.py:2742-2750); no scale is applied here.
//
// Replaces qk_impl / softmax_cpu / av_impl (runtime/src/encoders/
// bert_encoder.cpp:995-1135, :481-530).  The reference's padded keys carry
// weight <= 2^-120 / sum through its -1e30 mask and exp2 floor; here they
// carry exactly 0, and keys of a partial last block that belong to the next
// sequence are masked by index.
//
// Every wait is bounded (kWaitTimeoutNs); on timeout the CTA records an
// error in the device error word, drains what it issued with bounded waits,
// frees TMEM and returns.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cstdint>

#include "ptx.cuh"

namespace nebw {

constexpr int kAttnTcThreads = 192;  // TMA warp, MMA warp, 4 softmax warps
constexpr int kAttnTcKeys = 64;       // keys per block
constexpr int kAttnTcTmemCols = 128;  // S [0,64), O [64, 64 + head_dim)

// head_dim the tcgen05 kernel is built for: 64 (bge-base/large, ViT-base)
// and 32 (MiniLM, bge-small).  Rows of a 64-wide head tile are 128 bytes
// (128-byte swizzle), of a 32-wide one 64 bytes (64-byte swizzle).
__host__ __device__ constexpr bool attn_tc_head_dim(int d) { return d == 32 || d == 64; }

template <int D>
struct AttnTcShape {
  static_assert(attn_tc_head_dim(D), "head_dim 32 or 64");
  static constexpr int kTile = 128 * D * 2;             // one 128 x D bf16 Q tile
  static constexpr int kKvTile = kAttnTcKeys * D * 2;   // one 64 x D bf16 K or V tile
  static constexpr int kQSlots = 2, kKvSlots = 3;
  static constexpr int kQ0 = 0;                     // Q ring: 2 slots
  static constexpr int kKv0 = kQSlots * kTile;      // K/V ring: 3 slots, K_j V_j K_j+1 ...
  static constexpr int kP = kKv0 + kKvSlots * kKvTile;  // P, 16 KB (128 rows x 64 keys)
  static constexpr int kBars = kP + 16384;          // barriers
  static constexpr int kSmemBytes = kBars + 256;    // 73,984 B (D 64) / 45,312 B (D 32)
  static_assert(kKv0 % 1024 == 0 && kP % 1024 == 0 && kKvTile % 1024 == 0,
                "swizzled tiles stay 1 KB aligned");
};

// Shared-memory descriptors of the head tiles: K-major Q and K, MN-major V.
template <int D>
__device__ __forceinline__ uint64_t attn_desc_kmajor(uint32_t a) {
  return D == 64 ? sdesc_kmajor_sw128(a) : sdesc_kmajor_sw64(a);
}
template <int D>
__device__ __forceinline__ uint64_t attn_desc_v(uint32_t a) {
  return D == 64 ? sdesc_mnmajor_sw128(a) : sdesc_mnmajor_sw64(a);
}

template <typename T>
__device__ __forceinline__ T *smem_at(uint8_t *base, int off) {
  return reinterpret_cast<T *>(base + off);
}

// One unit of attention work: query tile `qt` of sequence `b` (all heads).
// Encoded as (b << 8) | qt in the work list attn_work_kernel builds.
struct AttnItem {
  int b, qt;
};

__device__ __forceinline__ AttnItem attn_item(const int *items, int item, int qtiles) {
  if (items) {
    const int e = __ldg(items + item);
    return {e >> 8, e & 255};
  }
  return {item / qtiles, item % qtiles};
}

// Valid keys of key block j of a sequence of length L, rounded up to 16 (the
// UMMA N granularity at M = 128 and the K step of P V).
__device__ __forceinline__ int attn_block_cols(int L, int j) {
  return (min(kAttnTcKeys, L - j * kAttnTcKeys) + 15) & ~15;
}

// Persistent: each CTA walks work indices w = blockIdx.x, +gridDim.x, ...
// over n_items x heads (w -> item w / heads, head w % heads), keeping the
// load / product / softmax pipeline running across items.  With `items`
// null, the items are every (b, qt < qtiles) and tiles past a sequence's
// length are skipped.
template <int D>
__global__ void __launch_bounds__(kAttnTcThreads, 3)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tmQKV,
                        const __grid_constant__ CUtensorMap tmKV, const int *__restrict__ seq_off,
                        const int *__restrict__ seq_len, const int *__restrict__ items,
                        const int *__restrict__ items_count, int n_items_host, int qtiles,
                        int heads, __nv_bfloat16 *__restrict__ ctx, int *err) {
  using S = AttnTcShape<D>;
  const int H = heads * D;
  const int n_items = items_count ? __ldg(items_count) : n_items_host;
  const int n_work = n_items * heads;

  extern __shared__ __align__(1024) uint8_t smem[];
  if (reinterpret_cast<uintptr_t>(smem) & 1023) {  // swizzled tiles need 1 KB alignment
    if (threadIdx.x == 0) record_err(err, kDevBadShape);
    return;
  }
  uint64_t *bars = smem_at<uint64_t>(smem, S::kBars);
  uint64_t *q_full = bars + 0;    // [2]
  uint64_t *q_empty = bars + 2;   // [2]
  uint64_t *kv_full = bars + 4;   // [3]
  uint64_t *kv_empty = bars + 7;  // [3]
  uint64_t *s_full = bars + 10, *s_free = bars + 11;
  uint64_t *p_full = bars + 12;
  uint64_t *o_full = bars + 13;
  uint64_t *drain = bars + 14;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 15);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmQKV);
    tma_prefetch_desc(&tmKV);
    for (int s = 0; s < S::kQSlots; ++s) {
      mbar_init(q_full + s, 1);
      mbar_init(q_empty + s, 1);
    }
    for (int s = 0; s < S::kKvSlots; ++s) {
      mbar_init(kv_full + s, 1);
      mbar_init(kv_empty + s, 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_free, 4);
    mbar_init(p_full, 4);
    mbar_init(o_full, 1);
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kAttnTcTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tO = tmem + kAttnTcKeys;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    // Q through a 2-slot ring (the next item's Q lands while this item
    // runs), K_j and V_j in issue order through a 3-slot ring; a slot is
    // reloaded once the MMA that read it has completed (its empty barrier).
    if (lane == 0) {
      bool ok = true;
      int t = 0, g = 0;  // Q loads and K/V loads issued
      for (int w = blockIdx.x; w < n_work && ok; w += gridDim.x) {
        const AttnItem it = attn_item(items, w / heads, qtiles);
        const int h = w % heads;
        const int L = __ldg(seq_len + it.b), q0 = it.qt * 128;
        if (q0 >= L) continue;
        const int base = __ldg(seq_off + it.b), nk = (L + kAttnTcKeys - 1) / kAttnTcKeys;
        {
          const int qs = t % S::kQSlots;
          if (!mbar_wait(q_empty + qs, ((t / S::kQSlots) & 1) ^ 1u, err)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(q_full + qs, S::kTile);
          tma_load_2d(smem + S::kQ0 + qs * S::kTile, &tmQKV, q_full + qs, h * D, base + q0);
          ++t;
        }
        for (int j = 0; j < nk && ok; ++j) {
          for (int kv = 0; kv < 2; ++kv, ++g) {  // K_j, then V_j
            const int ss = g % S::kKvSlots;
            if (!mbar_wait(kv_empty + ss, ((g / S::kKvSlots) & 1) ^ 1u, err)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(kv_full + ss, S::kKvTile);
            tma_load_2d(smem + S::kKv0 + ss * S::kKvTile, &tmKV, kv_full + ss,
                        (1 + kv) * H + h * D, base + j * kAttnTcKeys);
          }
        }
      }
      if (ok) {
        // every load issued has been consumed (so it landed) before exit
        for (int k = 0; k < S::kKvSlots; ++k, ++g)
          if (!mbar_wait(kv_empty + g % S::kKvSlots, ((g / S::kKvSlots) & 1) ^ 1u, err)) break;
        for (int k = 0; k < S::kQSlots; ++k, ++t)
          if (!mbar_wait(q_empty + t % S::kQSlots, ((t / S::kQSlots) & 1) ^ 1u, err)) break;
      } else {
        // wait (bounded) for the copies still in flight to land
        for (int k = g - 1; k >= 0 && k >= g - S::kKvSlots; --k)
          mbar_wait(kv_full + k % S::kKvSlots, (k / S::kKvSlots) & 1, err);
        for (int k = t - 1; k >= 0 && k >= t - S::kQSlots; --k)
          mbar_wait(q_full + k % S::kQSlots, (k / S::kQSlots) & 1, err);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    // The whole warp walks the schedule and waits (so that the loop state
    // and the descriptors are warp-uniform); one elected lane issues the
    // tcgen05 instructions.
    constexpr uint32_t idO = idesc_bf16_f32(128, D) | (1u << 16);  // B (V) MN-major
    const uint32_t pa = smem_u32(smem + S::kP);
    const bool leader = elect_one_sync();
    auto wait_all = [&](uint64_t *bar, uint32_t parity) -> bool {
      return __all_sync(0xffffffffu, mbar_wait(bar, parity, err));
    };
    bool ok = true, issued = false;
    int gb = 0, t = 0, g = 0;  // key blocks, Q slots and K/V slots consumed
    int pend_b = -1, pend_cols = 0, pend_v = 0;  // the P V still to issue
    bool pend_first = false;
    // O (+)= P_b V_b over the block's `cols` keys, V in K/V sequence slot
    // vq; an item's first block overwrites O.  The softmax warps' reads of
    // O (rescale, the previous item's output) precede their p_full arrive.
    auto issue_pv = [&](int b, int cols, int vq, bool first) -> bool {
      const int vs = vq % S::kKvSlots;
      if (!wait_all(kv_full + vs, (vq / S::kKvSlots) & 1) || !wait_all(p_full, b & 1)) return false;
      tc_fence_after();
      const uint64_t da = sdesc_kmajor_sw128(pa);
      const uint64_t db = attn_desc_v<D>(smem_u32(smem + S::kKv0 + vs * S::kKvTile));
      if (leader) {
        // descriptor start addresses advance in 16-byte units: P by 32 B per
        // 16 keys, V by 16 rows of 2 D bytes per 16 keys
#pragma unroll
        for (int ks = 0; ks < kAttnTcKeys / 16; ++ks)
          if (ks < cols / 16)
            umma_bf16(tO, da + ks * 2, db + ks * (2 * D), idO, (!first || ks > 0) ? 1u : 0u);
        umma_commit(o_full);
        umma_commit(kv_empty + vs);
      }
      __syncwarp();
      return true;
    };
    for (int w = blockIdx.x; w < n_work && ok; w += gridDim.x) {
      const AttnItem it = attn_item(items, w / heads, qtiles);
      const int L = __ldg(seq_len + it.b);
      if (it.qt * 128 >= L) continue;
      const int nk = (L + kAttnTcKeys - 1) / kAttnTcKeys;
      const int qs = t % S::kQSlots;
      if (!wait_all(q_full + qs, (t / S::kQSlots) & 1)) {
        ok = false;
        break;
      }
      ++t;
      const uint64_t dq = attn_desc_kmajor<D>(smem_u32(smem + S::kQ0 + qs * S::kTile));
      for (int j = 0; j < nk; ++j, ++gb, g += 2) {
        const int ks = g % S::kKvSlots;  // K_j at sequence g, V_j at g + 1
        const int cols = attn_block_cols(L, j);
        ok = wait_all(kv_full + ks, (g / S::kKvSlots) & 1) &&
             (gb == 0 || wait_all(s_free, (gb - 1) & 1));
        if (!ok) break;
        tc_fence_after();
        const uint64_t dk = attn_desc_kmajor<D>(smem_u32(smem + S::kKv0 + ks * S::kKvTile));
        const uint32_t idS = idesc_bf16_f32(128, cols);
        if (leader) {
#pragma unroll
          for (int k = 0; k < D / 16; ++k)  // +32 B per 16 elements of K
            umma_bf16(tS, dq + k * 2, dk + k * 2, idS, k > 0 ? 1u : 0u);
          umma_commit(s_full);
          umma_commit(kv_empty + ks);
          if (j == nk - 1) umma_commit(q_empty + qs);  // this item's Q is no longer read
        }
        __syncwarp();
        issued = true;
        if (pend_b >= 0 && !(ok = issue_pv(pend_b, pend_cols, pend_v, pend_first))) break;
        pend_b = gb;
        pend_cols = cols;
        pend_v = g + 1;
        pend_first = j == 0;
      }
      // the item's last P V goes out now rather than behind the next
      // item's loads: the softmax warps wait for it to write ctx
      if (ok && !(ok = issue_pv(pend_b, pend_cols, pend_v, pend_first))) break;
      pend_b = -1;
    }
    if (issued) {
      if (leader) umma_commit(drain);
      __syncwarp();
      wait_all(drain, 0);
    }
  } else {
    // ---------------- softmax and output (warps 2..5) ----------------
    // S_j is read from TMEM once, into registers (and S released at once, so
    // QK^T of the next block runs during this block's exponentials).  The
    // probabilities are taken against m_used, a running row max that is
    // only raised when the block's max exceeds it by more than 2^8 (in
    // base 2); then O in TMEM and the running sum are rescaled.  So
    // p <= 2^8, and after the first block O is rarely touched until the end.
    constexpr float kLog2e = 1.4426950408889634f;
    constexpr float kRescaleLog2 = 8.0f;
    const int w4 = warp & 3;
    const int r = w4 * 32 + lane;  // TMEM lane = query row within the tile
    const uint32_t lane_off = static_cast<uint32_t>(w4 * 32) << 16;
    uint8_t *prow = smem + S::kP + r * 128;
    const uint64_t log2e2 = pk2(kLog2e, kLog2e);
    bool ok = true;
    int g = 0;
    for (int w = blockIdx.x; w < n_work && ok; w += gridDim.x) {
      const AttnItem it = attn_item(items, w / heads, qtiles);
      const int h = w % heads;
      const int L = __ldg(seq_len + it.b), q0 = it.qt * 128;
      if (q0 >= L) continue;
      const int base = __ldg(seq_off + it.b), nk = (L + kAttnTcKeys - 1) / kAttnTcKeys;
      // warp-uniform: does any of this warp's 32 query rows belong to the sequence?
      const bool active = q0 + w4 * 32 < L;
      float m_used = -INFINITY, l = 0.f;
      for (int j = 0; j < nk; ++j, ++g) {
        if (!__all_sync(0xffffffffu, mbar_wait(s_full, g & 1, err))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int n = min(kAttnTcKeys, L - j * kAttnTcKeys);  // valid keys of this block
        const int nf = n >> 4;                // whole 16-key groups
        const int vl = n & 15;                // valid keys of a partial last group (0: none)
        constexpr int kG = kAttnTcKeys / 16;  // groups per block
        // s[c]: whole group c; a partial last group (then nf <= kG - 1) in s[kG - 1]
        uint32_t s[kG][16];
        if (active) {
#pragma unroll
          for (int c = 0; c < kG; ++c)
            if (c < nf) tmem_ld_32x32b_x16(tS + lane_off + c * 16, s[c]);
          if (vl) tmem_ld_32x32b_x16(tS + lane_off + nf * 16, s[kG - 1]);
          tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < kG; ++c)
            if (c < nf) pin_regs(s[c]);
          if (vl) pin_regs(s[kG - 1]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(s_free);  // S is in registers: the next QK^T may overwrite it
        float m_new = m_used;
        if (active) {
          // keys of the partial group past the valid ones -> -inf, so that
          // they neither raise the max nor (2^-inf = 0) add to P
          if (vl) {
#pragma unroll
            for (int i = 0; i < 16; ++i) s[kG - 1][i] = i < vl ? s[kG - 1][i] : 0xff800000u;
          }
          // row max, four independent chains of three-input maxima
          float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
          for (int c = 0; c < kG; ++c)
            if (c < nf) {
#pragma unroll
              for (int i = 0; i < 16; i += 2)
                m4[(i >> 1) & 3] = fmax3(m4[(i >> 1) & 3], __uint_as_float(s[c][i]),
                                         __uint_as_float(s[c][i + 1]));
            }
          if (vl) {
#pragma unroll
            for (int i = 0; i < 16; i += 2)
              m4[(i >> 1) & 3] = fmax3(m4[(i >> 1) & 3], __uint_as_float(s[kG - 1][i]),
                                       __uint_as_float(s[kG - 1][i + 1]));
          }
          m_new = fmax3(m_used, fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
        }
        const bool grow = __any_sync(0xffffffffu, active && (m_new - m_used) * kLog2e > kRescaleLog2);
        if (j > 0) {
          // P_j-1 V_j-1 has completed: the P tile is free and O is current
          if (!__all_sync(0xffffffffu, mbar_wait(o_full, (g - 1) & 1, err))) {
            ok = false;
            break;
          }
          tc_fence_after();
        }
        if (grow) {  // warp-uniform; every lane of the warp moves to its own new max
          const float sc = ex2_approx((m_used - m_new) * kLog2e);
          if (j > 0) {
            // 16 columns at a time: S_j is still held in 128 registers
#pragma unroll 1
            for (int q = 0; q < D / 16; ++q) {
              uint32_t va[16];
              tmem_ld_32x32b_x16(tO + lane_off + q * 16, va);
              tmem_wait_ld_regs(va);
#pragma unroll
              for (int i = 0; i < 16; ++i) va[i] = __float_as_uint(__uint_as_float(va[i]) * sc);
              tmem_st_32x32b_x16(tO + lane_off + q * 16, va);
            }
            tmem_wait_st();
          }
          l *= sc;
          m_used = m_new;
        }
        if (active) {
          // p, running sum, P (bf16) into the shared A tile, 8 keys at a
          // time as one swizzled 16-byte chunk; two packed partial sums
          const float m2 = m_used * kLog2e;
          const uint64_t negm2 = pk2(-m2, -m2);
          uint64_t acc2[2] = {pk2(0.f, 0.f), pk2(0.f, 0.f)};
          // the 16 keys of group c
          auto exp_group = [&](const uint32_t(&v)[16], int c) {
            uint8_t *blk = prow;
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
              uint32_t pk[4];
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const int k = hf * 8 + 2 * i;
                float x0, x1;
                unpk2(fma_x2(pk2(__uint_as_float(v[k]), __uint_as_float(v[k + 1])), log2e2, negm2),
                      x0, x1);
                const float p0 = ex2_approx(x0), p1 = ex2_approx(x1);  // 0 past the valid keys
                acc2[i & 1] = add_x2(acc2[i & 1], pk2(p0, p1));
                pk[i] = pack_bf16x2(p0, p1);
              }
              *reinterpret_cast<uint4 *>(blk + ((((c & 3) * 2 + hf) ^ (r & 7)) << 4)) =
                  make_uint4(pk[0], pk[1], pk[2], pk[3]);
            }
          };
#pragma unroll
          for (int c = 0; c < kG; ++c)
            if (c < nf) exp_group(s[c], c);
          if (vl) exp_group(s[kG - 1], nf);
          float a0, a1;
          unpk2(add_x2(acc2[0], acc2[1]), a0, a1);
          l += a0 + a1;
        }
        tc_fence_before();
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(p_full);  // P written (and O rescaled): P_j V_j may start
      }
      if (!ok || !__all_sync(0xffffffffu, mbar_wait(o_full, (g - 1) & 1, err))) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (active) {
        // ctx rows = O / sum as bf16, staged through this warp's own 32
        // rows of the P tile (free: the last P V has completed) so that
        // each global store writes whole 2D-byte row slices
        const float inv = 1.0f / l;
#pragma unroll 1
        for (int q = 0; q < D / 16; ++q) {
          uint32_t va[16];
          tmem_ld_32x32b_x16(tO + lane_off + q * 16, va);
          tmem_wait_ld_regs(va);
          uint32_t pk[8];
#pragma unroll
          for (int i = 0; i < 8; ++i)
            pk[i] = pack_bf16x2(__uint_as_float(va[2 * i]) * inv, __uint_as_float(va[2 * i + 1]) * inv);
          *reinterpret_cast<uint4 *>(prow + (((2 * q) ^ (r & 7)) << 4)) =
              make_uint4(pk[0], pk[1], pk[2], pk[3]);
          *reinterpret_cast<uint4 *>(prow + (((2 * q + 1) ^ (r & 7)) << 4)) =
              make_uint4(pk[4], pk[5], pk[6], pk[7]);
        }
        __syncwarp();
        constexpr int kChunks = D / 8;          // 16-byte chunks of a row slice
        constexpr int kRowsPer = 32 / kChunks;  // rows one warp-wide store covers
        const int ch = lane % kChunks;
#pragma unroll
        for (int i = 0; i < kChunks; ++i) {
          const int rr = w4 * 32 + kRowsPer * i + lane / kChunks;  // query row within the tile
          if (q0 + rr < L)
            *reinterpret_cast<uint4 *>(ctx + static_cast<int64_t>(base + q0 + rr) * H + h * D +
                                       ch * 8) =
                *reinterpret_cast<const uint4 *>(smem + S::kP + rr * 128 + ((ch ^ (rr & 7)) << 4));
        }
        __syncwarp();
      }
      // O reads are complete before this warp's next p_full arrive (the
      // fence there orders them before the next item's first P V)
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kAttnTcTmemCols);
  }
}

// The attention work list: one item per (sequence, 128-query tile), longest
// length class first (L > 256, then > 128, then the rest) so that the
// heaviest items start first and the tail of the persistent loop is short
// work; items[k] = (b << 8) | qt, count[0] = the number of items.  Built by
// block 0; B <= 65535, L <= 32767.
//
// Blocks past the first (when T_dev is set) zero the rows [T, min(rows,
// T256 + kAttnTcKeys)) of the Q|K|V buffer and of the QKV GEMM's A operand,
// T = *T_dev the packed row count and T256 = T rounded up to the CTA-pair
// GEMM's 256 rows.  The last sequence's partial 16-key group multiplies V
// rows past T by P = 0, which contributes 0 only if those rows are finite,
// and the QKV GEMM computes the rows [T, T256) from the A rows there; the
// buffers can hold any bits past T (another model's or a larger batch's
// leftovers).  Nothing else in a pass writes A past T and the GEMM writes
// finite rows from zero ones, so one clear per pass keeps them finite.
constexpr int kAttnTailBlocks = 16;

__global__ void __launch_bounds__(1024)
    attn_work_kernel(const int *__restrict__ seq_len, int B, int *__restrict__ items,
                     int *__restrict__ count, const int *__restrict__ T_dev, int64_t rows,
                     __nv_bfloat16 *__restrict__ qkv, int qkv_cols, __nv_bfloat16 *__restrict__ a,
                     int a_cols) {
  if (blockIdx.x > 0) {
    if (!T_dev) return;
    const int64_t T = __ldg(T_dev);
    const int64_t end = min(rows, ((T + 255) & ~int64_t{255}) + kAttnTcKeys);
    if (T >= end) return;
    const int64_t q8 = qkv_cols / 8, a8 = a_cols / 8, per_row = q8 + a8;
    const int64_t n = (end - T) * per_row;
    const uint4 z = make_uint4(0u, 0u, 0u, 0u);
    for (int64_t i = static_cast<int64_t>(blockIdx.x - 1) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x - 1) * blockDim.x) {
      const int64_t r = T + i / per_row, c = i % per_row;
      if (c < q8)
        reinterpret_cast<uint4 *>(qkv + r * qkv_cols)[c] = z;
      else
        reinterpret_cast<uint4 *>(a + r * a_cols)[c - q8] = z;
    }
    return;
  }
  __shared__ int cnt[3], start[3];
  if (threadIdx.x < 3) cnt[threadIdx.x] = 0;
  __syncthreads();
  for (int b = threadIdx.x; b < B; b += blockDim.x) {
    const int L = seq_len[b];
    atomicAdd(&cnt[L > 256 ? 0 : (L > 128 ? 1 : 2)], (L + 127) >> 7);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    start[0] = 0;
    start[1] = cnt[0];
    start[2] = cnt[0] + cnt[1];
    count[0] = cnt[0] + cnt[1] + cnt[2];
  }
  __syncthreads();
  for (int b = threadIdx.x; b < B; b += blockDim.x) {
    const int L = seq_len[b];
    const int k = L > 256 ? 0 : (L > 128 ? 1 : 2);
    const int nq = (L + 127) >> 7;
    const int at = atomicAdd(&start[k], nq);
    for (int q = 0; q < nq; ++q) items[at + q] = (b << 8) | q;
  }
}

}  // namespace nebw
