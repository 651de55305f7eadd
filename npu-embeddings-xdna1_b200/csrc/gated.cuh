// The two steps the gated / rotary encoder families (arch
// nomic_bert_rope_swiglu and gte_new_rope_geglu) add to the BERT schedule:
//
//   rope_qk_kernel  rotary positions on the Q and K blocks of the packed
//                   Q|K|V rows, in place (apply_rope_qkv, runtime/src/
//                   encoders/bert_encoder.cpp:926-993): per head, pairs
//                   (d, d + head_dim/2) rotate by the angle of the token's
//                   position in its sequence; V is not touched
//   glu_kernel      h[:, j] = up[:, j] * act(gate[:, j]) over the 2F-wide
//                   FFN-up output [up | gate], written in place over the up
//                   half so that the FFN-down GEMM reads the first F columns
//                   of each 2F row (swiglu_cpu, bert_encoder.cpp:582-627)
//
// Both are HBM-bound elementwise passes over bf16 rows; the arithmetic is
// fp32 with one RNE narrow at the end.
#pragma once

#include <cuda_bf16.h>
#include <cstdint>

#include "gemm_tc.cuh"  // gelu_erf
#include "ptx.cuh"
#include "rowops.cuh"

namespace nebw {

// One warp per token, grid (ceil(S / kRowWarps), B) as embed_ln_kernel: the
// token (b, s) is packed row seq_off[b] + s.  cos / sin: [S, HD] fp32 with
// cos[s, j] == cos[s, j + HD/2] (the reference's duplicated halves).  Lane
// work items are two adjacent d of one head of Q or K, so that a half-warp
// reads 64 contiguous bytes of each half.  The rotation is
//   o1 = fma(-x2, s, x1 c),  o2 = fma(x1, s, x2 c)
// the order in which the reference's own build (g++ -O2 -march=x86-64-v3)
// evaluates its AVX2 form: the second product of each line fused.
template <int HD>
__global__ void __launch_bounds__(kRowWarps * 32)
    rope_qk_kernel(__nv_bfloat16 *__restrict__ qkv, const int *__restrict__ seq_off,
                   const int *__restrict__ seq_len, int H, const float *__restrict__ cos_t,
                   const float *__restrict__ sin_t) {
  constexpr int kHalf = HD / 2, kPairs = kHalf / 2;  // bf16x2 items per head half
  const int lane = threadIdx.x & 31;
  const int b = blockIdx.y;
  const int s = blockIdx.x * kRowWarps + (threadIdx.x >> 5);
  if (s >= __ldg(seq_len + b)) return;
  __nv_bfloat16 *row = qkv + (static_cast<int64_t>(__ldg(seq_off + b)) + s) * (3 * H);
  const float *cs = cos_t + static_cast<int64_t>(s) * HD;
  const float *sn = sin_t + static_cast<int64_t>(s) * HD;
  const int per_block = (H / HD) * kPairs;  // items in Q (or K)
  for (int i = lane; i < 2 * per_block; i += 32) {
    const int qk = i / per_block, rem = i - qk * per_block;
    const int h = rem / kPairs, d = (rem - h * kPairs) * 2;
    __nv_bfloat16 *v = row + qk * H + h * HD;
    const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162 *>(v + d);
    const __nv_bfloat162 z = *reinterpret_cast<const __nv_bfloat162 *>(v + d + kHalf);
    const float2 x1 = __bfloat1622float2(a), x2 = __bfloat1622float2(z);
    const float c0 = __ldg(cs + d), c1 = __ldg(cs + d + 1);
    const float s0 = __ldg(sn + d), s1 = __ldg(sn + d + 1);
    const float o1a = __fmaf_rn(-x2.x, s0, __fmul_rn(x1.x, c0));
    const float o1b = __fmaf_rn(-x2.y, s1, __fmul_rn(x1.y, c1));
    const float o2a = __fmaf_rn(x1.x, s0, __fmul_rn(x2.x, c0));
    const float o2b = __fmaf_rn(x1.y, s1, __fmul_rn(x2.y, c1));
    *reinterpret_cast<__nv_bfloat162 *>(v + d) = __floats2bfloat162_rn(o1a, o1b);
    *reinterpret_cast<__nv_bfloat162 *>(v + d + kHalf) = __floats2bfloat162_rn(o2a, o2b);
  }
}

// Position of every packed row in its sequence (pos[seq_off[b] + s] = s),
// grid (ceil(S / 256), B): the rotary QKV epilogue's per-row input.
__global__ void __launch_bounds__(256)
    row_pos_kernel(const int *__restrict__ seq_off, const int *__restrict__ seq_len,
                   int *__restrict__ pos) {
  const int b = blockIdx.y;
  const int s = blockIdx.x * blockDim.x + threadIdx.x;
  if (s < __ldg(seq_len + b)) pos[__ldg(seq_off + b) + s] = s;
}

// SiLU as swiglu_cpu computes it: x / (1 + 2^max(-x log2 e, -120)).
__device__ __forceinline__ float silu_ref(float x) {
  const float a = fmaxf(__fmul_rn(-x, 1.4426950408889634f), -120.0f);
  return __fdiv_rn(x, __fadd_rn(1.0f, exp2f(a)));
}

// One thread per 8 columns of a row: h[r, j] = up[r, j] * act(gate[r, j])
// for j in [c, c + 8), where the row is 2F bf16 [up | gate].  Rows past the
// device-resident row count exit at once.
template <int GATE>  // 0 SiLU, 1 erf GELU
__global__ void __launch_bounds__(256)
    glu_kernel(__nv_bfloat16 *__restrict__ h, int rows, const int *__restrict__ rows_dev,
               int F) {
  const int per_row = F / 8;
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  int T = rows;
  if (rows_dev) T = min(T, __ldg(rows_dev));
  const int64_t r = i / per_row;
  if (r >= T) return;
  const int c = static_cast<int>(i - r * per_row) * 8;
  __nv_bfloat16 *up = h + r * 2 * F + c;
  const uint4 u = *reinterpret_cast<const uint4 *>(up);
  const uint4 g = *reinterpret_cast<const uint4 *>(up + F);
  const __nv_bfloat162 *u2 = reinterpret_cast<const __nv_bfloat162 *>(&u);
  const __nv_bfloat162 *g2 = reinterpret_cast<const __nv_bfloat162 *>(&g);
  uint4 o;
  __nv_bfloat162 *o2 = reinterpret_cast<__nv_bfloat162 *>(&o);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float2 uf = __bfloat1622float2(u2[k]), gf = __bfloat1622float2(g2[k]);
    float a0, a1;
    if constexpr (GATE == 0) {
      a0 = silu_ref(gf.x);
      a1 = silu_ref(gf.y);
    } else {
      a0 = gelu_erf(gf.x);
      a1 = gelu_erf(gf.y);
    }
    o2[k] = __floats2bfloat162_rn(__fmul_rn(uf.x, a0), __fmul_rn(uf.y, a1));
  }
  *reinterpret_cast<uint4 *>(up) = o;
}

}  // namespace nebw
