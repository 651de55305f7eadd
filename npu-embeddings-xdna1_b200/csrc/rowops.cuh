// Memory-bound row kernels of the encoder pass: the varlen packing scan,
// embedding gather + LayerNorm, LayerNorm, and pooling + L2 normalisation.
//
// Each LayerNorm row is owned by one warp: 128-bit loads, the row held in
// registers, two passes (mean, then biased variance about the mean) reduced
// with warp shuffles -- the reference's two-pass form (layer_norm_cpu,
// runtime/src/encoders/bert_encoder.cpp:416-463; kernels/layernorm.cc:65-142)
// -- and two stores: the fp32 residual stream and the bf16 RNE operand of the
// next GEMM (add_norm_bf16's twin output, bert_encoder.cpp:1304-1361).
#pragma once

#include <cuda_bf16.h>
#include <cstdint>

#include "ptx.cuh"

namespace nebw {

constexpr int kRowWarps = 8;  // rows (warps) per CTA for the LayerNorm kernels

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// seq_off[0..B] = exclusive prefix sum of seq_len; seq_off[B] = T (the
// packed token count).  Lengths outside [1, S] are reported (kDevBadLength)
// and clamped so that nothing downstream indexes out of bounds.
__global__ void __launch_bounds__(1024)
    pack_offsets_kernel(const int *__restrict__ seq_len_in, int B, int S, int *__restrict__ seq_len,
                        int *__restrict__ seq_off, int *err) {
  __shared__ int part[1024];
  const int tid = threadIdx.x;
  const int per = (B + blockDim.x - 1) / blockDim.x;
  const int lo = min(B, tid * per), hi = min(B, lo + per);
  int sum = 0;
  for (int i = lo; i < hi; ++i) {
    int l = seq_len_in[i];
    if (l < 1 || l > S) {
      record_err(err, kDevBadLength);
      l = l < 1 ? 1 : S;
    }
    seq_len[i] = l;
    sum += l;
  }
  part[tid] = sum;
  __syncthreads();
  for (int o = 1; o < blockDim.x; o <<= 1) {  // Hillis-Steele inclusive scan
    const int v = tid >= o ? part[tid - o] : 0;
    __syncthreads();
    part[tid] += v;
    __syncthreads();
  }
  int run = part[tid] - sum;  // exclusive prefix of this thread's chunk
  for (int i = lo; i < hi; ++i) {
    seq_off[i] = run;
    run += seq_len[i];
  }
  if (tid == blockDim.x - 1) seq_off[B] = part[tid];
}

// LayerNorm of one warp-owned row held as NV float4 per lane (H = 128*NV),
// in place.
template <int NV>
__device__ __forceinline__ void ln_normalise(float4 (&v)[NV], const float *__restrict__ g,
                                             const float *__restrict__ bta, float eps, int H,
                                             int lane) {
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
  const float mean = warp_sum(s) / static_cast<float>(H);
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const float a = v[i].x - mean, b = v[i].y - mean, c = v[i].z - mean, d = v[i].w - mean;
    q = fmaf(a, a, q);
    q = fmaf(b, b, q);
    q = fmaf(c, c, q);
    q = fmaf(d, d, q);
  }
  const float var = warp_sum(q) / static_cast<float>(H);
  const float is = 1.0f / sqrtf(var + eps);
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = (i * 32 + lane) * 4;
    const float4 gg = __ldg(reinterpret_cast<const float4 *>(g + c));
    const float4 bb = __ldg(reinterpret_cast<const float4 *>(bta + c));
    v[i].x = fmaf((v[i].x - mean) * is, gg.x, bb.x);
    v[i].y = fmaf((v[i].y - mean) * is, gg.y, bb.y);
    v[i].z = fmaf((v[i].z - mean) * is, gg.z, bb.z);
    v[i].w = fmaf((v[i].w - mean) * is, gg.w, bb.w);
  }
}

// LayerNorm of one warp-owned row, stored as fp32 (xo) and as the bf16 RNE
// operand of the next GEMM (ao), either may be null.
template <int NV>
__device__ __forceinline__ void ln_row_regs(float4 (&v)[NV], const float *__restrict__ g,
                                            const float *__restrict__ bta, float eps, int H,
                                            int lane, float *__restrict__ xo,
                                            __nv_bfloat16 *__restrict__ ao) {
  ln_normalise<NV>(v, g, bta, eps, H, lane);
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = (i * 32 + lane) * 4;
    if (xo) *reinterpret_cast<float4 *>(xo + c) = v[i];
    if (ao) {
      uint2 pk;
      pk.x = pack_bf16x2(v[i].x, v[i].y);
      pk.y = pack_bf16x2(v[i].z, v[i].w);
      *reinterpret_cast<uint2 *>(ao + c) = pk;
    }
  }
}

// Four consecutive elements of a GEMM output row, widened to fp32.
__device__ __forceinline__ float4 load4(const float *p) {
  return *reinterpret_cast<const float4 *>(p);
}
__device__ __forceinline__ float4 load4(const __nv_bfloat16 *p) {
  const uint2 u = *reinterpret_cast<const uint2 *>(p);
  return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u),
                     __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xffff0000u));
}

// x[r] = LN(x[r] (+ y[r])) for r < T; also a[r] = bf16(x[r]) when a != null.
// y is the GEMM output (fp32, or bf16 after the RNE narrow); x stays fp32.
template <int NV, typename YT>
__global__ void __launch_bounds__(kRowWarps * 32)
    layernorm_kernel(float *__restrict__ x, const YT *__restrict__ y,
                     const float *__restrict__ g, const float *__restrict__ bta, float eps,
                     int rows, const int *__restrict__ rows_dev, __nv_bfloat16 *__restrict__ a) {
  const int H = NV * 128;
  const int lane = threadIdx.x & 31;
  const int idx = blockIdx.x * kRowWarps + (threadIdx.x >> 5);
  int T = rows;
  if (rows_dev) T = min(T, __ldg(rows_dev));
  if (idx >= T) return;
  // Rows from the last one down: the GEMM that wrote y ended on its last
  // rows, which are still in L2, and the next GEMM starts on the first rows,
  // which this kernel writes last.  Each row's arithmetic is the same.
  const int row = T - 1 - idx;
  float *xr = x + static_cast<int64_t>(row) * H;
  float4 v[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = (i * 32 + lane) * 4;
    v[i] = *reinterpret_cast<const float4 *>(xr + c);
    if (y) {
      const float4 w = load4(y + static_cast<int64_t>(row) * H + c);
      v[i].x = w.x + v[i].x;
      v[i].y = w.y + v[i].y;
      v[i].z = w.z + v[i].z;
      v[i].w = w.w + v[i].w;
    }
  }
  ln_row_regs<NV>(v, g, bta, eps, H, lane, xr,
                  a ? a + static_cast<int64_t>(row) * H : nullptr);
}

// The int8 pass's add + LayerNorm: x[r] = LN(x[r] + y[r]) for r < T (y the
// dequantised fp32 output of an int8 GEMM, or null), and, when q is set, the
// normalised row quantised for the next int8 GEMM as add_norm_quant does
// (runtime/src/encoders/bert_encoder.cpp:1196-1302) -- quantise_a_int8's
// steps on the row held in registers: sc = max|x * ias| / 127 (1 for a zero
// row), q = rne(clamp((x * ias) * (1 / sc), +-127)).
template <int NV>
__global__ void __launch_bounds__(kRowWarps * 32)
    layernorm_quant_kernel(float *__restrict__ x, const float *__restrict__ y,
                           const float *__restrict__ g, const float *__restrict__ bta, float eps,
                           int rows, const int *__restrict__ rows_dev,
                           const float *__restrict__ ias, int8_t *__restrict__ q,
                           float *__restrict__ scale) {
  const int H = NV * 128;
  const int lane = threadIdx.x & 31;
  const int idx = blockIdx.x * kRowWarps + (threadIdx.x >> 5);
  int T = rows;
  if (rows_dev) T = min(T, __ldg(rows_dev));
  if (idx >= T) return;
  // Rows from the last one down: the GEMM that wrote y ended on its last
  // rows, which are still in L2, and the next GEMM starts on the first rows,
  // which this kernel writes last.  Each row's arithmetic is the same.
  const int row = T - 1 - idx;
  float *xr = x + static_cast<int64_t>(row) * H;
  float4 v[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = (i * 32 + lane) * 4;
    v[i] = *reinterpret_cast<const float4 *>(xr + c);
    if (y) {
      const float4 w = *reinterpret_cast<const float4 *>(y + static_cast<int64_t>(row) * H + c);
      v[i].x = w.x + v[i].x;
      v[i].y = w.y + v[i].y;
      v[i].z = w.z + v[i].z;
      v[i].w = w.w + v[i].w;
    }
  }
  ln_normalise<NV>(v, g, bta, eps, H, lane);
#pragma unroll
  for (int i = 0; i < NV; ++i)
    *reinterpret_cast<float4 *>(xr + (i * 32 + lane) * 4) = v[i];
  if (!q) return;
  float mx = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const float4 s = __ldg(reinterpret_cast<const float4 *>(ias + (i * 32 + lane) * 4));
    mx = fmaxf(fmaxf(mx, fabsf(v[i].x * s.x)), fabsf(v[i].y * s.y));
    mx = fmaxf(fmaxf(mx, fabsf(v[i].z * s.z)), fabsf(v[i].w * s.w));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  const float sc = mx > 0.0f ? mx / 127.0f : 1.0f;
  const float inv = 1.0f / sc;
  if (lane == 0) scale[row] = sc;
  int8_t *qr = q + static_cast<int64_t>(row) * H;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = (i * 32 + lane) * 4;
    const float4 s = __ldg(reinterpret_cast<const float4 *>(ias + c));
    const float e[4] = {v[i].x * s.x, v[i].y * s.y, v[i].z * s.z, v[i].w * s.w};
    uint32_t pk = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float t = fminf(fmaxf(e[k] * inv, -127.0f), 127.0f);
      pk |= (static_cast<uint32_t>(__float2int_rn(t)) & 0xffu) << (8 * k);
    }
    *reinterpret_cast<uint32_t *>(qr + c) = pk;
  }
}

// Embedding gather + LayerNorm for the packed rows of a padded id batch.
// Row off[b] + s (s < len[b]) gets LN((word[id] + pos[s]) + type[0]) --
// the reference's gather order (embed_service.cpp:51-57).
template <int NV>
__global__ void __launch_bounds__(kRowWarps * 32)
    embed_ln_kernel(const int *__restrict__ ids, int S, const int *__restrict__ seq_off,
                    const int *__restrict__ seq_len, const float *__restrict__ word, int vocab,
                    const float *__restrict__ pos, const float *__restrict__ typ,
                    const float *__restrict__ g, const float *__restrict__ bta, float eps,
                    float *__restrict__ x, __nv_bfloat16 *__restrict__ a, int *err) {
  const int H = NV * 128;
  const int lane = threadIdx.x & 31;
  const int b = blockIdx.y;
  const int s = blockIdx.x * kRowWarps + (threadIdx.x >> 5);
  if (s >= seq_len[b]) return;
  int id = ids[static_cast<int64_t>(b) * S + s];
  if (id < 0 || id >= vocab) {
    record_err(err, kDevBadTokenId);
    id = 0;
  }
  const int64_t row = seq_off[b] + s;
  const float *wr = word + static_cast<int64_t>(id) * H;
  const float *pr = pos + static_cast<int64_t>(s) * H;
  float4 v[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = (i * 32 + lane) * 4;
    const float4 w = __ldg(reinterpret_cast<const float4 *>(wr + c));
    const float4 p = __ldg(reinterpret_cast<const float4 *>(pr + c));
    const float4 t = __ldg(reinterpret_cast<const float4 *>(typ + c));
    v[i].x = (w.x + p.x) + t.x;
    v[i].y = (w.y + p.y) + t.y;
    v[i].z = (w.z + p.z) + t.z;
    v[i].w = (w.w + p.w) + t.w;
  }
  ln_row_regs<NV>(v, g, bta, eps, H, lane, x + row * H, a ? a + row * H : nullptr);
}

// Pooling + L2 normalisation, one CTA per sequence (app::pool_rows,
// runtime/include/common/app_state.hpp:335-374): CLS takes the sequence's
// first row; mean sums its rows in double in row order and divides by
// max(len, 1e-9); the L2 norm is accumulated in double and floored at 1e-24
// before the square root; the result is rounded to fp32 once.
constexpr int kPoolThreads = 256;

__global__ void __launch_bounds__(kPoolThreads)
    pool_l2_kernel(const float *__restrict__ h, const int *__restrict__ seq_off,
                   const int *__restrict__ seq_len, int H, int cls, int l2,
                   float *__restrict__ out) {
  __shared__ double red[kPoolThreads / 32];
  __shared__ double total;
  const int b = blockIdx.x;
  const int64_t r0 = seq_off[b];
  const int L = seq_len[b];
  constexpr int kMaxPer = 16;  // H <= 16 * kPoolThreads
  double acc[kMaxPer];
  double sq = 0.0;
  const float denom = fmaxf(static_cast<float>(L), 1e-9f);
#pragma unroll
  for (int k = 0; k < kMaxPer; ++k) {
    const int c = threadIdx.x + k * kPoolThreads;
    acc[k] = 0.0;
    if (c < H) {
      if (cls) {
        acc[k] = static_cast<double>(h[r0 * H + c]);
      } else {
        double a = 0.0;
        for (int s = 0; s < L; ++s) a += static_cast<double>(h[(r0 + s) * H + c]);
        acc[k] = a / static_cast<double>(denom);
      }
      sq += acc[k] * acc[k];
    }
  }
  double nrm = 1.0;
  if (l2) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sq;
    __syncthreads();
    if (threadIdx.x == 0) {
      double t = 0.0;
      for (int w = 0; w < kPoolThreads / 32; ++w) t += red[w];
      total = t;
    }
    __syncthreads();
    nrm = sqrt(fmax(total, 1e-24));
  }
#pragma unroll
  for (int k = 0; k < kMaxPer; ++k) {
    const int c = threadIdx.x + k * kPoolThreads;
    if (c < H) out[static_cast<int64_t>(b) * H + c] = static_cast<float>(acc[k] / nrm);
  }
}

// Weight staging: fp32 or bf16 [K, N] (the container's layout) to bf16
// [N, K] (K-major, the UMMA B-operand layout the GEMM's tensor map tiles),
// with round-to-nearest-even (to_bf16, host_kernels.hpp:157-161).
__global__ void stage_weight_kernel(const void *__restrict__ src, int src_bf16, int K, int N,
                                    __nv_bfloat16 *__restrict__ dst) {
  __shared__ float tile[32][33];
  const int k0 = blockIdx.y * 32, n0 = blockIdx.x * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int k = k0 + i, n = n0 + threadIdx.x;
    float v = 0.f;
    if (k < K && n < N) {
      const int64_t idx = static_cast<int64_t>(k) * N + n;
      v = src_bf16 ? __bfloat162float(static_cast<const __nv_bfloat16 *>(src)[idx])
                   : static_cast<const float *>(src)[idx];
    }
    tile[i][threadIdx.x] = v;
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int n = n0 + i, k = k0 + threadIdx.x;
    if (n < N && k < K) dst[static_cast<int64_t>(n) * K + k] = __float2bfloat16_rn(tile[threadIdx.x][i]);
  }
}

// fp32 -> bf16 RNE, elementwise (the standalone narrow, for op-level use).
__global__ void narrow_bf16_kernel(const float *__restrict__ x, int64_t n,
                                   __nv_bfloat16 *__restrict__ y) {
  const int64_t i = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 4;
  if (i + 3 < n) {
    const float4 v = *reinterpret_cast<const float4 *>(x + i);
    uint2 pk;
    pk.x = pack_bf16x2(v.x, v.y);
    pk.y = pack_bf16x2(v.z, v.w);
    *reinterpret_cast<uint2 *>(y + i) = pk;
  } else {
    for (int64_t j = i; j < n; ++j) y[j] = __float2bfloat16_rn(x[j]);
  }
}

}  // namespace nebw
