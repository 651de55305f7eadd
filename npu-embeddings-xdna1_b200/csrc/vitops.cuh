// Memory-bound kernels of the ViT encoder pass (arch vit_patch16_prenorm_gelu):
// the image -> patch-row step, the CLS/position assembly, the residual add
// fused with the pre-LN LayerNorm that follows it, and the uniform sequence
// table the attention kernels read.
#pragma once

#include <cuda_bf16.h>
#include <cstdint>

#include "rowops.cuh"

namespace nebw {

// im2col_patches (runtime/src/vit/image.cpp:732-755), narrowed to bf16 RNE
// for the patch-embedding GEMM: patch row (img, p, q) -> img * np + p * n + q,
// column (c * P + i) * P + j <- image[img][c][p * P + i][q * P + j].
// One thread per 8 consecutive pixels of one patch row (two float4 loads,
// one 16-byte store); P % 8 == 0, S % P == 0.
__global__ void __launch_bounds__(256)
    vit_im2col_kernel(const float *__restrict__ img, int64_t units, int C, int S, int P,
                      __nv_bfloat16 *__restrict__ patches) {
  const int64_t u = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (u >= units) return;
  const int n = S / P, p8 = P / 8;
  int64_t t = u;
  const int j8 = static_cast<int>(t % p8);
  t /= p8;
  const int i = static_cast<int>(t % P);
  t /= P;
  const int c = static_cast<int>(t % C);
  t /= C;
  const int q = static_cast<int>(t % n);
  t /= n;
  const int p = static_cast<int>(t % n);
  const int64_t im = t / n;
  const float *src = img + ((im * C + c) * S + p * P + i) * static_cast<int64_t>(S) + q * P + j8 * 8;
  const float4 a = *reinterpret_cast<const float4 *>(src);
  const float4 b = *reinterpret_cast<const float4 *>(src + 4);
  const int64_t row = (im * n + p) * n + q;
  __nv_bfloat16 *dst = patches + row * (static_cast<int64_t>(C) * P * P) + (c * P + i) * P + j8 * 8;
  *reinterpret_cast<uint4 *>(dst) = make_uint4(pack_bf16x2(a.x, a.y), pack_bf16x2(a.z, a.w),
                                               pack_bf16x2(b.x, b.y), pack_bf16x2(b.z, b.w));
}

// The encoder's input rows (runtime/src/vit/encoder.cpp:267-281):
//   x[img * n_pos]         = cls + pos[0]
//   x[img * n_pos + 1 + p] = pe[img * np + p] + pos[1 + p]
// pe is the patch GEMM's fp32 output (bias included).  One thread per float4.
__global__ void __launch_bounds__(256)
    vit_assemble_kernel(const float *__restrict__ pe, const float *__restrict__ cls,
                        const float *__restrict__ pos, int64_t n_images, int n_pos, int H,
                        float *__restrict__ x) {
  const int64_t v = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int h4 = H / 4;
  if (v >= n_images * n_pos * h4) return;
  const int col = static_cast<int>(v % h4) * 4;
  const int64_t r = v / h4;
  const int t = static_cast<int>(r % n_pos);
  const int64_t im = r / n_pos;
  const float *src = t == 0 ? cls : pe + (im * (n_pos - 1) + t - 1) * H;
  const float4 a = *reinterpret_cast<const float4 *>(src + col);
  const float4 b = *reinterpret_cast<const float4 *>(pos + static_cast<int64_t>(t) * H + col);
  *reinterpret_cast<float4 *>(x + r * H + col) = make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
}

// LayerNorm of rows r = 0..rows-1 of the residual stream, read at
// x + r * stride_rows * H, with the sublayer output y (bf16, same row layout;
// may be null) added first:
//   v = x[r] (+ y[r]);  if write_x: x[r] = v
//   out_f32[r] = LN(v) (may be null);  out_a[r] = bf16(LN(v)) (may be null)
// This is the pre-LN schedule's residual add (x += sublayer, encoder.cpp:
// 395-399, :408-411) fused with the next LayerNorm site, which reads the
// updated stream; the final LayerNorm reads only the CLS rows (stride n_pos)
// and writes nothing back.  Warp per row, two-pass fp32 as layernorm_kernel.
template <int NV>
__global__ void __launch_bounds__(kRowWarps * 32)
    ln_rows_kernel(float *__restrict__ x, const __nv_bfloat16 *__restrict__ y,
                   int64_t stride_rows, int rows, const float *__restrict__ g,
                   const float *__restrict__ bta, float eps, int write_x,
                   float *__restrict__ out_f32, __nv_bfloat16 *__restrict__ out_a) {
  const int H = NV * 128;
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * kRowWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int64_t at = static_cast<int64_t>(row) * stride_rows * H;
  float *xr = x + at;
  float4 v[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = (i * 32 + lane) * 4;
    v[i] = *reinterpret_cast<const float4 *>(xr + c);
    if (y) {
      const float4 w = load4(y + at + c);
      v[i].x = v[i].x + w.x;
      v[i].y = v[i].y + w.y;
      v[i].z = v[i].z + w.z;
      v[i].w = v[i].w + w.w;
      if (write_x) *reinterpret_cast<float4 *>(xr + c) = v[i];
    }
  }
  ln_row_regs<NV>(v, g, bta, eps, H, lane,
                  out_f32 ? out_f32 + static_cast<int64_t>(row) * H : nullptr,
                  out_a ? out_a + static_cast<int64_t>(row) * H : nullptr);
}

// Every image is one sequence of n_pos rows: len[b] = n_pos, off[b] = b * n_pos.
__global__ void uniform_seqs_kernel(int B, int L, int *__restrict__ len, int *__restrict__ off) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < B) len[b] = L;
  if (b <= B) off[b] = b * L;
}

}  // namespace nebw
