// The C ABI of include/nebw.h: device handles, weight staging, the op entry
// points, and the whole-encoder pass for one GPU.
//
// The encoder pass mirrors BertEncoder::run (runtime/src/encoders/
// bert_encoder.cpp:1419-1598) on packed variable-length rows:
//
//   pack_offsets   lens -> seq_off (T = seq_off[B] stays on the device)
//   embed_ln       x = LN_emb((word[id] + pos[s]) + type[0]);  a = bf16(x)
//   per layer L:
//     gemm QKV     qkv = bf16(a . Wqkv + b)
//     attention    ctx = softmax(Q K^T) V           (per sequence, per head)
//     gemm AO      y   = bf16(ctx . Wao + b)
//     layernorm    x   = LN1(y + x);  a = bf16(x)   (add_into + layer_norm)
//     gemm UP      h   = bf16(gelu(a . Wup + b))
//     gemm DOWN    y   = bf16(h . Wdn + b)
//     layernorm    x   = LN2(y + x);  a = bf16(x)
//
// Every GEMM output is narrowed to bf16 RNE as the reference's array path
// does (kernels/narrow_f32_bf16.cc:50-90, run on each GEMM C tile); the
// residual stream x and the LayerNorm arithmetic stay fp32.
//   pool_l2        out = normalise(pool(x))
//
// Nothing in a pass needs the host to know T: every kernel bounds itself by
// the device-resident count, so the pass is one asynchronous launch
// sequence.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cctype>
#include <cmath>
#include <cstdarg>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/nebw.h"
#include "attention.cuh"
#include "attention_tc.cuh"
#include "gated.cuh"
#include "gemm_i8.cuh"
#include "gemm_tc.cuh"
#include "npue_file.h"
#include "npue_pack.h"
#include "ptx.cuh"
#include "rowops.cuh"

using nebw::GemmArgs;

// ---------------------------------------------------------------------------
// errors
// ---------------------------------------------------------------------------

namespace {

thread_local std::string g_last_error;

int set_error(int code, const char *fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

#define NEBW_CUDA(call)                                                                   \
  do {                                                                                    \
    cudaError_t e_ = (call);                                                              \
    if (e_ != cudaSuccess)                                                                \
      return set_error(NEBW_ECUDA, "%s failed: %s (%s:%d)", #call, cudaGetErrorString(e_), \
                       __FILE__, __LINE__);                                               \
  } while (0)

#define NEBW_REQUIRE(cond, ...)                        \
  do {                                                 \
    if (!(cond)) return set_error(NEBW_EINVAL, __VA_ARGS__); \
  } while (0)

const char *dev_err_name(int code) {
  switch (code) {
    case nebw::kDevWaitTimeout: return "a bounded device wait timed out";
    case nebw::kDevBadTokenId: return "a token id is outside [0, vocab_size)";
    case nebw::kDevBadLength: return "a sequence length is outside [1, seq]";
    case nebw::kDevBadShape: return "a kernel was handed a shape its launch cannot cover";
    default: return "unknown device error";
  }
}

PFN_cuTensorMapEncodeTiled_v12000 g_encode_tiled = nullptr;
std::once_flag g_encode_once;

int load_tensor_map_encoder() {
  std::call_once(g_encode_once, [] {
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode_tiled = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (!g_encode_tiled)
    return set_error(NEBW_ECUDA, "cuTensorMapEncodeTiled is not available from the driver");
  return NEBW_OK;
}

// A 2-D bf16 K-major tensor map [rows, K] with a {64, box_rows} box and
// 128-byte swizzle (the GEMM's A and W operand tiles).
// `stride` is the row pitch in elements (0: K).
int make_tmap_kmajor(CUtensorMap *map, const void *ptr, int64_t rows, int64_t K, int box_rows,
                     int64_t stride = 0) {
  if (int rc = load_tensor_map_encoder()) return rc;
  if (reinterpret_cast<uintptr_t>(ptr) % 16)
    return set_error(NEBW_EINVAL, "GEMM operand address is not 16-byte aligned");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(stride ? stride : K) * 2};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(nebw::kGemmBK), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(ptr),
                              dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(NEBW_ECUDA, "cuTensorMapEncodeTiled failed (%d) for [%lld, %lld] box %d",
                     static_cast<int>(r), static_cast<long long>(rows),
                     static_cast<long long>(K), box_rows);
  return NEBW_OK;
}

// The attention kernel's head tiles: a bf16 [rows, cols] map with a
// {head_dim, box_rows} box over the packed Q|K|V rows, 128-byte swizzle for
// head_dim 64 (128-byte box rows), 64-byte swizzle for head_dim 32.
int make_tmap_head(CUtensorMap *map, const void *ptr, int64_t rows, int64_t cols, int head_dim,
                   int box_rows) {
  if (int rc = load_tensor_map_encoder()) return rc;
  NEBW_REQUIRE(head_dim == 32 || head_dim == 64, "head tile of width %d refused", head_dim);
  if (reinterpret_cast<uintptr_t>(ptr) % 16)
    return set_error(NEBW_EINVAL, "Q|K|V address is not 16-byte aligned");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * 2};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(head_dim), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(ptr),
                              dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                              head_dim == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(NEBW_ECUDA, "cuTensorMapEncodeTiled (head tiles) failed (%d) for [%lld, %lld]",
                     static_cast<int>(r), static_cast<long long>(rows), static_cast<long long>(cols));
  return NEBW_OK;
}

// An int8 K-major map [rows, K] with {128, box_rows} boxes (128-byte rows,
// 128-byte swizzle): the int8 GEMM's A and W tiles.  K % 16 == 0.
int make_tmap_i8(CUtensorMap *map, const void *ptr, int64_t rows, int64_t K, int box_rows) {
  if (int rc = load_tensor_map_encoder()) return rc;
  if (reinterpret_cast<uintptr_t>(ptr) % 16)
    return set_error(NEBW_EINVAL, "int8 GEMM operand address is not 16-byte aligned");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(K)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(nebw::kGemmI8BK), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(ptr), dims,
                              strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(NEBW_ECUDA, "cuTensorMapEncodeTiled (int8) failed (%d) for [%lld, %lld]",
                     static_cast<int>(r), static_cast<long long>(rows), static_cast<long long>(K));
  return NEBW_OK;
}

// A 2-D row-major output tensor map [rows, N] with a 32 x 32 box (the GEMM
// epilogue's TMA store chunk): fp32 rows of the box are 128 bytes (128-byte
// swizzle), bf16 rows 64 bytes (64-byte swizzle).
int make_tmap_out(CUtensorMap *map, const void *ptr, int64_t rows, int64_t N, bool bf16) {
  if (int rc = load_tensor_map_encoder()) return rc;
  if (reinterpret_cast<uintptr_t>(ptr) % 16)
    return set_error(NEBW_EINVAL, "GEMM output address is not 16-byte aligned");
  const int esz = bf16 ? 2 : 4;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(N) * esz};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode_tiled(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                              2, const_cast<void *>(ptr), dims, strides, box, estr,
                              CU_TENSOR_MAP_INTERLEAVE_NONE,
                              bf16 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(NEBW_ECUDA, "cuTensorMapEncodeTiled (output) failed (%d) for [%lld, %lld]",
                     static_cast<int>(r), static_cast<long long>(rows), static_cast<long long>(N));
  return NEBW_OK;
}

}  // namespace

// ---------------------------------------------------------------------------
// device handle
// ---------------------------------------------------------------------------

struct Weight {
  __nv_bfloat16 *ptr = nullptr;  // [N, K] bf16
  int64_t K = 0, N = 0;
  CUtensorMap map64, map128, map256;  // box rows 64 / 128 / 256
};

struct WeightI8 {
  int8_t *ptr = nullptr;  // [N, K] int8
  int64_t K = 0, N = 0;
  CUtensorMap map64, map128, map256;  // box rows 64 / 128 / 256, 128-byte K boxes
};

struct nebw_dev {
  int device = 0;
  int sm_count = 0;
  int cc_major = 0, cc_minor = 0;
  cudaStream_t stream = nullptr;
  // where passes are captured as CUDA graphs (nebw_model_set_graphs); created
  // on first use.  A graph is launched on the caller's stream, which may be
  // one capture is not allowed on (the legacy default stream).
  cudaStream_t cap_stream = nullptr;
  int *d_err = nullptr;
  std::map<uint64_t, Weight> weights;
  std::map<uint64_t, WeightI8> weights_i8;  // int8 GEMM operands (nebw_stage_weight_i8)
  uint64_t next_handle = 1;
  // CTA pairs the GPU can hold at once for the 2-CTA GEMM (0: use the
  // single-CTA kernel); NEBW_GEMM_CTAS=1 in the environment forces 0.
  int gemm_pairs = 0;
  // attention kernel: NEBW_ATTN_MMA (mma.sync flash) or NEBW_ATTN_TCGEN05
  // (UMMA/TMEM); see nebw_set_attention_kernel
  int attn_kind = NEBW_ATTN_TCGEN05;
};

namespace {

int use_dev(nebw_dev *d) {
  NEBW_REQUIRE(d != nullptr, "null device handle");
  NEBW_CUDA(cudaSetDevice(d->device));
  return NEBW_OK;
}

cudaStream_t pick_stream(nebw_dev *d, void *stream) {
  return stream ? static_cast<cudaStream_t>(stream) : d->stream;
}

template <int BN, int EPI>
int set_pair_attr() {
  NEBW_CUDA(cudaFuncSetAttribute(nebw::gemm_tc_pair_kernel<BN, EPI>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 nebw::GemmPairShape<BN>::kSmemBytes));
  return NEBW_OK;
}

template <int BN, int EPI>
int set_gemm_attr() {
  NEBW_CUDA(cudaFuncSetAttribute(nebw::gemm_tc_kernel<BN, EPI>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 nebw::GemmShape<BN>::kSmemBytes));
  return NEBW_OK;
}

int set_all_gemm_attrs() {
  int rc = 0;
  rc |= set_gemm_attr<128, nebw::kEpiBf16>();
  rc |= set_gemm_attr<128, nebw::kEpiBf16Gelu8>();
  rc |= set_gemm_attr<128, nebw::kEpiBf16Erf>();
  rc |= set_gemm_attr<128, nebw::kEpiF32>();
  rc |= set_gemm_attr<128, nebw::kEpiF32Resid>();
  rc |= set_gemm_attr<256, nebw::kEpiBf16>();
  rc |= set_gemm_attr<256, nebw::kEpiBf16Gelu8>();
  rc |= set_gemm_attr<256, nebw::kEpiBf16Erf>();
  rc |= set_gemm_attr<256, nebw::kEpiF32>();
  rc |= set_gemm_attr<256, nebw::kEpiF32Resid>();
  rc |= set_pair_attr<128, nebw::kEpiBf16>();
  rc |= set_pair_attr<128, nebw::kEpiBf16Gelu8>();
  rc |= set_pair_attr<128, nebw::kEpiBf16Erf>();
  rc |= set_pair_attr<128, nebw::kEpiF32>();
  rc |= set_pair_attr<128, nebw::kEpiF32Resid>();
  rc |= set_pair_attr<256, nebw::kEpiBf16>();
  rc |= set_pair_attr<256, nebw::kEpiBf16Gelu8>();
  rc |= set_pair_attr<256, nebw::kEpiBf16Erf>();
  rc |= set_pair_attr<256, nebw::kEpiF32>();
  rc |= set_pair_attr<128, nebw::kEpiBf16SwiGLU>();
  rc |= set_pair_attr<128, nebw::kEpiBf16GeGLU>();
  rc |= set_pair_attr<256, nebw::kEpiBf16SwiGLU>();
  rc |= set_pair_attr<256, nebw::kEpiBf16GeGLU>();
  rc |= set_pair_attr<128, nebw::kEpiBf16Rope>();
  rc |= set_pair_attr<256, nebw::kEpiBf16Rope>();
  rc |= set_pair_attr<256, nebw::kEpiF32Resid>();
  rc |= set_pair_attr<128, nebw::kEpiI8F32>();
  rc |= set_pair_attr<128, nebw::kEpiI8Gelu8>();
  rc |= set_pair_attr<128, nebw::kEpiI8Bf16>();
  rc |= set_pair_attr<256, nebw::kEpiI8F32>();
  rc |= set_pair_attr<256, nebw::kEpiI8Gelu8>();
  rc |= set_pair_attr<256, nebw::kEpiI8Bf16>();
  return rc ? NEBW_ECUDA : NEBW_OK;
}

// How many 2-CTA clusters of the pair GEMM fit on the GPU at once.
int query_gemm_pairs(int *pairs) {
  *pairs = 0;
  const char *force = std::getenv("NEBW_GEMM_CTAS");
  if (force && std::atoi(force) == 1) return NEBW_OK;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * 74);
  cfg.blockDim = dim3(nebw::kGemmThreads);
  cfg.dynamicSmemBytes = nebw::GemmPairShape<256>::kSmemBytes;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = 2;
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  int n = 0;
  NEBW_CUDA(cudaOccupancyMaxActiveClusters(&n, nebw::gemm_tc_pair_kernel<256, nebw::kEpiBf16>, &cfg));
  *pairs = n;
  return NEBW_OK;
}

// ---- launchers shared by the op entry points and the encoder pass ----------

int pick_epi(int act, int c_dtype, bool resid) {
  if (c_dtype == NEBW_F32) return resid ? nebw::kEpiF32Resid : nebw::kEpiF32;
  if (act == NEBW_ACT_GELU8) return nebw::kEpiBf16Gelu8;
  if (act == NEBW_ACT_GELU_ERF) return nebw::kEpiBf16Erf;
  return nebw::kEpiBf16;
}

template <int BN>
int launch_gemm_bn(nebw_dev *d, int epi, const CUtensorMap &mA, const CUtensorMap &mW,
                   const GemmArgs &a, cudaStream_t st) {
  const int64_t tiles = ((static_cast<int64_t>(a.M) + nebw::kGemmBM - 1) / nebw::kGemmBM) *
                        ((a.N + BN - 1) / BN);
  const int grid = static_cast<int>(std::min<int64_t>(tiles, d->sm_count));
  if (grid <= 0) return NEBW_OK;
  const dim3 g(grid), b(nebw::kGemmThreads);
  const size_t smem = nebw::GemmShape<BN>::kSmemBytes;
  switch (epi) {
    case nebw::kEpiBf16: nebw::gemm_tc_kernel<BN, nebw::kEpiBf16><<<g, b, smem, st>>>(mA, mW, a); break;
    case nebw::kEpiBf16Gelu8: nebw::gemm_tc_kernel<BN, nebw::kEpiBf16Gelu8><<<g, b, smem, st>>>(mA, mW, a); break;
    case nebw::kEpiBf16Erf: nebw::gemm_tc_kernel<BN, nebw::kEpiBf16Erf><<<g, b, smem, st>>>(mA, mW, a); break;
    case nebw::kEpiF32: nebw::gemm_tc_kernel<BN, nebw::kEpiF32><<<g, b, smem, st>>>(mA, mW, a); break;
    case nebw::kEpiF32Resid: nebw::gemm_tc_kernel<BN, nebw::kEpiF32Resid><<<g, b, smem, st>>>(mA, mW, a); break;
    default: return set_error(NEBW_EINVAL, "unknown GEMM epilogue %d", epi);
  }
  NEBW_CUDA(cudaGetLastError());
  return NEBW_OK;
}

// Tile width: 256 when N is a multiple of 256, else 128 (N % 128 == 0 keeps
// every tile full; other N % 8 == 0 widths run a masked last tile).
int gemm_bn_for(int64_t N) { return N % 256 == 0 ? 256 : 128; }

template <int BN>
int launch_gemm_pair(nebw_dev *d, int epi, const CUtensorMap &mA, const CUtensorMap &mW,
                     const CUtensorMap &mC,
                     const GemmArgs &a, cudaStream_t st) {
  const int64_t tiles = ((static_cast<int64_t>(a.M) + 2 * nebw::kGemmBM - 1) / (2 * nebw::kGemmBM)) *
                        ((a.N + BN - 1) / BN);
  const int pairs = static_cast<int>(std::min<int64_t>(tiles, d->gemm_pairs));
  if (pairs <= 0) return NEBW_OK;
  const dim3 g(2 * pairs), b(nebw::kGemmThreads);
  const size_t smem = nebw::GemmPairShape<BN>::kSmemBytes;
  switch (epi) {
    case nebw::kEpiBf16: nebw::gemm_tc_pair_kernel<BN, nebw::kEpiBf16><<<g, b, smem, st>>>(mA, mW, mC, a); break;
    case nebw::kEpiBf16Gelu8: nebw::gemm_tc_pair_kernel<BN, nebw::kEpiBf16Gelu8><<<g, b, smem, st>>>(mA, mW, mC, a); break;
    case nebw::kEpiBf16Erf: nebw::gemm_tc_pair_kernel<BN, nebw::kEpiBf16Erf><<<g, b, smem, st>>>(mA, mW, mC, a); break;
    case nebw::kEpiF32: nebw::gemm_tc_pair_kernel<BN, nebw::kEpiF32><<<g, b, smem, st>>>(mA, mW, mC, a); break;
    case nebw::kEpiF32Resid: nebw::gemm_tc_pair_kernel<BN, nebw::kEpiF32Resid><<<g, b, smem, st>>>(mA, mW, mC, a); break;
    case nebw::kEpiBf16SwiGLU: nebw::gemm_tc_pair_kernel<BN, nebw::kEpiBf16SwiGLU><<<g, b, smem, st>>>(mA, mW, mC, a); break;
    case nebw::kEpiBf16GeGLU: nebw::gemm_tc_pair_kernel<BN, nebw::kEpiBf16GeGLU><<<g, b, smem, st>>>(mA, mW, mC, a); break;
    case nebw::kEpiBf16Rope: nebw::gemm_tc_pair_kernel<BN, nebw::kEpiBf16Rope><<<g, b, smem, st>>>(mA, mW, mC, a); break;
    case nebw::kEpiI8F32: nebw::gemm_tc_pair_kernel<BN, nebw::kEpiI8F32><<<g, b, smem, st>>>(mA, mW, mC, a); break;
    case nebw::kEpiI8Gelu8: nebw::gemm_tc_pair_kernel<BN, nebw::kEpiI8Gelu8><<<g, b, smem, st>>>(mA, mW, mC, a); break;
    case nebw::kEpiI8Bf16: nebw::gemm_tc_pair_kernel<BN, nebw::kEpiI8Bf16><<<g, b, smem, st>>>(mA, mW, mC, a); break;
    default: return set_error(NEBW_EINVAL, "unknown GEMM epilogue %d", epi);
  }
  NEBW_CUDA(cudaGetLastError());
  return NEBW_OK;
}

// 2-CTA tiles (256 x BN per pair) when the GPU can place CTA pairs, else the
// single-CTA kernel (128 x BN).  The A tensor map's box is 128 rows either
// way; W's box is BN/2 rows for pairs and BN rows for single CTAs.
int launch_gemm(nebw_dev *d, const Weight &w, const CUtensorMap &mA128, const CUtensorMap &mC,
                int epi, const GemmArgs &a, cudaStream_t st) {
  const bool wide = gemm_bn_for(a.N) == 256;
  if (d->gemm_pairs > 0) {
    if (wide) return launch_gemm_pair<256>(d, epi, mA128, w.map128, mC, a, st);
    return launch_gemm_pair<128>(d, epi, mA128, w.map64, mC, a, st);
  }
  if (wide) return launch_gemm_bn<256>(d, epi, mA128, w.map256, a, st);
  return launch_gemm_bn<128>(d, epi, mA128, w.map128, a, st);
}

template <int NV>
void launch_ln_nv(float *x, const void *y, bool y_bf16, const float *g, const float *b, float eps,
                  int rows, const int *rows_dev, __nv_bfloat16 *a, cudaStream_t st) {
  const int grid = (rows + nebw::kRowWarps - 1) / nebw::kRowWarps;
  if (y_bf16)
    nebw::layernorm_kernel<NV, __nv_bfloat16><<<grid, nebw::kRowWarps * 32, 0, st>>>(
        x, static_cast<const __nv_bfloat16 *>(y), g, b, eps, rows, rows_dev, a);
  else
    nebw::layernorm_kernel<NV, float><<<grid, nebw::kRowWarps * 32, 0, st>>>(
        x, static_cast<const float *>(y), g, b, eps, rows, rows_dev, a);
}

int launch_layernorm(float *x, const void *y, bool y_bf16, const float *g, const float *b,
                     float eps, int64_t rows, int64_t H, const int *rows_dev, __nv_bfloat16 *a,
                     cudaStream_t st) {
  NEBW_REQUIRE(H % 128 == 0 && H >= 128 && H <= 2048,
               "LayerNorm width %lld refused: a multiple of 128 up to 2048 is required",
               static_cast<long long>(H));
  if (rows <= 0) return NEBW_OK;
  const int r = static_cast<int>(rows);
  switch (H / 128) {
#define NEBW_LN_CASE(n) \
  case n: launch_ln_nv<n>(x, y, y_bf16, g, b, eps, r, rows_dev, a, st); break;
    NEBW_LN_CASE(1) NEBW_LN_CASE(2) NEBW_LN_CASE(3) NEBW_LN_CASE(4) NEBW_LN_CASE(5)
    NEBW_LN_CASE(6) NEBW_LN_CASE(7) NEBW_LN_CASE(8) NEBW_LN_CASE(9) NEBW_LN_CASE(10)
    NEBW_LN_CASE(11) NEBW_LN_CASE(12) NEBW_LN_CASE(13) NEBW_LN_CASE(14) NEBW_LN_CASE(15)
    NEBW_LN_CASE(16)
#undef NEBW_LN_CASE
  }
  NEBW_CUDA(cudaGetLastError());
  return NEBW_OK;
}

template <int NV>
void launch_lnq_nv(float *x, const float *y, const float *g, const float *b, float eps, int rows,
                   const int *rows_dev, const float *ias, int8_t *q, float *scale,
                   cudaStream_t st) {
  const int grid = (rows + nebw::kRowWarps - 1) / nebw::kRowWarps;
  nebw::layernorm_quant_kernel<NV><<<grid, nebw::kRowWarps * 32, 0, st>>>(
      x, y, g, b, eps, rows, rows_dev, ias, q, scale);
}

// add_norm_quant: x = LN(x + y) for the live rows, and the rows quantised
// for the next int8 GEMM when q is set.
int launch_layernorm_quant(float *x, const float *y, const float *g, const float *b, float eps,
                           int64_t rows, int64_t H, const int *rows_dev, const float *ias,
                           int8_t *q, float *scale, cudaStream_t st) {
  NEBW_REQUIRE(H % 128 == 0 && H >= 128 && H <= 2048,
               "LayerNorm width %lld refused: a multiple of 128 up to 2048 is required",
               static_cast<long long>(H));
  NEBW_REQUIRE(!q || (ias && scale), "quantised LayerNorm output without its divisor or scales");
  NEBW_REQUIRE(rows < (1ll << 31), "LayerNorm rows %lld refused", static_cast<long long>(rows));
  if (rows <= 0) return NEBW_OK;
  const int r = static_cast<int>(rows);
  switch (H / 128) {
#define NEBW_LNQ_CASE(n) \
  case n: launch_lnq_nv<n>(x, y, g, b, eps, r, rows_dev, ias, q, scale, st); break;
    NEBW_LNQ_CASE(1) NEBW_LNQ_CASE(2) NEBW_LNQ_CASE(3) NEBW_LNQ_CASE(4) NEBW_LNQ_CASE(5)
    NEBW_LNQ_CASE(6) NEBW_LNQ_CASE(7) NEBW_LNQ_CASE(8) NEBW_LNQ_CASE(9) NEBW_LNQ_CASE(10)
    NEBW_LNQ_CASE(11) NEBW_LNQ_CASE(12) NEBW_LNQ_CASE(13) NEBW_LNQ_CASE(14) NEBW_LNQ_CASE(15)
    NEBW_LNQ_CASE(16)
#undef NEBW_LNQ_CASE
  }
  NEBW_CUDA(cudaGetLastError());
  return NEBW_OK;
}

// quantise_a_int8 over fp32 or bf16 rows [rows, K] (the live rows when
// rows_dev is set).
int launch_quantise(const void *x, bool x_bf16, int64_t rows, const int *rows_dev, int64_t K,
                    const float *ias, int8_t *q, float *scale, cudaStream_t st) {
  NEBW_REQUIRE(rows >= 0 && rows < (1ll << 31) && K > 0 && K < (1ll << 31),
               "quantise [%lld, %lld] refused", static_cast<long long>(rows),
               static_cast<long long>(K));
  if (rows == 0) return NEBW_OK;
  const bool aligned = reinterpret_cast<uintptr_t>(x) % 16 == 0 &&
                       reinterpret_cast<uintptr_t>(ias) % 16 == 0 &&
                       reinterpret_cast<uintptr_t>(q) % 4 == 0;
  const int r = static_cast<int>(rows), k = static_cast<int>(K);
  const unsigned g8 = static_cast<unsigned>((rows + 7) / 8);
#define NEBW_QW(n)                                                                                 \
  do {                                                                                             \
    if (x_bf16)                                                                                    \
      nebw::quantise_rows_warp_kernel<__nv_bfloat16, n><<<g8, 256, 0, st>>>(                       \
          static_cast<const __nv_bfloat16 *>(x), r, rows_dev, k, ias, q, scale);                   \
    else                                                                                           \
      nebw::quantise_rows_warp_kernel<float, n><<<g8, 256, 0, st>>>(                               \
          static_cast<const float *>(x), r, rows_dev, k, ias, q, scale);                           \
  } while (0)
#define NEBW_QC(n)                                                                                 \
  do {                                                                                             \
    if (x_bf16)                                                                                    \
      nebw::quantise_rows_cta_kernel<__nv_bfloat16, n><<<static_cast<unsigned>(rows),              \
                                                         nebw::kQuantThreads, 0, st>>>(            \
          static_cast<const __nv_bfloat16 *>(x), r, rows_dev, k, ias, q, scale);                   \
    else                                                                                           \
      nebw::quantise_rows_cta_kernel<float, n><<<static_cast<unsigned>(rows),                      \
                                                 nebw::kQuantThreads, 0, st>>>(                    \
          static_cast<const float *>(x), r, rows_dev, k, ias, q, scale);                           \
  } while (0)
  if (K % 4 == 0 && K <= 8192 && aligned) {
    // the row held in registers and read once: a warp per row up to 2048
    // values, a CTA per row beyond
    if (K <= 128) NEBW_QW(1);
    else if (K <= 256) NEBW_QW(2);
    else if (K <= 512) NEBW_QW(4);
    else if (K <= 1024) NEBW_QW(8);
    else if (K <= 2048) NEBW_QW(16);
    else if (K <= 4096) NEBW_QC(4);
    else NEBW_QC(8);
    NEBW_CUDA(cudaGetLastError());
    return NEBW_OK;
  }
#undef NEBW_QW
#undef NEBW_QC
  const unsigned grid = static_cast<unsigned>((rows + 7) / 8);
  if (x_bf16)
    nebw::quantise_rows_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(
        static_cast<const __nv_bfloat16 *>(x), static_cast<int>(rows), rows_dev,
        static_cast<int>(K), ias, q, scale);
  else
    nebw::quantise_rows_kernel<float><<<grid, 256, 0, st>>>(
        static_cast<const float *>(x), static_cast<int>(rows), rows_dev, static_cast<int>(K), ias,
        q, scale);
  NEBW_CUDA(cudaGetLastError());
  return NEBW_OK;
}

template <int BN>
void launch_gemm_i8_bn(const CUtensorMap &mA, const CUtensorMap &mW, const CUtensorMap &mC,
                       const nebw::GemmI8Args &a, bool gelu, dim3 g, cudaStream_t st) {
  const size_t smem = nebw::GemmI8Shape<BN>::kSmemBytes;
  const dim3 b(nebw::kGemmThreads);
  const bool bf16 = a.out_bf16 != nullptr;
  if (gelu && bf16) nebw::gemm_i8_kernel<BN, true, true><<<g, b, smem, st>>>(mA, mW, mC, a);
  else if (gelu) nebw::gemm_i8_kernel<BN, true, false><<<g, b, smem, st>>>(mA, mW, mC, a);
  else if (bf16) nebw::gemm_i8_kernel<BN, false, true><<<g, b, smem, st>>>(mA, mW, mC, a);
  else nebw::gemm_i8_kernel<BN, false, false><<<g, b, smem, st>>>(mA, mW, mC, a);
}

// The int8 GEMM over a staged operand: A's tensor map `mA` (128-row boxes),
// the output's `mC` (make_tmap_out: fp32, or bf16 when a.out_bf16 is set),
// a.M the row bound (a.M_dev the live count).
int launch_gemm_i8(nebw_dev *d, const WeightI8 &w, const CUtensorMap &mA, const CUtensorMap &mC,
                   const nebw::GemmI8Args &a, bool gelu, cudaStream_t st) {
  if (a.M <= 0) return NEBW_OK;
  const bool wide = w.N % 256 == 0;
  if (d->gemm_pairs > 0 && a.K >= 2048) {
    // the CTA-pair GEMM (256-row tiles: a third less operand traffic per SM
    // than the single-CTA tile) with the int8 MMA and epilogue.  Measured
    // faster at K 4096 (2.87 against 2.43 POPS at M 65,536, N 1024) and
    // slower at K 1024 (0.83 against 0.71 ms at M 135,792, N 4096 with
    // gelu8), where the epilogue bounds the tile and the pair's shared
    // accumulator barrier waits on both CTAs' epilogues.
    GemmArgs g{};
    g.M = a.M;
    g.M_dev = a.M_dev;
    g.N = a.N;
    g.K = a.K;
    g.bias = a.bias;
    g.sa = a.sa;
    g.ws = a.ws;
    g.err = a.err;
    g.out = a.out_bf16 ? static_cast<void *>(a.out_bf16) : static_cast<void *>(a.out);
    const int epi = a.out_bf16 ? nebw::kEpiI8Bf16 : gelu ? nebw::kEpiI8Gelu8 : nebw::kEpiI8F32;
    if (wide) return launch_gemm_pair<256>(d, epi, mA, w.map128, mC, g, st);
    return launch_gemm_pair<128>(d, epi, mA, w.map64, mC, g, st);
  }
  const int BN = wide ? 256 : 128;
  const int64_t tiles = ((int64_t{a.M} + nebw::kGemmBM - 1) / nebw::kGemmBM) * ((w.N + BN - 1) / BN);
  const dim3 g(static_cast<unsigned>(std::min<int64_t>(tiles, d->sm_count)));
  if (wide) launch_gemm_i8_bn<256>(mA, w.map256, mC, a, gelu, g, st);
  else launch_gemm_i8_bn<128>(mA, w.map128, mC, a, gelu, g, st);
  NEBW_CUDA(cudaGetLastError());
  return NEBW_OK;
}

template <int NV>
void launch_embed_nv(const int *ids, int B, int S, const int *off, const int *len,
                     const float *word, int vocab, const float *pos, const float *typ,
                     const float *g, const float *b, float eps, float *x, __nv_bfloat16 *a,
                     int *err, cudaStream_t st) {
  const dim3 grid((S + nebw::kRowWarps - 1) / nebw::kRowWarps, B);
  nebw::embed_ln_kernel<NV><<<grid, nebw::kRowWarps * 32, 0, st>>>(ids, S, off, len, word, vocab,
                                                                  pos, typ, g, b, eps, x, a, err);
}

int launch_embed_ln(const int *ids, int B, int S, const int *off, const int *len,
                    const float *word, int vocab, const float *pos, const float *typ,
                    const float *g, const float *b, float eps, int H, float *x,
                    __nv_bfloat16 *a, int *err, cudaStream_t st) {
  NEBW_REQUIRE(H % 128 == 0 && H >= 128 && H <= 2048,
               "hidden %d refused: a multiple of 128 up to 2048 is required", H);
  NEBW_REQUIRE(B > 0 && B <= 65535, "batch %d refused: 1..65535", B);
  switch (H / 128) {
#define NEBW_EMB_CASE(n) \
  case n: launch_embed_nv<n>(ids, B, S, off, len, word, vocab, pos, typ, g, b, eps, x, a, err, st); break;
    NEBW_EMB_CASE(1) NEBW_EMB_CASE(2) NEBW_EMB_CASE(3) NEBW_EMB_CASE(4) NEBW_EMB_CASE(5)
    NEBW_EMB_CASE(6) NEBW_EMB_CASE(7) NEBW_EMB_CASE(8) NEBW_EMB_CASE(9) NEBW_EMB_CASE(10)
    NEBW_EMB_CASE(11) NEBW_EMB_CASE(12) NEBW_EMB_CASE(13) NEBW_EMB_CASE(14) NEBW_EMB_CASE(15)
    NEBW_EMB_CASE(16)
#undef NEBW_EMB_CASE
  }
  NEBW_CUDA(cudaGetLastError());
  return NEBW_OK;
}

int launch_attention(const __nv_bfloat16 *qkv, const int *off, const int *len, int B, int max_len,
                     int heads, int hd, __nv_bfloat16 *ctx, cudaStream_t st) {
  NEBW_REQUIRE(hd == 32 || hd == 64, "head_dim %d refused: 32 or 64", hd);
  NEBW_REQUIRE(B > 0 && B <= 65535 && heads > 0 && heads <= 65535 && max_len > 0,
               "attention grid refused (B %d, heads %d, max_len %d)", B, heads, max_len);
  const int H = heads * hd;
  const dim3 grid((max_len + nebw::kAttnQTile - 1) / nebw::kAttnQTile, heads, B);
  if (hd == 64)
    nebw::attention_kernel<64><<<grid, nebw::kAttnThreads, 0, st>>>(qkv, off, len, H, ctx);
  else
    nebw::attention_kernel<32><<<grid, nebw::kAttnThreads, 0, st>>>(qkv, off, len, H, ctx);
  NEBW_CUDA(cudaGetLastError());
  return NEBW_OK;
}

// tcgen05 attention for head_dim 64 or 32: a persistent launch (three CTAs per SM)
// over the work items -- the device-built, longest-first list `items` with
// its count `items_count`, or, when `items` is null, every (sequence,
// 128-query tile < max_len) pair.
int launch_attention_tc(nebw_dev *d, const CUtensorMap &map, const CUtensorMap &map_kv,
                        const int *off, const int *len,
                        const int *items, const int *items_count, int B, int max_len, int heads,
                        int head_dim, __nv_bfloat16 *ctx, cudaStream_t st) {
  NEBW_REQUIRE(nebw::attn_tc_head_dim(head_dim), "head_dim %d refused by the tcgen05 attention",
               head_dim);
  NEBW_REQUIRE(B > 0 && B <= 65535 && heads > 0 && heads <= 65535 && max_len > 0 &&
                   max_len <= 32767,
               "attention grid refused (B %d, heads %d, max_len %d)", B, heads, max_len);
  const int qtiles = (max_len + 127) / 128;
  const int64_t n_items = static_cast<int64_t>(B) * qtiles;
  NEBW_REQUIRE(n_items * heads < (1ll << 31), "attention work too large");
  const dim3 grid(3 * d->sm_count);
  if (head_dim == 64)
    nebw::attention_tc_kernel<64><<<grid, nebw::kAttnTcThreads, nebw::AttnTcShape<64>::kSmemBytes, st>>>(
        map, map_kv, off, len, items, items_count, static_cast<int>(n_items), qtiles, heads, ctx,
        d->d_err);
  else
    nebw::attention_tc_kernel<32><<<grid, nebw::kAttnTcThreads, nebw::AttnTcShape<32>::kSmemBytes, st>>>(
        map, map_kv, off, len, items, items_count, static_cast<int>(n_items), qtiles, heads, ctx,
        d->d_err);
  NEBW_CUDA(cudaGetLastError());
  return NEBW_OK;
}

// Kernel launches of one attention step: one for either kernel at every
// head_dim and length (the arguments are kept for the launch-count callers).
int attention_launches(int head_dim, int max_len) {
  (void)head_dim;
  (void)max_len;
  return 1;
}

int launch_pool(const float *h, const int *off, const int *len, int B, int H, int pooling, int l2,
                float *out, cudaStream_t st) {
  NEBW_REQUIRE(H > 0 && H <= 16 * nebw::kPoolThreads, "pool width %d refused (<= 4096)", H);
  if (B <= 0) return NEBW_OK;
  nebw::pool_l2_kernel<<<B, nebw::kPoolThreads, 0, st>>>(h, off, len, H,
                                                         pooling == NEBW_POOL_CLS, l2, out);
  NEBW_CUDA(cudaGetLastError());
  return NEBW_OK;
}

int launch_pack(const int *len_in, int B, int S, int *len_out, int *off, int *err,
                cudaStream_t st) {
  NEBW_REQUIRE(B > 0 && B <= (1 << 24), "batch %d refused", B);
  nebw::pack_offsets_kernel<<<1, 1024, 0, st>>>(len_in, B, S, len_out, off, err);
  NEBW_CUDA(cudaGetLastError());
  return NEBW_OK;
}

}  // namespace

// ---------------------------------------------------------------------------
// C ABI: device
// ---------------------------------------------------------------------------

extern "C" const char *nebw_last_error(void) { return g_last_error.c_str(); }
extern "C" int nebw_abi_version(void) { return NEBW_ABI_VERSION; }

template <int BN>
int set_gemm_i8_attrs() {
  const int smem = nebw::GemmI8Shape<BN>::kSmemBytes;
  NEBW_CUDA(cudaFuncSetAttribute(nebw::gemm_i8_kernel<BN, false, false>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  NEBW_CUDA(cudaFuncSetAttribute(nebw::gemm_i8_kernel<BN, true, false>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  NEBW_CUDA(cudaFuncSetAttribute(nebw::gemm_i8_kernel<BN, false, true>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  NEBW_CUDA(cudaFuncSetAttribute(nebw::gemm_i8_kernel<BN, true, true>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  return NEBW_OK;
}

extern "C" int nebw_open(int device, nebw_dev **out) {
  NEBW_REQUIRE(out != nullptr, "null output handle");
  *out = nullptr;
  int n = 0;
  NEBW_CUDA(cudaGetDeviceCount(&n));
  NEBW_REQUIRE(device >= 0 && device < n, "device %d refused: %d CUDA device(s) visible", device, n);
  NEBW_CUDA(cudaSetDevice(device));
  cudaDeviceProp prop;
  NEBW_CUDA(cudaGetDeviceProperties(&prop, device));
  if (prop.major != 10 || prop.minor != 0)
    return set_error(NEBW_EINVAL,
                     "device %d is %s (sm_%d%d); this library is built for sm_100a (B200) only",
                     device, prop.name, prop.major, prop.minor);
  std::unique_ptr<nebw_dev> d(new nebw_dev());
  d->device = device;
  d->sm_count = prop.multiProcessorCount;
  d->cc_major = prop.major;
  d->cc_minor = prop.minor;
  NEBW_CUDA(cudaStreamCreateWithFlags(&d->stream, cudaStreamNonBlocking));
  NEBW_CUDA(cudaMalloc(&d->d_err, sizeof(int)));
  NEBW_CUDA(cudaMemset(d->d_err, 0, sizeof(int)));
  if (int rc = set_all_gemm_attrs()) return rc;
  if (int rc = set_gemm_i8_attrs<128>()) return rc;
  if (int rc = set_gemm_i8_attrs<256>()) return rc;
  NEBW_CUDA(cudaFuncSetAttribute(nebw::attention_tc_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 nebw::AttnTcShape<64>::kSmemBytes));
  NEBW_CUDA(cudaFuncSetAttribute(nebw::attention_tc_kernel<64>, cudaFuncAttributePreferredSharedMemoryCarveout,
                                 cudaSharedmemCarveoutMaxShared));
  NEBW_CUDA(cudaFuncSetAttribute(nebw::attention_tc_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 nebw::AttnTcShape<32>::kSmemBytes));
  NEBW_CUDA(cudaFuncSetAttribute(nebw::attention_tc_kernel<32>, cudaFuncAttributePreferredSharedMemoryCarveout,
                                 cudaSharedmemCarveoutMaxShared));

  if (int rc = query_gemm_pairs(&d->gemm_pairs)) return rc;
  if (int rc = load_tensor_map_encoder()) return rc;
  *out = d.release();
  return NEBW_OK;
}

extern "C" int nebw_close(nebw_dev *d) {
  if (!d) return NEBW_OK;
  cudaSetDevice(d->device);
  cudaStreamSynchronize(d->stream);
  for (auto &kv : d->weights) cudaFree(kv.second.ptr);
  for (auto &kv : d->weights_i8) cudaFree(kv.second.ptr);
  cudaFree(d->d_err);
  cudaStreamDestroy(d->stream);
  if (d->cap_stream) cudaStreamDestroy(d->cap_stream);
  delete d;
  return NEBW_OK;
}

extern "C" int nebw_sync(nebw_dev *d) {
  if (int rc = use_dev(d)) return rc;
  NEBW_CUDA(cudaStreamSynchronize(d->stream));
  int code = 0;
  NEBW_CUDA(cudaMemcpy(&code, d->d_err, sizeof(int), cudaMemcpyDeviceToHost));
  if (code != 0) {
    NEBW_CUDA(cudaMemset(d->d_err, 0, sizeof(int)));
    return set_error(NEBW_EDEVICE, "device error %d: %s", code, dev_err_name(code));
  }
  return NEBW_OK;
}

extern "C" int nebw_check_bounded_wait(nebw_dev *d, int64_t limit_ns, int32_t *expired) {
  NEBW_REQUIRE(expired != nullptr, "null output");
  NEBW_REQUIRE(limit_ns >= 1000 && limit_ns <= 1000000000ll,
               "wait limit %lld ns refused: 1 us .. 1 s", static_cast<long long>(limit_ns));
  if (int rc = use_dev(d)) return rc;
  int *out = nullptr;
  NEBW_CUDA(cudaMalloc(&out, sizeof(int)));
  NEBW_CUDA(cudaMemsetAsync(out, 0xff, sizeof(int), d->stream));
  nebw::wait_probe_kernel<<<1, 32, 0, d->stream>>>(static_cast<uint64_t>(limit_ns), d->d_err, out);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) e = cudaStreamSynchronize(d->stream);
  int v = -1;
  if (e == cudaSuccess) e = cudaMemcpy(&v, out, sizeof(int), cudaMemcpyDeviceToHost);
  cudaFree(out);
  if (e != cudaSuccess)
    return set_error(NEBW_ECUDA, "bounded-wait check: %s", cudaGetErrorString(e));
  NEBW_REQUIRE(v == 0 || v == 1, "bounded-wait check: the probe wrote no result");
  *expired = v;
  return NEBW_OK;
}

extern "C" int nebw_alloc(nebw_dev *d, size_t bytes, void **p) {
  if (int rc = use_dev(d)) return rc;
  NEBW_REQUIRE(p != nullptr, "null output pointer");
  if (cudaMalloc(p, bytes) != cudaSuccess) {
    cudaGetLastError();
    return set_error(NEBW_ENOMEM, "cudaMalloc of %zu bytes failed", bytes);
  }
  return NEBW_OK;
}

extern "C" int nebw_free(nebw_dev *d, void *p) {
  if (int rc = use_dev(d)) return rc;
  NEBW_CUDA(cudaFree(p));
  return NEBW_OK;
}

extern "C" int nebw_copy_h2d(nebw_dev *d, void *dst, const void *src, size_t bytes) {
  if (int rc = use_dev(d)) return rc;
  NEBW_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, d->stream));
  NEBW_CUDA(cudaStreamSynchronize(d->stream));
  return NEBW_OK;
}

extern "C" int nebw_copy_d2h(nebw_dev *d, void *dst, const void *src, size_t bytes) {
  if (int rc = use_dev(d)) return rc;
  NEBW_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, d->stream));
  NEBW_CUDA(cudaStreamSynchronize(d->stream));
  return NEBW_OK;
}

extern "C" int nebw_device_info(nebw_dev *d, int *sm, int *maj, int *min) {
  NEBW_REQUIRE(d != nullptr, "null device handle");
  if (sm) *sm = d->sm_count;
  if (maj) *maj = d->cc_major;
  if (min) *min = d->cc_minor;
  return NEBW_OK;
}

extern "C" int nebw_set_attention_kernel(nebw_dev *d, int kind) {
  NEBW_REQUIRE(d != nullptr, "null device handle");
  NEBW_REQUIRE(kind == NEBW_ATTN_MMA || kind == NEBW_ATTN_TCGEN05, "attention kernel %d refused",
               kind);
  d->attn_kind = kind;
  return NEBW_OK;
}

// ---------------------------------------------------------------------------
// C ABI: weights
// ---------------------------------------------------------------------------

namespace {

int stage_weight(nebw_dev *d, const void *host_kn, int dtype, int64_t K, int64_t N, Weight *w) {
  NEBW_REQUIRE(host_kn != nullptr, "null weight data");
  NEBW_REQUIRE(dtype == NEBW_F32 || dtype == NEBW_BF16, "weight dtype %d refused", dtype);
  NEBW_REQUIRE(K >= 64 && N >= 8 && K % 8 == 0 && N % 8 == 0 && K < (1 << 30) && N < (1 << 30),
               "weight [K=%lld, N=%lld] refused: K >= 64, K %% 8 == 0, N %% 8 == 0",
               static_cast<long long>(K), static_cast<long long>(N));
  const size_t esz = dtype == NEBW_F32 ? 4 : 2;
  const size_t src_bytes = static_cast<size_t>(K) * N * esz;
  void *tmp = nullptr;
  NEBW_CUDA(cudaMalloc(&tmp, src_bytes));
  __nv_bfloat16 *dst = nullptr;
  if (cudaMalloc(&dst, static_cast<size_t>(K) * N * 2) != cudaSuccess) {
    cudaFree(tmp);
    return set_error(NEBW_ENOMEM, "cudaMalloc for a [%lld, %lld] weight failed",
                     static_cast<long long>(N), static_cast<long long>(K));
  }
  cudaError_t e = cudaMemcpyAsync(tmp, host_kn, src_bytes, cudaMemcpyHostToDevice, d->stream);
  if (e == cudaSuccess) {
    const dim3 grid(static_cast<unsigned>((N + 31) / 32), static_cast<unsigned>((K + 31) / 32));
    nebw::stage_weight_kernel<<<grid, dim3(32, 8), 0, d->stream>>>(
        tmp, dtype == NEBW_BF16, static_cast<int>(K), static_cast<int>(N), dst);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) e = cudaStreamSynchronize(d->stream);
  cudaFree(tmp);
  if (e != cudaSuccess) {
    cudaFree(dst);
    return set_error(NEBW_ECUDA, "weight staging failed: %s", cudaGetErrorString(e));
  }
  w->ptr = dst;
  w->K = K;
  w->N = N;
  if (int rc = make_tmap_kmajor(&w->map128, dst, N, K, 128)) {
    cudaFree(dst);
    return rc;
  }
  if (int rc = make_tmap_kmajor(&w->map64, dst, N, K, 64)) {
    cudaFree(dst);
    return rc;
  }
  if (int rc = make_tmap_kmajor(&w->map256, dst, N, K, 256)) {
    cudaFree(dst);
    return rc;
  }
  return NEBW_OK;
}

// An operand already in the device layout (bf16 [N, K], K-major): one upload
// and the tensor maps.
int stage_weight_nk(nebw_dev *d, const uint16_t *host_nk, int64_t K, int64_t N, Weight *w) {
  NEBW_REQUIRE(host_nk != nullptr, "null weight data");
  NEBW_REQUIRE(K >= 64 && N >= 8 && K % 8 == 0 && N % 8 == 0 && K < (1 << 30) && N < (1 << 30),
               "weight [N=%lld, K=%lld] refused: K >= 64, K %% 8 == 0, N %% 8 == 0",
               static_cast<long long>(N), static_cast<long long>(K));
  __nv_bfloat16 *dst = nullptr;
  if (cudaMalloc(&dst, static_cast<size_t>(K) * N * 2) != cudaSuccess) {
    cudaGetLastError();
    return set_error(NEBW_ENOMEM, "cudaMalloc for a [%lld, %lld] weight failed",
                     static_cast<long long>(N), static_cast<long long>(K));
  }
  cudaError_t e = cudaMemcpyAsync(dst, host_nk, static_cast<size_t>(K) * N * 2,
                                  cudaMemcpyHostToDevice, d->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(d->stream);
  if (e != cudaSuccess) {
    cudaFree(dst);
    return set_error(NEBW_ECUDA, "weight upload failed: %s", cudaGetErrorString(e));
  }
  w->ptr = dst;
  w->K = K;
  w->N = N;
  for (auto mp : {std::make_pair(&w->map64, 64), std::make_pair(&w->map128, 128),
                  std::make_pair(&w->map256, 256)})
    if (int rc = make_tmap_kmajor(mp.first, dst, N, K, mp.second)) {
      cudaFree(dst);
      w->ptr = nullptr;
      return rc;
    }
  return NEBW_OK;
}

}  // namespace

extern "C" int nebw_stage_weight(nebw_dev *d, const void *host_kn, int dtype, int64_t K, int64_t N,
                                 uint64_t *handle) {
  if (int rc = use_dev(d)) return rc;
  NEBW_REQUIRE(handle != nullptr, "null handle output");
  Weight w;
  if (int rc = stage_weight(d, host_kn, dtype, K, N, &w)) return rc;
  *handle = d->next_handle++;
  d->weights[*handle] = w;
  return NEBW_OK;
}

extern "C" int nebw_release_weight(nebw_dev *d, uint64_t handle) {
  if (int rc = use_dev(d)) return rc;
  auto it = d->weights.find(handle);
  auto it8 = d->weights_i8.find(handle);
  NEBW_REQUIRE(it != d->weights.end() || it8 != d->weights_i8.end(),
               "unknown weight handle %llu", static_cast<unsigned long long>(handle));
  NEBW_CUDA(cudaStreamSynchronize(d->stream));
  if (it != d->weights.end()) {
    cudaFree(it->second.ptr);
    d->weights.erase(it);
  } else {
    cudaFree(it8->second.ptr);
    d->weights_i8.erase(it8);
  }
  return NEBW_OK;
}

// ---------------------------------------------------------------------------
// C ABI: ops
// ---------------------------------------------------------------------------

extern "C" int nebw_gemm(nebw_dev *d, uint64_t weight, const void *A, int64_t M, int64_t K,
                         int64_t N, const float *bias, const float *residual, int act, void *C,
                         int c_dtype, void *stream) {
  if (int rc = use_dev(d)) return rc;
  auto it = d->weights.find(weight);
  NEBW_REQUIRE(it != d->weights.end(), "unknown weight handle %llu",
               static_cast<unsigned long long>(weight));
  const Weight &w = it->second;
  NEBW_REQUIRE(K == w.K && N == w.N, "GEMM [M, %lld] x [%lld, %lld] does not match the staged "
               "weight [K=%lld, N=%lld]", static_cast<long long>(K), static_cast<long long>(K),
               static_cast<long long>(N), static_cast<long long>(w.K), static_cast<long long>(w.N));
  NEBW_REQUIRE(M >= 0 && M < (1 << 30), "M %lld refused", static_cast<long long>(M));
  NEBW_REQUIRE(A != nullptr && C != nullptr, "null GEMM operand");
  NEBW_REQUIRE(c_dtype == NEBW_F32 || c_dtype == NEBW_BF16, "output dtype %d refused", c_dtype);
  NEBW_REQUIRE(act == NEBW_ACT_NONE || act == NEBW_ACT_GELU8 || act == NEBW_ACT_GELU_ERF,
               "activation %d refused", act);
  NEBW_REQUIRE(!(residual && c_dtype != NEBW_F32), "a residual needs fp32 output");
  NEBW_REQUIRE(!(act != NEBW_ACT_NONE && c_dtype != NEBW_BF16),
               "an activation epilogue writes bf16 output");
  NEBW_REQUIRE(reinterpret_cast<uintptr_t>(C) % 16 == 0 &&
                   (!residual || reinterpret_cast<uintptr_t>(residual) % 16 == 0) &&
                   (!bias || reinterpret_cast<uintptr_t>(bias) % 16 == 0),
               "GEMM output, residual and bias must be 16-byte aligned");
  if (M == 0) return NEBW_OK;
  CUtensorMap mA, mC;
  if (int rc = make_tmap_kmajor(&mA, A, M, K, nebw::kGemmBM)) return rc;
  if (int rc = make_tmap_out(&mC, C, M, N, c_dtype == NEBW_BF16)) return rc;
  GemmArgs a{};
  a.M = static_cast<int>(M);
  a.M_dev = nullptr;
  a.N = static_cast<int>(N);
  a.K = static_cast<int>(K);
  a.bias = bias;
  a.resid = residual;
  a.out = C;
  a.err = d->d_err;
  return launch_gemm(d, w, mA, mC, pick_epi(act, c_dtype, residual != nullptr), a,
                     pick_stream(d, stream));
}

extern "C" int nebw_layernorm(nebw_dev *d, float *x, const void *y, int y_dtype,
                              const float *gamma, const float *beta, float eps, int64_t rows,
                              int64_t H, void *a_bf16, void *stream) {
  if (int rc = use_dev(d)) return rc;
  NEBW_REQUIRE(x && gamma && beta, "null LayerNorm operand");
  NEBW_REQUIRE(y_dtype == NEBW_F32 || y_dtype == NEBW_BF16, "y dtype %d refused", y_dtype);
  NEBW_REQUIRE(rows >= 0 && rows < (1ll << 31) / 2, "rows %lld refused", static_cast<long long>(rows));
  return launch_layernorm(x, y, y_dtype == NEBW_BF16, gamma, beta, eps, rows, H, nullptr,
                          static_cast<__nv_bfloat16 *>(a_bf16), pick_stream(d, stream));
}

extern "C" int nebw_attention(nebw_dev *d, const void *qkv, int64_t rows, const int32_t *off,
                              const int32_t *len, int32_t B, int32_t max_len, int32_t heads,
                              int32_t hd, void *ctx, void *stream) {
  if (int rc = use_dev(d)) return rc;
  NEBW_REQUIRE(qkv && off && len && ctx, "null attention operand");
  NEBW_REQUIRE(rows > 0 && rows < (1ll << 31), "rows %lld refused", static_cast<long long>(rows));
  if (d->attn_kind == NEBW_ATTN_TCGEN05 && nebw::attn_tc_head_dim(hd)) {
    CUtensorMap map, map_kv;
    if (int rc = make_tmap_head(&map, qkv, rows, 3 * static_cast<int64_t>(heads) * hd, hd, 128))
      return rc;
    if (int rc = make_tmap_head(&map_kv, qkv, rows, 3 * static_cast<int64_t>(heads) * hd, hd, 64))
      return rc;
    return launch_attention_tc(d, map, map_kv, off, len, nullptr, nullptr, B, max_len, heads, hd,
                               static_cast<__nv_bfloat16 *>(ctx), pick_stream(d, stream));
  }
  return launch_attention(static_cast<const __nv_bfloat16 *>(qkv), off, len, B, max_len, heads, hd,
                          static_cast<__nv_bfloat16 *>(ctx), pick_stream(d, stream));
}

extern "C" int nebw_pack_offsets(nebw_dev *d, const int32_t *len_in, int32_t B, int32_t S,
                                 int32_t *len_out, int32_t *off, void *stream) {
  if (int rc = use_dev(d)) return rc;
  NEBW_REQUIRE(len_in && len_out && off, "null packing operand");
  return launch_pack(len_in, B, S, len_out, off, d->d_err, pick_stream(d, stream));
}

extern "C" int nebw_embed_ln(nebw_dev *d, const int32_t *ids, const int32_t *off,
                             const int32_t *len, int32_t B, int32_t S, const float *word,
                             int32_t vocab, const float *pos, const float *typ, const float *gamma,
                             const float *beta, float eps, int32_t H, float *x, void *a_bf16,
                             void *stream) {
  if (int rc = use_dev(d)) return rc;
  NEBW_REQUIRE(ids && off && len && word && pos && typ && gamma && beta && x,
               "null embedding operand");
  return launch_embed_ln(ids, B, S, off, len, word, vocab, pos, typ, gamma, beta, eps, H, x,
                         static_cast<__nv_bfloat16 *>(a_bf16), d->d_err, pick_stream(d, stream));
}

extern "C" int nebw_pool_l2(nebw_dev *d, const float *h, const int32_t *off, const int32_t *len,
                            int32_t B, int32_t H, int pooling, int l2, float *out, void *stream) {
  if (int rc = use_dev(d)) return rc;
  NEBW_REQUIRE(h && off && len && out, "null pooling operand");
  NEBW_REQUIRE(pooling == NEBW_POOL_MEAN || pooling == NEBW_POOL_CLS, "pooling %d refused", pooling);
  return launch_pool(h, off, len, B, H, pooling, l2, out, pick_stream(d, stream));
}

extern "C" int nebw_narrow_bf16(nebw_dev *d, const float *x, int64_t n, void *y, void *stream) {
  if (int rc = use_dev(d)) return rc;
  NEBW_REQUIRE(x && y && n >= 0, "bad narrow operand");
  NEBW_REQUIRE(reinterpret_cast<uintptr_t>(x) % 16 == 0 && reinterpret_cast<uintptr_t>(y) % 8 == 0,
               "narrow operands must be 16/8-byte aligned");
  if (n == 0) return NEBW_OK;
  const int64_t threads = 256, per = 4;
  const int64_t blocks = (n + threads * per - 1) / (threads * per);
  nebw::narrow_bf16_kernel<<<static_cast<unsigned>(blocks), threads, 0, pick_stream(d, stream)>>>(
      x, n, static_cast<__nv_bfloat16 *>(y));
  NEBW_CUDA(cudaGetLastError());
  return NEBW_OK;
}

// ---- the int8 datapath (the reference's --dtype i8 array path) -------------

namespace {
// An int8 operand [K, N] (host, row-major) staged as [N, K] (the tensor-core
// B layout) with its 128- and 256-row tensor maps.
int stage_i8(const int8_t *host_kn, int64_t K, int64_t N, WeightI8 &w) {
  NEBW_REQUIRE(K > 0 && N > 0 && K % 16 == 0 && N % 8 == 0,
               "int8 weight [%lld, %lld] refused: K %% 16 == 0 and N %% 8 == 0 required",
               static_cast<long long>(K), static_cast<long long>(N));
  std::vector<int8_t> nk(static_cast<size_t>(K * N));
  for (int64_t k = 0; k < K; ++k)
    for (int64_t n = 0; n < N; ++n) nk[static_cast<size_t>(n * K + k)] = host_kn[k * N + n];
  w = WeightI8{};
  w.K = K;
  w.N = N;
  NEBW_CUDA(cudaMalloc(&w.ptr, nk.size()));
  if (cudaMemcpy(w.ptr, nk.data(), nk.size(), cudaMemcpyHostToDevice) != cudaSuccess) {
    cudaGetLastError();
    cudaFree(w.ptr);
    w.ptr = nullptr;
    return set_error(NEBW_ECUDA, "int8 weight upload failed");
  }
  int rc = make_tmap_i8(&w.map64, w.ptr, N, K, 64);
  if (!rc) rc = make_tmap_i8(&w.map128, w.ptr, N, K, 128);
  if (!rc) rc = make_tmap_i8(&w.map256, w.ptr, N, K, 256);
  if (rc) {
    cudaFree(w.ptr);
    w.ptr = nullptr;
  }
  return rc;
}
}  // namespace

extern "C" int nebw_stage_weight_i8(nebw_dev *d, const int8_t *host_kn, int64_t K, int64_t N,
                                    uint64_t *handle) {
  if (int rc = use_dev(d)) return rc;
  NEBW_REQUIRE(host_kn && handle, "null argument");
  WeightI8 w;
  if (int rc = stage_i8(host_kn, K, N, w)) return rc;
  const uint64_t h = d->next_handle++;
  d->weights_i8[h] = w;
  *handle = h;
  return NEBW_OK;
}

extern "C" int nebw_gemm_i8_ex(nebw_dev *d, uint64_t weight, const int8_t *A, const float *sa,
                               int64_t M, int64_t K, int64_t N, const float *ws, const float *bias,
                               int act, void *C, int c_dtype, void *stream) {
  if (int rc = use_dev(d)) return rc;
  auto it = d->weights_i8.find(weight);
  NEBW_REQUIRE(it != d->weights_i8.end(), "unknown int8 weight handle %llu",
               static_cast<unsigned long long>(weight));
  const WeightI8 &w = it->second;
  NEBW_REQUIRE(K == w.K && N == w.N, "int8 GEMM [%lld x %lld] . [%lld x %lld] mismatch",
               static_cast<long long>(M), static_cast<long long>(K),
               static_cast<long long>(w.K), static_cast<long long>(w.N));
  NEBW_REQUIRE(A && sa && ws && C, "null int8 GEMM operand");
  NEBW_REQUIRE(M >= 0 && M < (1ll << 31), "M %lld refused", static_cast<long long>(M));
  NEBW_REQUIRE(act == NEBW_ACT_NONE || act == NEBW_ACT_GELU8, "int8 GEMM act %d refused", act);
  NEBW_REQUIRE(c_dtype == NEBW_F32 || c_dtype == NEBW_BF16, "int8 GEMM c_dtype %d refused",
               c_dtype);
  NEBW_REQUIRE(reinterpret_cast<uintptr_t>(C) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(ws) % 16 == 0 &&
                   (!bias || reinterpret_cast<uintptr_t>(bias) % 16 == 0),
               "int8 GEMM C, ws and bias must be 16-byte aligned");
  if (M == 0) return NEBW_OK;
  CUtensorMap mA, mC;
  if (int rc = make_tmap_i8(&mA, A, M, K, nebw::kGemmBM)) return rc;
  if (int rc = make_tmap_out(&mC, C, M, N, c_dtype == NEBW_BF16)) return rc;
  nebw::GemmI8Args a{};
  a.M = static_cast<int>(M);
  a.N = static_cast<int>(N);
  a.K = static_cast<int>(K);
  a.sa = sa;
  a.ws = ws;
  a.bias = bias;
  if (c_dtype == NEBW_F32) a.out = static_cast<float *>(C);
  else a.out_bf16 = static_cast<__nv_bfloat16 *>(C);
  a.err = d->d_err;
  return launch_gemm_i8(d, w, mA, mC, a, act == NEBW_ACT_GELU8, pick_stream(d, stream));
}

extern "C" int nebw_gemm_i8(nebw_dev *d, uint64_t weight, const int8_t *A, const float *sa,
                            int64_t M, int64_t K, int64_t N, const float *ws, const float *bias,
                            int act, float *C, void *stream) {
  return nebw_gemm_i8_ex(d, weight, A, sa, M, K, N, ws, bias, act, C, NEBW_F32, stream);
}

extern "C" int nebw_quantise_rows(nebw_dev *d, const float *x, int64_t rows, int64_t K,
                                  const float *ias, int8_t *q, float *scale, void *stream) {
  if (int rc = use_dev(d)) return rc;
  NEBW_REQUIRE(x && ias && q && scale, "null quantise operand");
  return launch_quantise(x, false, rows, nullptr, K, ias, q, scale, pick_stream(d, stream));
}

extern "C" int nebw_quantise_rows_bf16(nebw_dev *d, const void *x, int64_t rows, int64_t K,
                                       const float *ias, int8_t *q, float *scale, void *stream) {
  if (int rc = use_dev(d)) return rc;
  NEBW_REQUIRE(x && ias && q && scale, "null quantise operand");
  return launch_quantise(x, true, rows, nullptr, K, ias, q, scale, pick_stream(d, stream));
}

extern "C" int nebw_layernorm_quant(nebw_dev *d, float *x, const float *y, const float *g,
                                    const float *b, float eps, int64_t rows, int64_t H,
                                    const float *ias, int8_t *q, float *scale, void *stream) {
  if (int rc = use_dev(d)) return rc;
  NEBW_REQUIRE(x && g && b, "null LayerNorm operand");
  for (const void *p : {static_cast<const void *>(x), static_cast<const void *>(y),
                        static_cast<const void *>(g), static_cast<const void *>(b),
                        static_cast<const void *>(ias)})
    NEBW_REQUIRE(reinterpret_cast<uintptr_t>(p) % 16 == 0,
                 "LayerNorm operands must be 16-byte aligned");
  NEBW_REQUIRE(!q || reinterpret_cast<uintptr_t>(q) % 4 == 0, "q must be 4-byte aligned");
  return launch_layernorm_quant(x, y, g, b, eps, rows, H, nullptr, ias, q, scale,
                                pick_stream(d, stream));
}

// ---------------------------------------------------------------------------
// C ABI: the whole encoder
// ---------------------------------------------------------------------------

struct LayerW {
  Weight qkv, ao, up, dn;
  float *b_qkv = nullptr, *b_ao = nullptr, *b_up = nullptr, *b_dn = nullptr;
  float *ln1_g = nullptr, *ln1_b = nullptr, *ln2_g = nullptr, *ln2_b = nullptr;
};

// An int8 GEMM operand of the int8 datapath (nebw_model_set_int8_operand):
// int8 [N, K] on the device with its tensor maps, the column scales and the
// reciprocals of the activation's SmoothQuant divisors.
struct OperandI8 {
  WeightI8 w;
  float *ws = nullptr;   // [N]
  float *ias = nullptr;  // [K], 1 / asmooth in float
};
struct LayerI8 {
  OperandI8 qkv, ao, up, dn;
};

// The activation buffers of one encoder pass: the model's own (grown with
// cudaMalloc to the largest batch seen) or a view carved out of the static
// scratch of nebw_encode_device_static.
struct Workspace {
  int64_t rows_cap = 0, batch_cap = 0;  // padded rows B * S and sequences it holds
  float *x = nullptr;                   // residual stream (fp32)
  __nv_bfloat16 *y = nullptr;           // sublayer output: AO / FFN-down GEMM, RNE bf16
  __nv_bfloat16 *a = nullptr, *qkv = nullptr, *ctx = nullptr, *h = nullptr;
  int *len = nullptr, *off = nullptr;
  int *att_items = nullptr;  // attention work list (longest first) [B * S/128 + B + 1]
  // rotary positions applied in the QKV GEMM's epilogue (CTA pairs,
  // head_dim 64): the position of each packed row, [rows_cap] ints
  int *row_pos = nullptr;
  CUtensorMap map_qkv_att, map_kv_att;  // Q|K|V head tiles, head_dim x 128 / head_dim x 64 rows
  CUtensorMap map_a, map_ctx, map_h;    // GEMM A operands (TMA loads)
  CUtensorMap out_qkv, out_y, out_h;    // GEMM outputs (TMA stores)
  // the int8 datapath's buffers (allocated only for it): the quantised A
  // rows [rows, max(H, F)] with their scales [rows], the dequantised fp32
  // outputs of the attention-out / FFN-down GEMMs [rows, H] and of FFN-up
  // [rows, F]; A's tensor maps at K = H and K = F
  int8_t *aq = nullptr;
  float *sa = nullptr, *y32 = nullptr, *h32 = nullptr;
  CUtensorMap map_aq_h, map_aq_f;
  CUtensorMap out_y32, out_h32;  // int8 GEMM outputs (TMA stores)
};

struct nebw_model {
  nebw_dev *dev = nullptr;
  nebw_config cfg{};
  float *word = nullptr, *pos = nullptr, *typ = nullptr, *emb_g = nullptr, *emb_b = nullptr;
  // rotary tables [max_seq_len, head_dim] fp32 (cfg.rope), built on first use
  // from rope_freq (nebw_model_set_rope_freq) or cfg.rope_theta
  float *rope_cos = nullptr, *rope_sin = nullptr;
  std::vector<double> rope_freq;
  // gated FFN with the GLU fused into the FFN-up GEMM's epilogue (CTA pairs
  // available): ffn_up's columns are staged interleaved in groups of 64 =
  // [32 up | 32 gate] and the GEMM writes h [rows, F] directly
  bool glu_fused = false;
  std::vector<LayerW> layers;
  std::map<std::string, bool> staged;  // container name -> set
  // the int8 datapath: its operands (sized to the layers on the first set)
  // and the arithmetic the passes run (NEBW_DATAPATH_BF16 / _I8)
  std::vector<LayerI8> i8;
  int datapath = NEBW_DATAPATH_BF16;
  // CUDA graphs of whole passes (nebw_model_set_graphs): one per (B, S,
  // datapath, attention kernel), replayed by nebw_encode between its input
  // and output copies; dropped whenever what they captured changes (the
  // weights, the workspace, the datapath)
  struct PassGraph {
    int B, S, datapath, attn;
    const int *ids, *lens;
    float *out;
    cudaGraphExec_t exec;
  };
  bool use_graphs = false;
  std::vector<PassGraph> graphs;
  Workspace ws;                        // capacity ws.rows_cap = B * S of the largest call so far
  // host-buffer entry point (nebw_encode): device copies of its inputs and output
  int64_t ids_cap = 0;
  int *ids = nullptr, *len_in = nullptr;
  float *out = nullptr;
  // per-kernel timing: one event before each launch (tagged with the kernel
  // kind) and one after the last; interval i belongs to marks[i].kind
  bool prof = false;
  std::vector<std::pair<cudaEvent_t, int>> marks;
  std::vector<cudaEvent_t> ev_pool;
  size_t ev_used = 0;
};

namespace {

constexpr size_t kMaxPassGraphs = 16;

void drop_graphs(nebw_model *m) {
  if (m->graphs.empty()) return;
  cudaDeviceSynchronize();  // no replay may still be running, on whatever stream
  for (auto &g : m->graphs) cudaGraphExecDestroy(g.exec);
  m->graphs.clear();
}

void free_workspace(nebw_model *m) {
  drop_graphs(m);
  Workspace &w = m->ws;
  for (void *p : {static_cast<void *>(w.x), static_cast<void *>(w.y), static_cast<void *>(w.a),
                  static_cast<void *>(w.qkv), static_cast<void *>(w.ctx), static_cast<void *>(w.h),
                  static_cast<void *>(w.len), static_cast<void *>(w.off),
                  static_cast<void *>(w.att_items), static_cast<void *>(w.row_pos),
                  static_cast<void *>(w.aq), static_cast<void *>(w.sa),
                  static_cast<void *>(w.y32), static_cast<void *>(w.h32),
                  static_cast<void *>(m->ids), static_cast<void *>(m->len_in),
                  static_cast<void *>(m->out)})
    cudaFree(p);
  w = Workspace{};
  m->ids = m->len_in = nullptr;
  m->out = nullptr;
  m->ids_cap = 0;
}

// Whether the QKV GEMM's epilogue applies the rotary positions (it needs a
// [rows] position array in the workspace): rotary models with head_dim 64
// on a GPU with CTA pairs.
bool rope_in_epilogue(const nebw_model *m) {
  return m->cfg.rope && m->cfg.head_dim == 64 && m->dev->gemm_pairs > 0;
}

// Width of the FFN-up output buffer h: [up | gate] when the GLU is a
// separate pass, else F.
int64_t ffn_up_width(const nebw_model *m) {
  return m->cfg.gated_ffn && !m->glu_fused ? 2 * int64_t{m->cfg.intermediate}
                                           : int64_t{m->cfg.intermediate};
}

// The TMA descriptors of a workspace whose buffers are set, for `R` rows.
int make_workspace_maps(const nebw_model *m, Workspace &w, int64_t R) {
  const int64_t H = m->cfg.hidden, F = m->cfg.intermediate, FW = ffn_up_width(m);
  int rc;
  if ((rc = make_tmap_kmajor(&w.map_a, w.a, R, H, nebw::kGemmBM))) return rc;
  if ((rc = make_tmap_kmajor(&w.map_ctx, w.ctx, R, H, nebw::kGemmBM))) return rc;
  // FFN-down reads the first F columns of each FW-wide row of h
  if ((rc = make_tmap_kmajor(&w.map_h, w.h, R, F, nebw::kGemmBM, FW))) return rc;
  if ((rc = make_tmap_out(&w.out_qkv, w.qkv, R, 3 * H, true))) return rc;
  if ((rc = make_tmap_out(&w.out_y, w.y, R, H, true))) return rc;
  if ((rc = make_tmap_out(&w.out_h, w.h, R, FW, true))) return rc;
  if (nebw::attn_tc_head_dim(m->cfg.head_dim)) {
    if ((rc = make_tmap_head(&w.map_qkv_att, w.qkv, R, 3 * H, m->cfg.head_dim, 128))) return rc;
    if ((rc = make_tmap_head(&w.map_kv_att, w.qkv, R, 3 * H, m->cfg.head_dim, 64))) return rc;
  }
  if (w.aq) {
    if ((rc = make_tmap_i8(&w.map_aq_h, w.aq, R, H, nebw::kGemmBM))) return rc;
    if ((rc = make_tmap_i8(&w.map_aq_f, w.aq, R, F, nebw::kGemmBM))) return rc;
    if ((rc = make_tmap_out(&w.out_y32, w.y32, R, H, false))) return rc;
    if ((rc = make_tmap_out(&w.out_h32, w.h32, R, F, false))) return rc;
  }
  return NEBW_OK;
}

int ensure_workspace(nebw_model *m, int64_t B, int64_t S) {
  const int64_t rows = B * S;
  const bool need_i8 = m->datapath == NEBW_DATAPATH_I8;
  if (rows <= m->ws.rows_cap && B <= m->ws.batch_cap && (!need_i8 || m->ws.aq)) return NEBW_OK;
  NEBW_CUDA(cudaStreamSynchronize(m->dev->stream));
  const int64_t R = std::max(rows, m->ws.rows_cap), Bc = std::max(B, m->ws.batch_cap);
  free_workspace(m);
  const int64_t H = m->cfg.hidden, FW = ffn_up_width(m);
  auto alloc = [&](void **p, size_t bytes) -> int {
    if (cudaMalloc(p, bytes) != cudaSuccess) {
      cudaGetLastError();
      return set_error(NEBW_ENOMEM, "workspace allocation of %zu bytes failed", bytes);
    }
    return NEBW_OK;
  };
  Workspace &w = m->ws;
  int rc = 0;
  rc = rc ? rc : alloc(reinterpret_cast<void **>(&w.x), R * H * 4);
  rc = rc ? rc : alloc(reinterpret_cast<void **>(&w.y), R * H * 2);
  rc = rc ? rc : alloc(reinterpret_cast<void **>(&w.a), R * H * 2);
  rc = rc ? rc : alloc(reinterpret_cast<void **>(&w.qkv), R * 3 * H * 2);
  rc = rc ? rc : alloc(reinterpret_cast<void **>(&w.ctx), R * H * 2);
  rc = rc ? rc : alloc(reinterpret_cast<void **>(&w.h), R * FW * 2);
  rc = rc ? rc : alloc(reinterpret_cast<void **>(&w.len), Bc * 4);
  rc = rc ? rc : alloc(reinterpret_cast<void **>(&w.off), (Bc + 1) * 4);
  rc = rc ? rc : alloc(reinterpret_cast<void **>(&w.att_items), (R / 128 + Bc + 1) * 4);
  if (rope_in_epilogue(m)) rc = rc ? rc : alloc(reinterpret_cast<void **>(&w.row_pos), R * 4);
  if (need_i8) {
    const int64_t F = m->cfg.intermediate;
    rc = rc ? rc : alloc(reinterpret_cast<void **>(&w.aq), R * std::max(H, F));
    rc = rc ? rc : alloc(reinterpret_cast<void **>(&w.sa), R * 4);
    rc = rc ? rc : alloc(reinterpret_cast<void **>(&w.y32), R * H * 4);
    rc = rc ? rc : alloc(reinterpret_cast<void **>(&w.h32), R * F * 4);
  }
  rc = rc ? rc : alloc(reinterpret_cast<void **>(&m->ids), R * 4);
  rc = rc ? rc : alloc(reinterpret_cast<void **>(&m->len_in), Bc * 4);
  rc = rc ? rc : alloc(reinterpret_cast<void **>(&m->out), Bc * H * 4);
  if (rc) {
    free_workspace(m);
    return rc;
  }
  w.rows_cap = R;
  w.batch_cap = Bc;
  m->ids_cap = R;
  return make_workspace_maps(m, w, R);
}

int upload_f32(nebw_dev *d, float **dst, const void *src, int dtype, int64_t n) {
  NEBW_REQUIRE(dtype == NEBW_F32, "this tensor must be F32 (as the container stores it)");
  if (*dst == nullptr) NEBW_CUDA(cudaMalloc(dst, n * 4));
  NEBW_CUDA(cudaMemcpyAsync(*dst, src, n * 4, cudaMemcpyHostToDevice, d->stream));
  NEBW_CUDA(cudaStreamSynchronize(d->stream));
  return NEBW_OK;
}

// Column n of the interleaved gated FFN-up operand (groups of 64 = [32 up |
// 32 gate] of the same 32 output columns) takes column glu_src(n) of the
// container's [up | gate] halves.
int64_t glu_src(int64_t n, int64_t F) {
  const int64_t g = n / 64, i = n % 64;
  return i < 32 ? g * 32 + i : F + g * 32 + (i - 32);
}

// A host [rows, cols] array of `esize`-byte elements with its columns
// (by_rows false) or rows (by_rows true) reordered by glu_src.
std::vector<unsigned char> glu_interleave(const void *src, int64_t rows, int64_t cols,
                                          size_t esize, int64_t F, bool by_rows) {
  std::vector<unsigned char> out(static_cast<size_t>(rows * cols) * esize);
  const unsigned char *in = static_cast<const unsigned char *>(src);
  if (by_rows) {
    for (int64_t r = 0; r < rows; ++r)
      std::memcpy(&out[static_cast<size_t>(r * cols) * esize],
                  in + static_cast<size_t>(glu_src(r, F) * cols) * esize,
                  static_cast<size_t>(cols) * esize);
  } else {
    for (int64_t r = 0; r < rows; ++r)
      for (int64_t n = 0; n < cols; ++n)
        std::memcpy(&out[static_cast<size_t>(r * cols + n) * esize],
                    in + static_cast<size_t>(r * cols + glu_src(n, F)) * esize, esize);
  }
  return out;
}

std::vector<std::string> required_names(const nebw_config &c) {
  std::vector<std::string> v = {"embeddings.word", "embeddings.token_type",
                                "embeddings.ln.weight", "embeddings.ln.bias"};
  if (!c.rope) v.push_back("embeddings.position");  // rotary models need no table
  for (int L = 0; L < c.num_layers; ++L) {
    const std::string p = "layer." + std::to_string(L) + ".";
    for (const char *s : {"qkv", "qkv.bias", "attn_out", "attn_out.bias", "ln1.weight", "ln1.bias",
                          "ffn_up", "ffn_up.bias", "ffn_down", "ffn_down.bias", "ln2.weight",
                          "ln2.bias"})
      v.push_back(p + s);
  }
  return v;
}

int model_ready(const nebw_model *m) {
  for (const auto &n : required_names(m->cfg))
    if (!m->staged.count(n))
      return set_error(NEBW_ESTATE, "model tensor '%s' has not been staged", n.c_str());
  return NEBW_OK;
}

// Rotary models: the cos / sin tables [max_seq_len, head_dim] as
// apply_rope_qkv builds them (bert_encoder.cpp:929-952): angle = s *
// inv_freq[j] in double, cos and sin rounded to fp32, the same value in
// columns j and j + head_dim/2; inv_freq from the container's data or
// theta^(-2j / head_dim) (gemma_rope_tables, gemma_kernels.cpp:114-136).
// A rotary model gets a zero position table at creation (the reference's
// containers carry a zero placeholder that its embedding adds; a staged
// table overwrites it).  Built when the model is created (theta known) or
// its frequency set is given, never during a pass -- the static-scratch
// entry point allocates nothing.
int build_rope(nebw_model *m) {
  const nebw_config &c = m->cfg;
  if (!c.rope) return NEBW_OK;
  const int64_t H = c.hidden, S = c.max_seq_len, hd = c.head_dim, half = hd / 2;
  if (!m->pos) {
    NEBW_CUDA(cudaMalloc(&m->pos, S * H * 4));
    NEBW_CUDA(cudaMemset(m->pos, 0, S * H * 4));
  }
  if (m->rope_cos) return NEBW_OK;
  if (m->rope_freq.empty() && !(c.rope_theta > 0.0)) return NEBW_OK;  // set later
  std::vector<double> inv(static_cast<size_t>(half));
  if (!m->rope_freq.empty()) {
    inv = m->rope_freq;
  } else {
    for (int64_t j = 0; j < half; ++j)
      inv[static_cast<size_t>(j)] =
          1.0 / std::pow(c.rope_theta, 2.0 * static_cast<double>(j) / static_cast<double>(hd));
  }
  std::vector<float> cs(static_cast<size_t>(S * hd)), sn(static_cast<size_t>(S * hd));
  for (int64_t s = 0; s < S; ++s)
    for (int64_t j = 0; j < half; ++j) {
      const double ang = static_cast<double>(s) * inv[static_cast<size_t>(j)];
      const float cv = static_cast<float>(std::cos(ang)), sv = static_cast<float>(std::sin(ang));
      cs[s * hd + j] = cs[s * hd + half + j] = cv;
      sn[s * hd + j] = sn[s * hd + half + j] = sv;
    }
  float *dc = nullptr, *ds = nullptr;
  NEBW_CUDA(cudaMalloc(&dc, cs.size() * 4));
  NEBW_CUDA(cudaMalloc(&ds, sn.size() * 4));
  NEBW_CUDA(cudaMemcpy(dc, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice));
  NEBW_CUDA(cudaMemcpy(ds, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice));
  m->rope_cos = dc;
  m->rope_sin = ds;
  return NEBW_OK;
}

// A pass over a rotary model needs its tables (built at creation or by
// nebw_model_set_rope_freq).
int rope_ready(const nebw_model *m) {
  NEBW_REQUIRE(!m->cfg.rope || (m->rope_cos && m->pos),
               "rotary model without its frequency set: give rope_theta at creation or call "
               "nebw_model_set_rope_freq");
  return NEBW_OK;
}

int launch_rope(const nebw_model *m, const Workspace &w, int B, int S, cudaStream_t st) {
  const nebw_config &c = m->cfg;
  const dim3 grid((S + nebw::kRowWarps - 1) / nebw::kRowWarps, B);
  if (c.head_dim == 64)
    nebw::rope_qk_kernel<64><<<grid, nebw::kRowWarps * 32, 0, st>>>(
        w.qkv, w.off, w.len, c.hidden, m->rope_cos, m->rope_sin);
  else
    nebw::rope_qk_kernel<32><<<grid, nebw::kRowWarps * 32, 0, st>>>(
        w.qkv, w.off, w.len, c.hidden, m->rope_cos, m->rope_sin);
  NEBW_CUDA(cudaGetLastError());
  return NEBW_OK;
}

int launch_glu(const nebw_model *m, const Workspace &w, int rows, const int *rows_dev,
               cudaStream_t st) {
  const int64_t F = m->cfg.intermediate;
  const int64_t threads = static_cast<int64_t>(rows) * (F / 8);
  const unsigned grid = static_cast<unsigned>((threads + 255) / 256);
  if (m->cfg.gated_act == NEBW_GATE_SILU)
    nebw::glu_kernel<0><<<grid, 256, 0, st>>>(w.h, rows, rows_dev, static_cast<int>(F));
  else
    nebw::glu_kernel<1><<<grid, 256, 0, st>>>(w.h, rows, rows_dev, static_cast<int>(F));
  NEBW_CUDA(cudaGetLastError());
  return NEBW_OK;
}

int prof_mark(nebw_model *m, bool on, int kind, cudaStream_t st) {
  if (!on) return NEBW_OK;
  if (m->ev_used == m->ev_pool.size()) {
    cudaEvent_t e;
    NEBW_CUDA(cudaEventCreate(&e));
    m->ev_pool.push_back(e);
  }
  cudaEvent_t e = m->ev_pool[m->ev_used++];
  NEBW_CUDA(cudaEventRecord(e, st));
  m->marks.emplace_back(e, kind);
  return NEBW_OK;
}

// The refusals every encoder entry point makes before touching the device.
int check_pass(const nebw_model *m, int B, int S) {
  if (int rc = model_ready(m)) return rc;
  NEBW_REQUIRE(B > 0 && B <= 65535, "batch %d refused: 1..65535", B);
  NEBW_REQUIRE(S > 0 && S <= m->cfg.max_seq_len, "seq %d refused: 1..max_seq_len (%d)", S,
               m->cfg.max_seq_len);
  return rope_ready(m);
}

// One encoder pass of B sequences padded to S into `out`, on the
// workspace `ws` (which holds at least B * S rows and B sequences).  `prof`:
// bracket each launch with the model's profiling events.
int encode_device_bf16(nebw_model *m, Workspace &ws, bool prof, const int *ids, const int *len_in,
                       int B, int S, float *out, cudaStream_t st) {
  nebw_dev *d = m->dev;
  const nebw_config &c = m->cfg;
  if (B * static_cast<int64_t>(S) > ws.rows_cap || B > ws.batch_cap)
    return set_error(NEBW_EINVAL, "internal: workspace too small for batch %d x seq %d", B, S);
  const int64_t H = c.hidden, F = c.intermediate;
  const int rows = static_cast<int>(static_cast<int64_t>(B) * S);
  const int *T_dev = ws.off + B;
  int rc;
  if ((rc = prof_mark(m, prof, NEBW_K_PACK, st))) return rc;
  if ((rc = launch_pack(len_in, B, S, ws.len, ws.off, d->d_err, st))) return rc;
  const bool tc_attention =
      d->attn_kind == NEBW_ATTN_TCGEN05 && nebw::attn_tc_head_dim(c.head_dim);
  if (tc_attention) {
    // with the work list, zero the Q|K|V and A rows just past the packed
    // rows, up to the workspace's extent (the attention's last partial key
    // group reads V there)
    nebw::attn_work_kernel<<<1 + nebw::kAttnTailBlocks, 1024, 0, st>>>(
        ws.len, B, ws.att_items + 1, ws.att_items, T_dev, ws.rows_cap, ws.qkv,
        static_cast<int>(3 * H), ws.a, static_cast<int>(H));
    NEBW_CUDA(cudaGetLastError());
  }
  if ((rc = prof_mark(m, prof, NEBW_K_EMBED_LN, st))) return rc;
  if ((rc = launch_embed_ln(ids, B, S, ws.off, ws.len, m->word, c.vocab_size, m->pos, m->typ,
                            m->emb_g, m->emb_b, c.layer_norm_eps, c.hidden, ws.x, ws.a, d->d_err,
                            st)))
    return rc;
  const int up_epi = c.activation == NEBW_ACT_GELU_ERF ? nebw::kEpiBf16Erf : nebw::kEpiBf16Gelu8;
  // rotary in the QKV epilogue when the workspace holds the row positions
  const bool rope_fused = c.rope && ws.row_pos != nullptr;
  if (rope_fused) {
    const dim3 pg((S + 255) / 256, B);
    nebw::row_pos_kernel<<<pg, 256, 0, st>>>(ws.off, ws.len, ws.row_pos);
    NEBW_CUDA(cudaGetLastError());
  }
  for (int L = 0; L < c.num_layers; ++L) {
    const LayerW &w = m->layers[L];
    GemmArgs a{};
    a.M = rows;
    a.M_dev = T_dev;
    a.err = d->d_err;
    // QKV
    a.N = static_cast<int>(3 * H);
    a.K = static_cast<int>(H);
    a.bias = w.b_qkv;
    a.resid = nullptr;
    a.out = ws.qkv;
    if ((rc = prof_mark(m, prof, NEBW_K_GEMM_QKV, st))) return rc;
    if (rope_fused) {  // rotary positions applied in the epilogue
      a.row_pos = ws.row_pos;
      a.rope_cos = m->rope_cos;
      a.rope_sin = m->rope_sin;
      a.rope_rows = c.max_seq_len;
      a.rope_cols = static_cast<int>(2 * H);
    }
    if ((rc = launch_gemm(d, w.qkv, ws.map_a, ws.out_qkv,
                          rope_fused ? nebw::kEpiBf16Rope : nebw::kEpiBf16, a, st)))
      return rc;
    a.row_pos = nullptr;
    a.rope_cos = a.rope_sin = nullptr;
    a.rope_rows = a.rope_cols = 0;
    // attention (rotary positions on Q and K first when not fused, timed with it)
    if ((rc = prof_mark(m, prof, NEBW_K_ATTENTION, st))) return rc;
    if (c.rope && !rope_fused && (rc = launch_rope(m, ws, B, S, st))) return rc;
    if (tc_attention)
      rc = launch_attention_tc(d, ws.map_qkv_att, ws.map_kv_att, ws.off, ws.len, ws.att_items + 1,
                               ws.att_items, B, S, c.num_heads, c.head_dim, ws.ctx, st);
    else
      rc = launch_attention(ws.qkv, ws.off, ws.len, B, S, c.num_heads, c.head_dim, ws.ctx, st);
    if (rc)
      return rc;
    // attention-out + bias + residual (fp32, in place)
    a.N = static_cast<int>(H);
    a.K = static_cast<int>(H);
    a.bias = w.b_ao;
    a.resid = nullptr;
    a.out = ws.y;
    if ((rc = prof_mark(m, prof, NEBW_K_GEMM_AO, st))) return rc;
    if ((rc = launch_gemm(d, w.ao, ws.map_ctx, ws.out_y, nebw::kEpiBf16, a, st))) return rc;
    if ((rc = prof_mark(m, prof, NEBW_K_LN, st))) return rc;
    if ((rc = launch_layernorm(ws.x, ws.y, true, w.ln1_g, w.ln1_b, c.layer_norm_eps, rows, H, T_dev,
                               ws.a, st)))
      return rc;
    // FFN up + bias + GELU -> bf16; gated: up | gate (2F wide, plain
    // narrow), then h = up * act(gate) over the first F columns (timed with
    // the GEMM, as the fused activation of the plain FFN is)
    a.N = static_cast<int>(c.gated_ffn ? 2 * F : F);
    a.K = static_cast<int>(H);
    a.bias = w.b_up;
    a.resid = nullptr;
    a.out = ws.h;
    if ((rc = prof_mark(m, prof, NEBW_K_GEMM_UP, st))) return rc;
    const int epi = !c.gated_ffn ? up_epi
                    : m->glu_fused ? (c.gated_act == NEBW_GATE_SILU ? nebw::kEpiBf16SwiGLU
                                                                    : nebw::kEpiBf16GeGLU)
                                   : nebw::kEpiBf16;
    if ((rc = launch_gemm(d, w.up, ws.map_a, ws.out_h, epi, a, st))) return rc;
    if (c.gated_ffn && !m->glu_fused && (rc = launch_glu(m, ws, rows, T_dev, st))) return rc;
    // FFN down + bias + residual (fp32, in place)
    a.N = static_cast<int>(H);
    a.K = static_cast<int>(F);
    a.bias = w.b_dn;
    a.resid = nullptr;
    a.out = ws.y;
    if ((rc = prof_mark(m, prof, NEBW_K_GEMM_DOWN, st))) return rc;
    if ((rc = launch_gemm(d, w.dn, ws.map_h, ws.out_y, nebw::kEpiBf16, a, st))) return rc;
    if ((rc = prof_mark(m, prof, NEBW_K_LN, st))) return rc;
    if ((rc = launch_layernorm(ws.x, ws.y, true, w.ln2_g, w.ln2_b, c.layer_norm_eps, rows, H, T_dev,
                               L + 1 < c.num_layers ? ws.a : nullptr, st)))
      return rc;
  }
  if ((rc = prof_mark(m, prof, NEBW_K_POOL, st))) return rc;
  if ((rc = launch_pool(ws.x, ws.off, ws.len, B, c.hidden, c.pooling, c.l2_normalize, out, st)))
    return rc;
  return prof_mark(m, prof, -1, st);
}

// One pass of the int8 datapath (NEBW_DATAPATH_I8): BertEncoder::run's
// array path for an int8 container (bert_encoder.cpp:1419-1598, gemm()'s
// array branch :763-923, with the fused epilogues), the GEMMs on
// tcgen05.mma kind::i8:
//   x = LN(embeddings); A = quantise(x, 1/asmooth_qkv) (layer 0)
//   per layer:
//     qkv  = dequantise(A . W_qkv), narrowed to bf16 for the attention
//     ctx  = attention(qkv) (the bf16 tensor-core kernel)
//     A    = quantise(ctx, 1/asmooth_ao); y = dequantise(A . W_ao) (fp32)
//     x    = LN1(x + y); A = quantise(x, 1/asmooth_up)    (add_norm_quant)
//     h    = gelu8(dequantise(A . W_up)); A = quantise(h, 1/asmooth_down)
//                                                      (dequant_act_quant)
//     y    = dequantise(A . W_down)
//     x    = LN2(x + y); A = quantise(x, 1/asmooth_qkv of the next layer)
//   pool + L2.
// Every step runs over the packed rows (T on the device); the quantiser, the
// dequantisation and gelu8 are the reference's operations bit for bit (the
// int32 products are exact).  The bf16 narrow of qkv and the bf16 attention
// are this library's, as on the bf16 datapath.
int encode_device_i8(nebw_model *m, Workspace &ws, bool prof, const int *ids, const int *len_in,
                     int B, int S, float *out, cudaStream_t st) {
  nebw_dev *d = m->dev;
  const nebw_config &c = m->cfg;
  if (!ws.aq || B * static_cast<int64_t>(S) > ws.rows_cap || B > ws.batch_cap)
    return set_error(NEBW_EINVAL, "internal: int8 workspace missing or too small for batch %d x "
                     "seq %d", B, S);
  if (static_cast<int>(m->i8.size()) != c.num_layers)
    return set_error(NEBW_ESTATE, "the int8 datapath has no operands");
  const int64_t H = c.hidden, F = c.intermediate;
  const int rows = static_cast<int>(static_cast<int64_t>(B) * S);
  const int *T_dev = ws.off + B;
  int rc;
  if ((rc = prof_mark(m, prof, NEBW_K_PACK, st))) return rc;
  if ((rc = launch_pack(len_in, B, S, ws.len, ws.off, d->d_err, st))) return rc;
  const bool tc_attention =
      d->attn_kind == NEBW_ATTN_TCGEN05 && nebw::attn_tc_head_dim(c.head_dim);
  if (tc_attention) {
    // the work list; and the Q|K|V rows just past the packed rows zeroed
    // (the attention's last partial key group reads V there; the int8 GEMM
    // writes only the packed rows)
    nebw::attn_work_kernel<<<1 + nebw::kAttnTailBlocks, 1024, 0, st>>>(
        ws.len, B, ws.att_items + 1, ws.att_items, T_dev, ws.rows_cap, ws.qkv,
        static_cast<int>(3 * H), ws.a, static_cast<int>(H));
    NEBW_CUDA(cudaGetLastError());
  }
  if ((rc = prof_mark(m, prof, NEBW_K_EMBED_LN, st))) return rc;
  if ((rc = launch_embed_ln(ids, B, S, ws.off, ws.len, m->word, c.vocab_size, m->pos, m->typ,
                            m->emb_g, m->emb_b, c.layer_norm_eps, c.hidden, ws.x, nullptr,
                            d->d_err, st)))
    return rc;
  if ((rc = launch_quantise(ws.x, false, rows, T_dev, H, m->i8[0].qkv.ias, ws.aq, ws.sa, st)))
    return rc;
  for (int L = 0; L < c.num_layers; ++L) {
    const LayerW &w = m->layers[L];
    const LayerI8 &q = m->i8[L];
    nebw::GemmI8Args a{};
    a.M = rows;
    a.M_dev = T_dev;
    a.sa = ws.sa;
    a.err = d->d_err;
    // QKV -> bf16 Q|K|V
    a.N = static_cast<int>(3 * H);
    a.K = static_cast<int>(H);
    a.ws = q.qkv.ws;
    a.bias = w.b_qkv;
    a.out = nullptr;
    a.out_bf16 = ws.qkv;
    if ((rc = prof_mark(m, prof, NEBW_K_GEMM_QKV, st))) return rc;
    if ((rc = launch_gemm_i8(d, q.qkv.w, ws.map_aq_h, ws.out_qkv, a, false, st))) return rc;
    if ((rc = prof_mark(m, prof, NEBW_K_ATTENTION, st))) return rc;
    if (tc_attention)
      rc = launch_attention_tc(d, ws.map_qkv_att, ws.map_kv_att, ws.off, ws.len, ws.att_items + 1,
                               ws.att_items, B, S, c.num_heads, c.head_dim, ws.ctx, st);
    else
      rc = launch_attention(ws.qkv, ws.off, ws.len, B, S, c.num_heads, c.head_dim, ws.ctx, st);
    if (rc) return rc;
    // attention-out: quantise ctx, product, dequantise (fp32)
    if ((rc = prof_mark(m, prof, NEBW_K_GEMM_AO, st))) return rc;
    if ((rc = launch_quantise(ws.ctx, true, rows, T_dev, H, q.ao.ias, ws.aq, ws.sa, st))) return rc;
    a.N = static_cast<int>(H);
    a.K = static_cast<int>(H);
    a.ws = q.ao.ws;
    a.bias = w.b_ao;
    a.out = ws.y32;
    a.out_bf16 = nullptr;
    if ((rc = launch_gemm_i8(d, q.ao.w, ws.map_aq_h, ws.out_y32, a, false, st))) return rc;
    if ((rc = prof_mark(m, prof, NEBW_K_LN, st))) return rc;
    if ((rc = launch_layernorm_quant(ws.x, ws.y32, w.ln1_g, w.ln1_b, c.layer_norm_eps, rows, H,
                                     T_dev, q.up.ias, ws.aq, ws.sa, st)))
      return rc;
    // FFN-up with gelu8, then quantised for FFN-down (dequant_act_quant)
    a.N = static_cast<int>(F);
    a.K = static_cast<int>(H);
    a.ws = q.up.ws;
    a.bias = w.b_up;
    a.out = ws.h32;
    if ((rc = prof_mark(m, prof, NEBW_K_GEMM_UP, st))) return rc;
    if ((rc = launch_gemm_i8(d, q.up.w, ws.map_aq_h, ws.out_h32, a, true, st))) return rc;
    if ((rc = launch_quantise(ws.h32, false, rows, T_dev, F, q.dn.ias, ws.aq, ws.sa, st)))
      return rc;
    // FFN-down (fp32), then add + LayerNorm + the next layer's quantisation
    a.N = static_cast<int>(H);
    a.K = static_cast<int>(F);
    a.ws = q.dn.ws;
    a.bias = w.b_dn;
    a.out = ws.y32;
    if ((rc = prof_mark(m, prof, NEBW_K_GEMM_DOWN, st))) return rc;
    if ((rc = launch_gemm_i8(d, q.dn.w, ws.map_aq_f, ws.out_y32, a, false, st))) return rc;
    if ((rc = prof_mark(m, prof, NEBW_K_LN, st))) return rc;
    const bool last = L + 1 == c.num_layers;
    if ((rc = launch_layernorm_quant(ws.x, ws.y32, w.ln2_g, w.ln2_b, c.layer_norm_eps, rows, H,
                                     T_dev, last ? nullptr : m->i8[L + 1].qkv.ias,
                                     last ? nullptr : ws.aq, last ? nullptr : ws.sa, st)))
      return rc;
  }
  if ((rc = prof_mark(m, prof, NEBW_K_POOL, st))) return rc;
  if ((rc = launch_pool(ws.x, ws.off, ws.len, B, c.hidden, c.pooling, c.l2_normalize, out, st)))
    return rc;
  return prof_mark(m, prof, -1, st);
}

// One encoder pass on the model's datapath.
int encode_device(nebw_model *m, Workspace &ws, bool prof, const int *ids, const int *len_in,
                  int B, int S, float *out, cudaStream_t st) {
  if (m->datapath == NEBW_DATAPATH_I8)
    return encode_device_i8(m, ws, prof, ids, len_in, B, S, out, st);
  return encode_device_bf16(m, ws, prof, ids, len_in, B, S, out, st);
}

}  // namespace

extern "C" int nebw_model_create(nebw_dev *d, const nebw_config *cfg, nebw_model **out) {
  if (int rc = use_dev(d)) return rc;
  NEBW_REQUIRE(cfg && out, "null argument");
  const nebw_config &c = *cfg;
  NEBW_REQUIRE(c.num_layers > 0 && c.hidden > 0 && c.num_heads > 0 && c.max_seq_len > 0 &&
                   c.vocab_size > 0 && c.intermediate > 0 && c.type_vocab_size > 0,
               "the model reports a non-positive shape");
  NEBW_REQUIRE(c.head_dim * c.num_heads == c.hidden, "head_dim * heads != hidden");
  NEBW_REQUIRE(c.head_dim == 32 || c.head_dim == 64, "head_dim %d refused: 32 or 64", c.head_dim);
  NEBW_REQUIRE(c.hidden % 128 == 0 && c.hidden <= 2048, "hidden %d refused: multiple of 128, <= 2048",
               c.hidden);
  NEBW_REQUIRE(c.intermediate % 64 == 0, "intermediate %d refused: multiple of 64", c.intermediate);
  NEBW_REQUIRE(c.pooling == NEBW_POOL_MEAN || c.pooling == NEBW_POOL_CLS, "pooling %d refused",
               c.pooling);
  NEBW_REQUIRE(c.activation == NEBW_ACT_GELU8 || c.activation == NEBW_ACT_GELU_ERF,
               "activation %d refused", c.activation);
  NEBW_REQUIRE(c.gated_ffn == 0 || c.gated_ffn == 1, "gated_ffn %d refused: 0 or 1", c.gated_ffn);
  NEBW_REQUIRE(!c.gated_ffn || c.gated_act == NEBW_GATE_SILU || c.gated_act == NEBW_GATE_GELU_ERF,
               "gated activation %d refused", c.gated_act);
  NEBW_REQUIRE(c.rope == 0 || c.rope == 1, "rope %d refused: 0 or 1", c.rope);
  NEBW_REQUIRE(!c.rope || c.rope_theta >= 0.0, "negative rope_theta refused");
  std::unique_ptr<nebw_model> m(new nebw_model());
  m->dev = d;
  m->cfg = c;
  m->glu_fused = c.gated_ffn && d->gemm_pairs > 0;
  m->layers.resize(c.num_layers);
  if (int rc = build_rope(m.get())) {
    const std::string msg = g_last_error;
    nebw_model_destroy(m.release());
    return set_error(rc, "%s", msg.c_str());
  }
  *out = m.release();
  return NEBW_OK;
}

extern "C" int nebw_model_set_tensor(nebw_model *m, const char *name, const void *host, int dtype,
                                     int64_t rows, int64_t cols) {
  NEBW_REQUIRE(m && name && host, "null argument");
  if (int rc = use_dev(m->dev)) return rc;
  drop_graphs(m);  // a captured pass reads the tensors being replaced
  const nebw_config &c = m->cfg;
  const std::string n(name);
  const int64_t H = c.hidden, F = c.intermediate;
  auto expect = [&](int64_t r, int64_t cc) -> int {
    if (rows != r || cols != cc)
      return set_error(NEBW_EINVAL, "tensor '%s' is [%lld, %lld], expected [%lld, %lld]", name,
                       static_cast<long long>(rows), static_cast<long long>(cols),
                       static_cast<long long>(r), static_cast<long long>(cc));
    return NEBW_OK;
  };
  int rc = NEBW_OK;
  if (n == "embeddings.word") {
    if (!(rc = expect(c.vocab_size, H))) rc = upload_f32(m->dev, &m->word, host, dtype, rows * cols);
  } else if (n == "embeddings.position") {
    NEBW_REQUIRE(cols == H && rows >= c.max_seq_len, "position table '%s' needs >= %d rows of %lld",
                 name, c.max_seq_len, static_cast<long long>(H));
    rc = upload_f32(m->dev, &m->pos, host, dtype, static_cast<int64_t>(c.max_seq_len) * H);
  } else if (n == "embeddings.token_type") {
    NEBW_REQUIRE(cols == H && rows >= 1, "token-type table must be [>=1, hidden]");
    rc = upload_f32(m->dev, &m->typ, host, dtype, H);  // type id 0 only
  } else if (n == "embeddings.ln.weight") {
    if (!(rc = expect(1, H)) || !(rc = expect(H, 1)) || true) {
      NEBW_REQUIRE(rows * cols == H, "'%s' must hold hidden values", name);
      rc = upload_f32(m->dev, &m->emb_g, host, dtype, H);
    }
  } else if (n == "embeddings.ln.bias") {
    NEBW_REQUIRE(rows * cols == H, "'%s' must hold hidden values", name);
    rc = upload_f32(m->dev, &m->emb_b, host, dtype, H);
  } else if (n.rfind("layer.", 0) == 0) {
    const size_t dot = n.find('.', 6);
    NEBW_REQUIRE(dot != std::string::npos, "malformed tensor name '%s'", name);
    const int L = std::atoi(n.substr(6, dot - 6).c_str());
    NEBW_REQUIRE(L >= 0 && L < c.num_layers, "tensor '%s' names a layer outside [0, %d)", name,
                 c.num_layers);
    const std::string leaf = n.substr(dot + 1);
    LayerW &w = m->layers[L];
    auto vec = [&](float **dst, int64_t len) -> int {
      if (rows * cols != len)
        return set_error(NEBW_EINVAL, "tensor '%s' must hold %lld values", name,
                         static_cast<long long>(len));
      return upload_f32(m->dev, dst, host, dtype, len);
    };
    auto gemm_w = [&](Weight *dst, int64_t K, int64_t N) -> int {
      if (int e = expect(K, N)) return e;
      if (dst->ptr) {
        cudaFree(dst->ptr);
        dst->ptr = nullptr;
      }
      return stage_weight(m->dev, host, dtype, K, N, dst);
    };
    if (leaf == "qkv") rc = gemm_w(&w.qkv, H, 3 * H);
    else if (leaf == "qkv.bias") rc = vec(&w.b_qkv, 3 * H);
    else if (leaf == "attn_out") rc = gemm_w(&w.ao, H, H);
    else if (leaf == "attn_out.bias") rc = vec(&w.b_ao, H);
    else if (leaf == "ffn_up" && m->glu_fused) {
      // interleaved [32 up | 32 gate] column groups for the fused GLU epilogue
      if (!(rc = expect(H, 2 * F))) {
        const auto inter =
            glu_interleave(host, H, 2 * F, dtype == NEBW_F32 ? 4 : 2, F, /*by_rows=*/false);
        if (w.up.ptr) {
          cudaFree(w.up.ptr);
          w.up.ptr = nullptr;
        }
        rc = stage_weight(m->dev, inter.data(), dtype, H, 2 * F, &w.up);
      }
    } else if (leaf == "ffn_up.bias" && m->glu_fused) {
      if (rows * cols != 2 * F)
        rc = set_error(NEBW_EINVAL, "tensor '%s' must hold %lld values", name,
                       static_cast<long long>(2 * F));
      else if (dtype != NEBW_F32)
        rc = set_error(NEBW_EINVAL, "this tensor must be F32 (as the container stores it)");
      else {
        const auto inter = glu_interleave(host, 1, 2 * F, 4, F, false);
        rc = upload_f32(m->dev, &w.b_up, inter.data(), dtype, 2 * F);
      }
    } else if (leaf == "ffn_up") rc = gemm_w(&w.up, H, c.gated_ffn ? 2 * F : F);
    else if (leaf == "ffn_up.bias") rc = vec(&w.b_up, c.gated_ffn ? 2 * F : F);
    else if (leaf == "ffn_down") rc = gemm_w(&w.dn, F, H);
    else if (leaf == "ffn_down.bias") rc = vec(&w.b_dn, H);
    else if (leaf == "ln1.weight") rc = vec(&w.ln1_g, H);
    else if (leaf == "ln1.bias") rc = vec(&w.ln1_b, H);
    else if (leaf == "ln2.weight") rc = vec(&w.ln2_g, H);
    else if (leaf == "ln2.bias") rc = vec(&w.ln2_b, H);
    else return set_error(NEBW_EINVAL, "unknown tensor '%s'", name);
  } else {
    return set_error(NEBW_EINVAL, "unknown tensor '%s'", name);
  }
  if (rc == NEBW_OK) m->staged[n] = true;
  return rc;
}

extern "C" int nebw_model_set_gemm_nk(nebw_model *m, const char *name, const uint16_t *host,
                                      int64_t n_rows, int64_t k_cols) {
  NEBW_REQUIRE(m && name && host, "null argument");
  if (int rc = use_dev(m->dev)) return rc;
  drop_graphs(m);  // a captured pass reads the tensors being replaced
  const nebw_config &c = m->cfg;
  const std::string n(name);
  const int64_t H = c.hidden, F = c.intermediate;
  NEBW_REQUIRE(n.rfind("layer.", 0) == 0, "'%s' is not a GEMM operand", name);
  const size_t dot = n.find('.', 6);
  NEBW_REQUIRE(dot != std::string::npos, "malformed tensor name '%s'", name);
  const int L = std::atoi(n.substr(6, dot - 6).c_str());
  NEBW_REQUIRE(L >= 0 && L < c.num_layers, "tensor '%s' names a layer outside [0, %d)", name,
               c.num_layers);
  const std::string leaf = n.substr(dot + 1);
  LayerW &w = m->layers[L];
  Weight *dst = nullptr;
  int64_t K = 0, N = 0;
  if (leaf == "qkv") dst = &w.qkv, K = H, N = 3 * H;
  else if (leaf == "attn_out") dst = &w.ao, K = H, N = H;
  else if (leaf == "ffn_up") dst = &w.up, K = H, N = c.gated_ffn ? 2 * F : F;
  else if (leaf == "ffn_down") dst = &w.dn, K = F, N = H;
  else return set_error(NEBW_EINVAL, "'%s' is not a GEMM operand", name);
  std::vector<unsigned char> inter;
  if (leaf == "ffn_up" && m->glu_fused && n_rows == N && k_cols == K) {
    inter = glu_interleave(host, N, K, 2, F, /*by_rows=*/true);  // [N, K]: reorder rows
    host = reinterpret_cast<const uint16_t *>(inter.data());
  }
  if (n_rows != N || k_cols != K)
    return set_error(NEBW_EINVAL, "GEMM operand '%s' is [%lld, %lld] (N, K), expected [%lld, %lld]",
                     name, static_cast<long long>(n_rows), static_cast<long long>(k_cols),
                     static_cast<long long>(N), static_cast<long long>(K));
  if (dst->ptr) {
    cudaFree(dst->ptr);
    dst->ptr = nullptr;
  }
  if (int rc = stage_weight_nk(m->dev, host, K, N, dst)) return rc;
  m->staged[n] = true;
  return NEBW_OK;
}

extern "C" int nebw_model_destroy(nebw_model *m) {
  if (!m) return NEBW_OK;
  cudaSetDevice(m->dev->device);
  cudaStreamSynchronize(m->dev->stream);
  free_workspace(m);
  for (cudaEvent_t e : m->ev_pool) cudaEventDestroy(e);
  for (float *p : {m->word, m->pos, m->typ, m->emb_g, m->emb_b, m->rope_cos, m->rope_sin})
    cudaFree(p);
  for (auto &w : m->layers) {
    for (Weight *x : {&w.qkv, &w.ao, &w.up, &w.dn}) cudaFree(x->ptr);
    for (float *p : {w.b_qkv, w.b_ao, w.b_up, w.b_dn, w.ln1_g, w.ln1_b, w.ln2_g, w.ln2_b})
      cudaFree(p);
  }
  for (auto &l : m->i8)
    for (OperandI8 *o : {&l.qkv, &l.ao, &l.up, &l.dn}) {
      cudaFree(o->w.ptr);
      cudaFree(o->ws);
      cudaFree(o->ias);
    }
  delete m;
  return NEBW_OK;
}

extern "C" int nebw_model_set_int8_operand(nebw_model *m, const char *name, const int8_t *host_kn,
                                           const float *wscale, const float *asmooth, int64_t K,
                                           int64_t N) {
  NEBW_REQUIRE(m && name && host_kn && wscale && asmooth, "null argument");
  if (int rc = use_dev(m->dev)) return rc;
  drop_graphs(m);  // a captured pass reads the tensors being replaced
  const nebw_config &c = m->cfg;
  int layer = -1;
  char kind[16] = {0};
  char tail = 0;
  NEBW_REQUIRE(std::sscanf(name, "layer.%d.%15[a-z_]%c", &layer, kind, &tail) == 2 && layer >= 0 &&
                   layer < c.num_layers,
               "int8 operand name '%s' refused: layer.{i}.{qkv,attn_out,ffn_up,ffn_down}", name);
  const std::string k = kind;
  const int64_t H = c.hidden, F = c.intermediate;
  int64_t wantK = 0, wantN = 0;
  if (k == "qkv") wantK = H, wantN = 3 * H;
  else if (k == "attn_out") wantK = H, wantN = H;
  else if (k == "ffn_up") wantK = H, wantN = c.gated_ffn ? 2 * F : F;
  else if (k == "ffn_down") wantK = F, wantN = H;
  else return set_error(NEBW_EINVAL, "int8 operand '%s': unknown GEMM '%s'", name, kind);
  NEBW_REQUIRE(K == wantK && N == wantN, "int8 operand '%s' is [%lld, %lld]; the model's is "
               "[%lld, %lld]", name, static_cast<long long>(K), static_cast<long long>(N),
               static_cast<long long>(wantK), static_cast<long long>(wantN));
  std::vector<float> ias(static_cast<size_t>(K));
  for (int64_t j = 0; j < K; ++j) {
    const float a = asmooth[j];
    // the reference divides by it (bert_encoder.cpp:767-772) and would carry
    // inf / NaN into every row; refused by name instead
    NEBW_REQUIRE(a > 0.0f && std::isfinite(a), "%s.asmooth[%lld] = %g: SmoothQuant divisors must "
                 "be positive and finite", name, static_cast<long long>(j), static_cast<double>(a));
    ias[static_cast<size_t>(j)] = 1.0f / a;
  }
  for (int64_t j = 0; j < N; ++j)
    NEBW_REQUIRE(std::isfinite(wscale[j]), "%s.wscale[%lld] is not finite", name,
                 static_cast<long long>(j));
  if (m->i8.empty()) m->i8.resize(static_cast<size_t>(c.num_layers));
  LayerI8 &l = m->i8[static_cast<size_t>(layer)];
  OperandI8 &o = k == "qkv" ? l.qkv : k == "attn_out" ? l.ao : k == "ffn_up" ? l.up : l.dn;
  NEBW_CUDA(cudaDeviceSynchronize());  // a pass may still read the operand being replaced
  cudaFree(o.w.ptr);
  cudaFree(o.ws);
  cudaFree(o.ias);
  o = OperandI8{};
  if (int rc = stage_i8(host_kn, K, N, o.w)) return rc;
  NEBW_CUDA(cudaMalloc(&o.ws, N * 4));
  NEBW_CUDA(cudaMalloc(&o.ias, K * 4));
  NEBW_CUDA(cudaMemcpy(o.ws, wscale, N * 4, cudaMemcpyHostToDevice));
  NEBW_CUDA(cudaMemcpy(o.ias, ias.data(), K * 4, cudaMemcpyHostToDevice));
  return NEBW_OK;
}

extern "C" int nebw_model_set_datapath(nebw_model *m, int32_t datapath) {
  NEBW_REQUIRE(m, "null model");
  NEBW_REQUIRE(datapath == NEBW_DATAPATH_BF16 || datapath == NEBW_DATAPATH_I8,
               "datapath %d refused: NEBW_DATAPATH_BF16 or NEBW_DATAPATH_I8", datapath);
  if (datapath == NEBW_DATAPATH_I8) {
    const nebw_config &c = m->cfg;
    NEBW_REQUIRE(!c.gated_ffn && !c.rope && c.activation == NEBW_ACT_GELU8,
                 "the int8 datapath runs the plain BERT encoder (gelu8 FFN, absolute positions): "
                 "this model is gated, rotary or uses another activation");
    for (int L = 0; L < c.num_layers; ++L) {
      const bool have = !m->i8.empty() && m->i8[L].qkv.w.ptr && m->i8[L].ao.w.ptr &&
                        m->i8[L].up.w.ptr && m->i8[L].dn.w.ptr;
      NEBW_REQUIRE(have, "the int8 datapath needs the four int8 operands of every layer; layer "
                   "%d lacks one (nebw_model_set_int8_operand, or an int8 container)", L);
    }
  }
  if (datapath != m->datapath) drop_graphs(m);
  m->datapath = datapath;
  return NEBW_OK;
}

extern "C" int nebw_model_set_graphs(nebw_model *m, int32_t on) {
  NEBW_REQUIRE(m, "null model");
  if (int rc = use_dev(m->dev)) return rc;
  if (!on) drop_graphs(m);
  m->use_graphs = on != 0;
  return NEBW_OK;
}

extern "C" int nebw_model_set_rope_freq(nebw_model *m, const double *inv_freq, int32_t n) {
  NEBW_REQUIRE(m && inv_freq, "null argument");
  if (int rc = use_dev(m->dev)) return rc;
  drop_graphs(m);  // a captured pass reads the tensors being replaced
  NEBW_REQUIRE(m->cfg.rope, "the model is not rotary (config.rope is 0)");
  NEBW_REQUIRE(n == m->cfg.head_dim / 2, "%d rotary frequencies given, head_dim / 2 = %d expected",
               n, m->cfg.head_dim / 2);
  for (int32_t j = 0; j < n; ++j)
    NEBW_REQUIRE(std::isfinite(inv_freq[j]) && inv_freq[j] >= 0.0,
                 "rotary frequency %d is %g", j, inv_freq[j]);
  NEBW_CUDA(cudaStreamSynchronize(m->dev->stream));
  m->rope_freq.assign(inv_freq, inv_freq + n);
  cudaFree(m->rope_cos);
  cudaFree(m->rope_sin);
  m->rope_cos = m->rope_sin = nullptr;
  return build_rope(m);
}

extern "C" int nebw_model_get_config(const nebw_model *m, nebw_config *cfg) {
  NEBW_REQUIRE(m && cfg, "null argument");
  *cfg = m->cfg;
  return NEBW_OK;
}

namespace {
// The layout this library reads a tma_bf16 container's GEMM operands in:
// sha256 of the canonical descriptor {"dtype":"BF16","kind":"dense",
// "order":"n,k"} (dense row-major [N, K] bf16; TMA applies the swizzle as it
// loads).  The packer writes the same hash beside each operand.
constexpr char kTmaLayoutHash[] =
    "11a82b85f370c9a7fa302e55afdde7415734be70c40e25d543c57a860f15ae3a";
}  // namespace

extern "C" const char *nebw_tma_layout_hash(void) { return kTmaLayoutHash; }

extern "C" int nebw_pack_checkpoint(const char *model_dir, const char *out_path,
                                    const char *layout, int32_t max_seq, int32_t fold_scale,
                                    uint64_t *bytes) {
  NEBW_REQUIRE(model_dir && out_path, "null path");
  nebw::PackOptions opt;
  if (layout) opt.layout = layout;
  if (max_seq > 0) opt.max_seq = max_seq;
  opt.fold_scale = fold_scale != 0;
  try {
    const uint64_t n = nebw::pack_checkpoint(model_dir, out_path, opt);
    if (bytes) *bytes = n;
  } catch (const std::exception &e) {
    return set_error(NEBW_EIO, "pack %s: %s", model_dir, e.what());
  }
  return NEBW_OK;
}

namespace {
// A block_panel GEMM operand -- the reference's pre-tiled array layout, BF16
// or I8 -- back to fp32 row-major [K, N], I8 dequantised per column by the
// operand's `.wscale`, as the reference's host_b_kn (runtime/include/common/
// host_b.hpp:74-224) reads it.  The flat panel runs over the axes (kb, nb,
// ri, ci, si, ti), ti fastest, with k = kb*tile_k + ri*mac_s + si and
// n = nb*tile_n + ci*mac_t + ti.  For an I8 panel, `raw` (when given) gets
// the int8 values themselves, [K, N] row-major.
int panel_to_kn(const nebw::NpueFile &f, const std::string &name, std::vector<float> &out,
                std::vector<int8_t> *raw = nullptr) {
  const nebw::NpueTensor &t = f.tensor(name);
  NEBW_REQUIRE(t.shape.size() == 2, "'%s' is not a 2-D GEMM operand", name.c_str());
  const int64_t K = t.shape[0], N = t.shape[1];
  NEBW_REQUIRE(t.padded_shape.empty() ||
                   (t.padded_shape.size() == 2 && t.padded_shape[0] == K && t.padded_shape[1] == N),
               "'%s': logical and padded shapes differ; repack it", name.c_str());
  NEBW_REQUIRE(t.layout_kind == "block_panel" && t.layout_order == "k,n,kt,nt" &&
                   t.layout_inner == "s,t",
               "'%s': layout '%s' (order '%s', inner '%s') refused: block_panel k,n,kt,nt / s,t is "
               "the pre-tiled layout this library reads", name.c_str(), t.layout_kind.c_str(),
               t.layout_order.c_str(), t.layout_inner.c_str());
  const int64_t tk = t.tile_k, tn = t.tile_n, s = t.mac_s, tt = t.mac_t;
  NEBW_REQUIRE(tk > 0 && tn > 0 && s > 0 && tt > 0 && K % tk == 0 && N % tn == 0 && tk % s == 0 &&
                   tn % tt == 0,
               "'%s': [%lld, %lld] does not tile into (%lld, %lld) with mac (%lld, %lld)",
               name.c_str(), static_cast<long long>(K), static_cast<long long>(N),
               static_cast<long long>(tk), static_cast<long long>(tn), static_cast<long long>(s),
               static_cast<long long>(tt));
  const bool i8 = t.dtype == "I8";
  NEBW_REQUIRE((i8 || t.dtype == "BF16") && t.layout_dtype == t.dtype,
               "'%s': a %s panel described as %s; BF16 or I8 panels are read", name.c_str(),
               t.dtype.c_str(), t.layout_dtype.c_str());
  NEBW_REQUIRE(t.nbytes == static_cast<uint64_t>(K * N * (i8 ? 1 : 2)),
               "'%s': %llu bytes for a [%lld, %lld] %s panel", name.c_str(),
               static_cast<unsigned long long>(t.nbytes), static_cast<long long>(K),
               static_cast<long long>(N), t.dtype.c_str());
  std::vector<float> ws;
  if (i8) {
    const std::string wn = name + ".wscale";
    NEBW_REQUIRE(f.has(wn), "int8 operand '%s' has no %s", name.c_str(), wn.c_str());
    const nebw::NpueTensor &w = f.tensor(wn);
    NEBW_REQUIRE(w.dtype == "F32" && w.nbytes == static_cast<uint64_t>(N) * 4,
                 "%s must be F32 [%lld]", wn.c_str(), static_cast<long long>(N));
    ws.resize(static_cast<size_t>(N));
    std::memcpy(ws.data(), w.data, static_cast<size_t>(N) * 4);
  }
  out.assign(static_cast<size_t>(K * N), 0.0f);
  if (raw) raw->assign(i8 ? static_cast<size_t>(K * N) : 0, 0);
  const int64_t R0 = tk / s, C0 = tn / tt;
  int64_t idx = 0;
  for (int64_t kb = 0; kb < K / tk; ++kb)
    for (int64_t nb = 0; nb < N / tn; ++nb)
      for (int64_t ri = 0; ri < R0; ++ri)
        for (int64_t ci = 0; ci < C0; ++ci)
          for (int64_t si = 0; si < s; ++si) {
            const int64_t at = (kb * tk + ri * s + si) * N + nb * tn + ci * tt;
            float *row = out.data() + at;
            for (int64_t ti = 0; ti < tt; ++ti, ++idx) {
              if (i8) {
                const int8_t q = reinterpret_cast<const int8_t *>(t.data)[idx];
                if (raw) (*raw)[static_cast<size_t>(at + ti)] = q;
                row[ti] = static_cast<float>(q) * ws[static_cast<size_t>(nb * tn + ci * tt + ti)];
              } else {
                uint16_t h;
                std::memcpy(&h, t.data + 2 * idx, 2);
                const uint32_t bits = static_cast<uint32_t>(h) << 16;
                std::memcpy(&row[ti], &bits, 4);
              }
            }
          }
  return NEBW_OK;
}
}  // namespace

extern "C" int nebw_npue_gemm_kn(const char *path, const char *name, float *out, int64_t K,
                                 int64_t N) {
  NEBW_REQUIRE(path && name && out, "null argument");
  try {
    nebw::NpueFile f(path);
    const nebw::NpueTensor &t = f.tensor(name);
    NEBW_REQUIRE(t.shape.size() == 2 && t.shape[0] == K && t.shape[1] == N,
                 "'%s' is not [%lld, %lld]", name, static_cast<long long>(K),
                 static_cast<long long>(N));
    std::vector<float> kn;
    if (int rc = panel_to_kn(f, name, kn)) return rc;
    std::memcpy(out, kn.data(), kn.size() * 4);
    return NEBW_OK;
  } catch (const std::exception &e) {
    return set_error(NEBW_EIO, "%s", e.what());
  }
}

// The container is read and checked before the device is touched (the model
// is created last), so a refused container is refused on any host.
extern "C" int nebw_model_load_npue(nebw_dev *d, const char *path, nebw_model **out) {
  NEBW_REQUIRE(path && out, "null argument");
  *out = nullptr;
  try {
    nebw::NpueFile f(path);
    const std::string arch = f.config_string("arch");
    if (arch != "bert_abs_gelu_postln" && arch != "nomic_bert_rope_swiglu" &&
        arch != "gte_new_rope_geglu")
      return set_error(NEBW_EINVAL,
                       "container architecture '%s' has no encoder in this library; "
                       "bert_abs_gelu_postln, nomic_bert_rope_swiglu and gte_new_rope_geglu "
                       "are implemented", arch.c_str());
    std::string layout = "pretiled_bf16";
    if (f.has_config("gemm_layout")) layout = f.config_string("gemm_layout");
    if (layout != "host" && layout != "tma_bf16" && layout != "pretiled_bf16")
      return set_error(NEBW_EINVAL,
                       "container gemm_layout '%s' refused: this library reads \"host\" (F32 "
                       "[K, N]), \"tma_bf16\" (bf16 [N, K], nebw.pack) and the reference's "
                       "pre-tiled block panels (\"pretiled_bf16\", a_dtype bf16 or i8)",
                       layout.c_str());
    const bool nk_layout = layout == "tma_bf16";
    const bool panels = layout == "pretiled_bf16";
    // a pre-tiled container's operand type: bf16 panels, or int8 panels with
    // per-column .wscale and the activation's SmoothQuant divisor .asmooth
    std::string a_dtype = "bf16";
    if (panels && f.has_config("a_dtype")) a_dtype = f.config_string("a_dtype");
    for (char &ch : a_dtype) ch = static_cast<char>(std::tolower(static_cast<unsigned char>(ch)));
    // (the BERT packer writes "bf16" / "i8", the ViT packer "BF16" / "I8")
    if (panels && a_dtype != "bf16" && a_dtype != "i8")
      return set_error(NEBW_EINVAL, "pre-tiled container with a_dtype '%s' refused: bf16 or i8 "
                       "(int4 panels are not read)", a_dtype.c_str());
    nebw_config c{};
    c.num_layers = static_cast<int32_t>(f.config_int("num_layers"));
    c.hidden = static_cast<int32_t>(f.config_int("hidden"));
    c.num_heads = static_cast<int32_t>(f.config_int("num_heads"));
    c.head_dim = static_cast<int32_t>(f.config_int("head_dim"));
    c.intermediate = static_cast<int32_t>(f.config_int("intermediate"));
    c.max_seq_len = static_cast<int32_t>(f.config_int("max_seq_len"));
    const auto &word = f.tensor("embeddings.word");
    c.vocab_size = static_cast<int32_t>(word.shape.at(0));
    c.type_vocab_size = static_cast<int32_t>(f.tensor("embeddings.token_type").shape.at(0));
    const std::string pool = f.config_string("pooling");
    if (pool == "cls") c.pooling = NEBW_POOL_CLS;
    else if (pool == "mean") c.pooling = NEBW_POOL_MEAN;
    else return set_error(NEBW_EINVAL, "unknown pooling mode '%s' in the container", pool.c_str());
    c.l2_normalize = f.has_config("l2_normalize") ? f.config_string("l2_normalize") == "true" : 1;
    c.activation = NEBW_ACT_GELU8;  // what the reference's BERT host path runs (gelu_cpu)
    c.layer_norm_eps = 1e-12f;      // hard-coded by layer_norm_cpu (bert_encoder.cpp:438)
    // The rotary / gated families, with set_model_shape's refusals
    // (app_state.hpp:440-560): position encoding and gating asserted, the
    // order of the fused FFN-up halves and the gate's activation read.
    std::vector<double> inv_freq;
    if (arch != "bert_abs_gelu_postln") {
      const std::string pet = f.config_string("position_embedding_type");
      if (pet != "rope")
        return set_error(NEBW_EINVAL, "container arch is %s but position_embedding_type is '%s', "
                         "expected 'rope'", arch.c_str(), pet.c_str());
      if (!f.has_config("gated_ffn") || f.config_string("gated_ffn") != "true")
        return set_error(NEBW_EINVAL, "container arch is %s but gated_ffn is not true: refusing a "
                         "plain FFN over a fused up|gate weight", arch.c_str());
      c.gated_ffn = 1;
      c.rope = 1;
      if (arch == "nomic_bert_rope_swiglu") {
        const std::string halves = f.config_string("swiglu_halves");
        if (halves != "fc11_up|fc12_gate")
          return set_error(NEBW_EINVAL, "unrecognised swiglu_halves ordering '%s' (expected "
                           "'fc11_up|fc12_gate')", halves.c_str());
        c.rope_theta = f.config_double("rope_theta");
        if (!(c.rope_theta > 0.0))
          return set_error(NEBW_EINVAL, "nomic_bert_rope_swiglu container has a non-positive "
                           "rope_theta");
      } else {
        const std::string halves = f.config_string("glu_halves");
        if (halves.rfind("up_first|gate_second", 0) != 0)
          return set_error(NEBW_EINVAL, "unrecognised glu_halves ordering '%s' (expected it to "
                           "begin 'up_first|gate_second')", halves.c_str());
        if (!f.has_config("rope_inv_freq"))
          return set_error(NEBW_EINVAL, "gte_new_rope_geglu container carries no rope_inv_freq "
                           "(the frequency set is data, not derivable from rope_theta)");
        // a JSON array of numbers held as a string, as the packer writes it
        const std::string raw = f.config_string("rope_inv_freq");
        const char *q = raw.c_str();
        while (*q && *q != '[') ++q;
        if (*q == '[') ++q;
        while (*q) {
          while (*q == ' ' || *q == ',' || *q == '\n' || *q == '\t') ++q;
          if (*q == ']' || !*q) break;
          char *end = nullptr;
          const double v = std::strtod(q, &end);
          if (end == q)
            return set_error(NEBW_EINVAL, "rope_inv_freq is not a JSON array of numbers");
          inv_freq.push_back(static_cast<double>(static_cast<float>(v)));  // held as float
          q = end;
        }
        if (static_cast<int>(inv_freq.size()) != c.head_dim / 2)
          return set_error(NEBW_EINVAL, "rope_inv_freq holds %zu values, head_dim / 2 = %d "
                           "expected", inv_freq.size(), c.head_dim / 2);
      }
      // the gate's activation is data: "silu" or "gelu" (exact erf); absent
      // means silu on a nomic container and is refused on a gte one
      std::string act = "silu";
      if (f.has_config("activation")) act = f.config_string("activation");
      else if (arch == "gte_new_rope_geglu")
        return set_error(NEBW_EINVAL, "gte_new_rope_geglu container carries no 'activation' key");
      if (act == "silu") c.gated_act = NEBW_GATE_SILU;
      else if (act == "gelu") c.gated_act = NEBW_GATE_GELU_ERF;
      else
        return set_error(NEBW_EINVAL, "unknown gated-FFN activation '%s' (silu or gelu)",
                         act.c_str());
    }
    std::vector<std::string> names = required_names(c);
    // a tma_bf16 operand laid out for another reader is refused by its
    // layout hash, as the reference's runtime refuses a design whose
    // b_layout_hash differs from the model's (runtime/src/runtime.cpp:190-222)
    if (nk_layout)
      for (const auto &n : names) {
        const auto &t = f.tensor(n);
        if (!(t.shape.size() == 2 && n.rfind("layer.", 0) == 0)) continue;
        if (t.layout_hash != kTmaLayoutHash)
          return set_error(NEBW_EINVAL,
                           "tma_bf16 container: GEMM operand '%s' has layout_hash %s; this "
                           "library reads %.16s... (dense [N, K] BF16): repack it with nebw.pack",
                           n.c_str(),
                           t.layout_hash.empty() ? "(none)"
                                                 : ("'" + t.layout_hash.substr(0, 16) + "...'").c_str(),
                           kTmaLayoutHash);
      }
    nebw_model *m = nullptr;
    if (int rc = nebw_model_create(d, &c, &m)) return rc;
    if (!inv_freq.empty()) {
      if (int rc = nebw_model_set_rope_freq(m, inv_freq.data(),
                                            static_cast<int32_t>(inv_freq.size()))) {
        const std::string msg = g_last_error;
        nebw_model_destroy(m);
        return set_error(rc, "%s", msg.c_str());
      }
    }
    // a rotary container's zero position placeholder is staged as the
    // reference's embedding adds it (absent, a zero table is used)
    if (c.rope && f.has("embeddings.position")) names.push_back("embeddings.position");
    for (const auto &n : names) {
      const auto &t = f.tensor(n);
      const bool gemm_operand = t.shape.size() == 2 && n.rfind("layer.", 0) == 0;
      if (t.dtype != "F32" && t.dtype != "BF16" && !(panels && gemm_operand && t.dtype == "I8")) {
        nebw_model_destroy(m);
        return set_error(NEBW_EINVAL, "tensor '%s' has dtype %s; F32 or BF16 expected",
                         n.c_str(), t.dtype.c_str());
      }
      const int64_t r = t.shape.size() >= 1 ? t.shape[0] : 1;
      const int64_t cc = t.shape.size() >= 2 ? t.shape[1] : 1;
      const int dt = t.dtype == "F32" ? NEBW_F32 : NEBW_BF16;
      int rc;
      if (panels && gemm_operand) {
        // untiled on the host and staged as F32 [K, N]; for int8 the
        // dequantised weights take the activation's divisor as well:
        // (a / asmooth) . W == a . (W / asmooth[k]), the reference's host
        // product (host_gemm, bert_encoder.cpp:714-739) moved onto W
        std::vector<float> kn;
        std::vector<int8_t> q8;
        rc = panel_to_kn(f, n, kn, a_dtype == "i8" ? &q8 : nullptr);
        if (!rc && a_dtype == "i8") {
          const std::string an = n + ".asmooth";
          if (!f.has(an) || f.tensor(an).dtype != "F32" ||
              f.tensor(an).nbytes != static_cast<uint64_t>(r) * 4) {
            nebw_model_destroy(m);
            return set_error(NEBW_EINVAL, "int8 operand '%s' has no F32 [%lld] %s", n.c_str(),
                             static_cast<long long>(r), an.c_str());
          }
          std::vector<float> as(static_cast<size_t>(r));
          std::memcpy(as.data(), f.tensor(an).data, as.size() * 4);
          for (int64_t k = 0; k < r; ++k) {
            const float a = as[static_cast<size_t>(k)];
            if (!(a > 0.0f) || !std::isfinite(a)) {
              // the reference would divide by it and carry inf / NaN into
              // every row; refused by name instead
              nebw_model_destroy(m);
              return set_error(NEBW_EINVAL, "%s[%lld] = %g: SmoothQuant divisors must be "
                               "positive and finite", an.c_str(), static_cast<long long>(k),
                               static_cast<double>(a));
            }
            for (int64_t j = 0; j < cc; ++j) kn[static_cast<size_t>(k * cc + j)] /= a;
          }
          // and the int8 operand itself, for the int8 datapath
          rc = nebw_model_set_int8_operand(
              m, n.c_str(), q8.data(), reinterpret_cast<const float *>(f.tensor(n + ".wscale").data),
              as.data(), r, cc);
        }
        if (!rc) rc = nebw_model_set_tensor(m, n.c_str(), kn.data(), NEBW_F32, r, cc);
      } else if (nk_layout && gemm_operand) {
        if (t.dtype != "BF16") {
          nebw_model_destroy(m);
          return set_error(NEBW_EINVAL, "tma_bf16 container: GEMM operand '%s' is %s, BF16 "
                           "expected", n.c_str(), t.dtype.c_str());
        }
        rc = nebw_model_set_gemm_nk(m, n.c_str(), reinterpret_cast<const uint16_t *>(t.data), r, cc);
      } else {
        rc = nebw_model_set_tensor(m, n.c_str(), t.data, dt, r, cc);
      }
      if (rc) {
        const std::string msg = g_last_error;
        nebw_model_destroy(m);
        return set_error(rc, "%s", msg.c_str());
      }
    }
    *out = m;
    return NEBW_OK;
  } catch (const std::exception &e) {
    return set_error(NEBW_EIO, "%s", e.what());
  }
}

namespace {
// The graph of one pass of B x S on the model's workspace, from device ids /
// lens to device out: found in the model's cache (keyed by the shape, the
// datapath, the attention kernel and the three buffers), or captured from
// encode_device on the device's capture stream and instantiated (the oldest
// of kMaxPassGraphs is dropped to make room).  The caller launches it on its
// own stream.  The packed row count and the attention work list are computed
// on the device inside the pass, so one graph serves every length pattern of
// that shape.
int pass_graph(nebw_model *m, int B, int S, const int *ids, const int *lens, float *out,
               cudaGraphExec_t *exec_out) {
  const int attn = m->dev->attn_kind;
  for (const auto &g : m->graphs)
    if (g.B == B && g.S == S && g.datapath == m->datapath && g.attn == attn && g.ids == ids &&
        g.lens == lens && g.out == out) {
      *exec_out = g.exec;
      return NEBW_OK;
    }
  if (m->graphs.size() >= kMaxPassGraphs) {
    NEBW_CUDA(cudaDeviceSynchronize());  // the oldest may still run, on any stream
    cudaGraphExecDestroy(m->graphs.front().exec);
    m->graphs.erase(m->graphs.begin());
  }
  nebw_dev *d = m->dev;
  if (!d->cap_stream) NEBW_CUDA(cudaStreamCreateWithFlags(&d->cap_stream, cudaStreamNonBlocking));
  cudaStream_t cs = d->cap_stream;
  cudaGraph_t graph = nullptr;
  NEBW_CUDA(cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal));
  const int rc = encode_device(m, m->ws, false, ids, lens, B, S, out, cs);
  const std::string why = rc ? g_last_error : std::string();
  const cudaError_t e = cudaStreamEndCapture(cs, &graph);
  if (rc || e != cudaSuccess) {
    if (graph) cudaGraphDestroy(graph);
    cudaGetLastError();
    if (rc) return set_error(rc, "%s", why.c_str());
    return set_error(NEBW_ECUDA, "capturing the pass as a CUDA graph failed: %s",
                     cudaGetErrorString(e));
  }
  cudaGraphExec_t exec = nullptr;
  const cudaError_t ei = cudaGraphInstantiate(&exec, graph, 0);
  cudaGraphDestroy(graph);
  if (ei != cudaSuccess) {
    cudaGetLastError();
    return set_error(NEBW_ECUDA, "instantiating the pass graph failed: %s", cudaGetErrorString(ei));
  }
  m->graphs.push_back({B, S, m->datapath, attn, ids, lens, out, exec});
  *exec_out = exec;
  return NEBW_OK;
}
}  // namespace

// One pass on the model's own workspace: replayed from the graph cache when
// the model has graphs on (and is not profiling), else launched directly.
int run_pass(nebw_model *m, const int *ids, const int *lens, int B, int S, float *out,
             cudaStream_t st) {
  if (m->use_graphs && !m->prof) {
    cudaGraphExec_t exec = nullptr;
    if (int rc = pass_graph(m, B, S, ids, lens, out, &exec)) return rc;
    NEBW_CUDA(cudaGraphLaunch(exec, st));
    return NEBW_OK;
  }
  return encode_device(m, m->ws, m->prof, ids, lens, B, S, out, st);
}

extern "C" int nebw_encode_device(nebw_model *m, const int32_t *ids, const int32_t *lens, int32_t B,
                                  int32_t S, float *out, void *stream) {
  NEBW_REQUIRE(m && ids && lens && out, "null argument");
  if (int rc = use_dev(m->dev)) return rc;
  if (int rc = check_pass(m, B, S)) return rc;
  if (int rc = ensure_workspace(m, B, S)) return rc;
  return run_pass(m, ids, lens, B, S, out, pick_stream(m->dev, stream));
}

extern "C" int nebw_encode(nebw_model *m, const int32_t *ids, const int32_t *lens, int32_t B,
                           int32_t S, float *out) {
  NEBW_REQUIRE(m && ids && lens && out, "null argument");
  if (int rc = use_dev(m->dev)) return rc;
  NEBW_REQUIRE(B > 0 && S > 0, "empty batch refused");
  if (int rc = check_pass(m, B, S)) return rc;
  if (int rc = ensure_workspace(m, B, S)) return rc;
  nebw_dev *d = m->dev;
  cudaStream_t st = d->stream;
  NEBW_CUDA(cudaMemcpyAsync(m->ids, ids, static_cast<size_t>(B) * S * 4, cudaMemcpyHostToDevice, st));
  NEBW_CUDA(cudaMemcpyAsync(m->len_in, lens, static_cast<size_t>(B) * 4, cudaMemcpyHostToDevice, st));
  if (int rc = run_pass(m, m->ids, m->len_in, B, S, m->out, st)) return rc;
  NEBW_CUDA(cudaMemcpyAsync(out, m->out, static_cast<size_t>(B) * m->cfg.hidden * 4,
                            cudaMemcpyDeviceToHost, st));
  return nebw_sync(d);
}

extern "C" int nebw_encode_launch_count(const nebw_model *m, int32_t seq) {
  if (!m) return set_error(NEBW_EINVAL, "null model"), -1;
  const int S = seq > 0 ? seq : m->cfg.max_seq_len;
  const bool tc =
      m->dev->attn_kind == NEBW_ATTN_TCGEN05 && nebw::attn_tc_head_dim(m->cfg.head_dim);
  const bool rope_fused = rope_in_epilogue(m);
  if (m->datapath == NEBW_DATAPATH_I8)  // pack, work list, embed, quantise, 9 per layer, pool
    return 4 + (tc ? 1 : 0) + m->cfg.num_layers * (8 + attention_launches(tc ? 64 : 0, S));
  const int per_layer = 6 + attention_launches(tc ? 64 : 0, S) +
                        (m->cfg.rope && !rope_fused ? 1 : 0) +
                        (m->cfg.gated_ffn && !m->glu_fused ? 1 : 0);
  return 3 + (tc ? 1 : 0) + (rope_fused ? 1 : 0) + m->cfg.num_layers * per_layer;
}

extern "C" int nebw_model_profile(nebw_model *m, int enable) {
  NEBW_REQUIRE(m != nullptr, "null model");
  m->prof = enable != 0;
  return NEBW_OK;
}

extern "C" int nebw_model_profile_collect(nebw_model *m, int64_t launches[NEBW_K_COUNT],
                                          double ms[NEBW_K_COUNT]) {
  NEBW_REQUIRE(m && launches && ms, "null argument");
  if (int rc = use_dev(m->dev)) return rc;
  for (int k = 0; k < NEBW_K_COUNT; ++k) {
    launches[k] = 0;
    ms[k] = 0.0;
  }
  for (size_t i = 0; i + 1 < m->marks.size(); ++i) {
    const int kind = m->marks[i].second;
    if (kind < 0) continue;  // end of one pass -> start of the next
    NEBW_CUDA(cudaEventSynchronize(m->marks[i + 1].first));
    float t = 0.f;
    NEBW_CUDA(cudaEventElapsedTime(&t, m->marks[i].first, m->marks[i + 1].first));
    launches[kind] += 1;
    ms[kind] += t;
  }
  m->marks.clear();
  m->ev_used = 0;
  return NEBW_OK;
}

// ---------------------------------------------------------------------------
// The encoder pass without any allocation at call time.
//
// For callers that cannot allocate device memory when a request arrives --
// a serving process that sizes and claims all of its GPU memory at start-up
// and must then run within that budget, or a host program that shares the
// GPU under a fixed partition and may not grow it -- nebw_encode_device
// is unsuitable as-is, because the model grows its activation workspace with
// cudaMalloc the first time it sees a larger batch.  This variant keeps every
// intermediate of the pass (residual stream, sublayer output, bf16 operands,
// Q|K|V, attention context, FFN activations, packed lengths and offsets) in
// one file-scope __device__ array of kStaticScratchBytes, which each GPU that
// loads this library holds from module load until the process exits.
//
// The array's name in host code is only a host-side stand-in, never a
// device address, so the kernels are handed the address cudaGetSymbolAddress
// returns for it: looked up once per device, on that device's first call of
// nebw_encode_device_static, with the device current.  That first call
// therefore does the set-up and should come before any stream capture.
//
// Every call shares the one array, which keeps the last call's contents.
// The caller clears nothing: every element the pass reads for a real token is
// written earlier in the same pass, and the rows just past the packed ones
// that a kernel reads (the last partial key group of the tcgen05 attention,
// the CTA-pair GEMM's last 256-row tile) are zeroed at the start of each
// pass.  Calls whose work overlaps on the GPU (different streams, or
// different models on one device) race on the array and must be serialised
// by the caller.  Static calls record no per-kernel profiling events.
// ---------------------------------------------------------------------------

namespace {

constexpr size_t kStaticScratchBytes = 64ull << 20;  // 64 MiB per GPU
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

constexpr int kMaxStaticDevices = 64;
std::mutex g_static_mu;
void *g_static_ptr[kMaxStaticDevices] = {};

int static_scratch_address(int device, void **out) {
  NEBW_REQUIRE(device >= 0 && device < kMaxStaticDevices, "device %d out of range", device);
  std::lock_guard<std::mutex> lk(g_static_mu);
  if (!g_static_ptr[device]) {
    void *p = nullptr;
    NEBW_CUDA(cudaGetSymbolAddress(&p, g_static_scratch));  // the caller made `device` current
    g_static_ptr[device] = p;
  }
  *out = g_static_ptr[device];
  return NEBW_OK;
}

size_t align256(size_t n) { return (n + 255) & ~static_cast<size_t>(255); }

// Bytes of static scratch one pass over `rows` padded rows of `batch`
// sequences needs, in the carve order of static_workspace: per padded row
// 16 * hidden + 2 * (FFN-up output width) bytes, plus 4 for the row
// positions of a rotary model whose QKV epilogue rotates, plus the lengths,
// offsets and attention work list, each buffer rounded up to 256 bytes.
size_t static_scratch_need(const nebw_model *m, int64_t rows, int64_t batch) {
  const size_t R = static_cast<size_t>(rows), H = m->cfg.hidden,
               FW = static_cast<size_t>(ffn_up_width(m)), Bs = static_cast<size_t>(batch);
  return align256(R * H * 4) + align256(R * H * 2) + align256(R * H * 2) +
         align256(R * 3 * H * 2) + align256(R * H * 2) + align256(R * FW * 2) +
         align256(Bs * 4) + align256((Bs + 1) * 4) + align256((R / 128 + Bs + 1) * 4) +
         (rope_in_epilogue(m) ? align256(R * 4) : 0);
}

// A workspace for `rows` padded rows of `batch` sequences carved out of the
// static scratch at `base` (static_scratch_need bytes).  It holds what the
// model's own workspace holds, so both entry points launch the same kernels.
int static_workspace(const nebw_model *m, void *base, int64_t rows, int64_t batch, Workspace *w) {
  const size_t H = m->cfg.hidden, R = static_cast<size_t>(rows), Bs = static_cast<size_t>(batch),
               FW = static_cast<size_t>(ffn_up_width(m));
  unsigned char *p = static_cast<unsigned char *>(base);
  auto carve = [&p](size_t bytes) {
    unsigned char *q = p;
    p += align256(bytes);
    return q;
  };
  w->x = reinterpret_cast<float *>(carve(R * H * 4));
  w->y = reinterpret_cast<__nv_bfloat16 *>(carve(R * H * 2));
  w->a = reinterpret_cast<__nv_bfloat16 *>(carve(R * H * 2));
  w->qkv = reinterpret_cast<__nv_bfloat16 *>(carve(R * 3 * H * 2));
  w->ctx = reinterpret_cast<__nv_bfloat16 *>(carve(R * H * 2));
  w->h = reinterpret_cast<__nv_bfloat16 *>(carve(R * FW * 2));
  w->len = reinterpret_cast<int *>(carve(Bs * 4));
  w->off = reinterpret_cast<int *>(carve((Bs + 1) * 4));
  w->att_items = reinterpret_cast<int *>(carve((R / 128 + Bs + 1) * 4));
  w->row_pos = rope_in_epilogue(m) ? reinterpret_cast<int *>(carve(R * 4)) : nullptr;
  w->rows_cap = rows;
  w->batch_cap = batch;
  return make_workspace_maps(m, *w, rows);
}

}  // namespace

extern "C" int nebw_encode_device_static(nebw_model *m, const int32_t *ids, const int32_t *lens,
                                         int32_t B, int32_t S, float *out, void *stream) {
  NEBW_REQUIRE(m && ids && lens && out, "null argument");
  if (int rc = use_dev(m->dev)) return rc;
  if (int rc = check_pass(m, B, S)) return rc;
  NEBW_REQUIRE(m->datapath == NEBW_DATAPATH_BF16,
               "nebw_encode_device_static runs the bf16 datapath; this model is set to the int8 "
               "datapath (use nebw_encode_device)");
  const int64_t rows = static_cast<int64_t>(B) * S;
  const size_t need = static_scratch_need(m, rows, B);
  NEBW_REQUIRE(need <= kStaticScratchBytes,
               "batch %d x seq %d needs %zu bytes of scratch for this model; the static scratch "
               "of nebw_encode_device_static holds %zu bytes (use nebw_encode_device)",
               B, S, need, kStaticScratchBytes);
  void *base = nullptr;
  if (int rc = static_scratch_address(m->dev->device, &base)) return rc;
  // the workspace is a stack object over the static array: the model's own
  // workspace is neither used nor grown, and no per-kernel profiling events
  // are recorded (they would be created on demand)
  Workspace w;
  if (int rc = static_workspace(m, base, rows, B, &w)) return rc;
  return encode_device(m, w, false, ids, lens, B, S, out, pick_stream(m->dev, stream));
}

// ---------------------------------------------------------------------------
// The ViT encoder: same translation unit (it uses the helpers above).
// ---------------------------------------------------------------------------

#include "vit.cuh"

// ---------------------------------------------------------------------------
// Several GPUs: the sharded pass and the NCCL gather.
// ---------------------------------------------------------------------------

#include "multi.cuh"
