// TEST INFRASTRUCTURE ONLY -- part of the parity oracle, never shipped.
//
// A C ABI over the reference's own int8 host steps, the header templates of
// runtime/include/common/host_kernels.hpp compiled from the reference tree
// where it lies (namespace app):
//   quantise_a_int8    :263-315  A -> int8 per row, SmoothQuant divisor folded
//   dequantise_c       :529-614  int32 C -> fp32 with row/column scales + bias
//   dequant_act_quant  :404-526  the FFN-up epilogue: dequantise, act, quantise
// and the reference's reader of pre-tiled GEMM operands,
//   npue::hostb::host_b_kn (runtime/include/common/host_b.hpp:74-224)
// over a container opened with npue::File (runtime/src/model.cpp).
// Rows run serially (the templates' par_rows argument); the act given to
// dequant_act_quant applies the reference's gelu8 (host_kernels.hpp:325-352),
// the BERT FFN's activation.  The buffers handed to the reference are
// 32-byte aligned with N % 8 == 0, as its streaming loads require
// (require_stream_aligned, host_kernels.hpp:112-130).

#include <immintrin.h>

#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <exception>

#include "common/host_kernels.hpp"
#include "runtime/model.hpp"
#include "common/host_b.hpp"

namespace {

auto serial_rows = [](int64_t n, auto f) { f(int64_t{0}, n); };

// An aligned copy of C, since the caller's buffer need not be 32-byte aligned.
struct AlignedC {
  int32_t *p = nullptr;
  AlignedC(const int32_t *src, size_t n) {
    p = static_cast<int32_t *>(std::aligned_alloc(32, ((n * 4 + 31) / 32) * 32));
    if (p) std::memcpy(p, src, n * 4);
  }
  ~AlignedC() { std::free(p); }
};

}  // namespace

extern "C" {

int nebw_ref_quantise_a_int8(const float *a, int64_t rows, int64_t K, const float *ias,
                             int8_t *q, float *scale) {
  try {
    app::quantise_a_int8(a, rows, K, ias, q, scale, serial_rows);
    return 0;
  } catch (const std::exception &) {
    return 1;
  }
}

int nebw_ref_dequantise_c(const int32_t *c, int64_t rows, int64_t N, const float *sa,
                          const float *ws, const float *bias, float *out) {
  AlignedC ca(c, static_cast<size_t>(rows * N));
  if (!ca.p) return 2;
  try {
    app::dequantise_c(ca.p, 4, rows, N, sa, ws, bias, out, serial_rows);
    return 0;
  } catch (const std::exception &) {
    return 1;
  }
}

int nebw_ref_dequant_gelu_quant(const int32_t *c, int64_t rows, int64_t N, const float *sa,
                                const float *ws, const float *bias, const float *ias_next,
                                int8_t *q, float *sa_next) {
  AlignedC ca(c, static_cast<size_t>(rows * N));
  if (!ca.p) return 2;
  auto gelu = [](float *v, int64_t n) {
    int64_t j = 0;
    for (; j + 8 <= n; j += 8) _mm256_storeu_ps(v + j, app::gelu8(_mm256_loadu_ps(v + j)));
    for (; j < n; ++j) v[j] = app::gelu8(v[j]);
  };
  try {
    app::dequant_act_quant(ca.p, 4, rows, N, N, gelu, sa, ws, bias, ias_next, q, sa_next,
                           serial_rows);
    return 0;
  } catch (const std::exception &) {
    return 1;
  }
}

// `name` of the container at `path` as fp32 [K, N] (BF16 widened, I8
// dequantised by .wscale); returns 0, or 1 when the reference refuses.
int nebw_ref_host_b_kn(const char *path, const char *name, float *out, int64_t K, int64_t N) {
  try {
    npue::File f(path);
    const std::vector<float> kn = npue::hostb::host_b_kn(f, name);
    if (static_cast<int64_t>(kn.size()) != K * N) return 2;
    std::memcpy(out, kn.data(), kn.size() * 4);
    return 0;
  } catch (const std::exception &) {
    return 1;
  }
}

}  // extern "C"
