// TEST INFRASTRUCTURE ONLY -- part of the parity oracle, never shipped.
//
// A C-ABI front for the reference's OWN host-CPU ViT encoder, compiled from
// the reference tree (see oracle/Makefile):
//
//   read_geometry(file)          runtime/include/vit/geometry.hpp
//   VitEncoder(file, design, pool, geometry), set_streams, stage_all
//                                runtime/src/vit/encoder.cpp:23-189
//   x = VitEncoder::run(patches) runtime/src/vit/encoder.cpp:222-431
//     (host GEMMs through NpuGemm::run_host = hostconv::gemm_nt, host
//     layernorm_rows / gelu_erf_inplace / attention from
//     runtime/src/whisper/npu_ops.cpp:449-620, as an empty --npu-ops selects)
//
// on a `gemm_layout:"host"` container.  The image -> patch step
// (im2col_patches, runtime/src/vit/image.cpp:732-755) lives in a file that
// also decodes JPEG/PNG and needs libjpeg, which this box does not have, so
// its index arithmetic is restated below, next to its citation.

#include <cstdint>
#include <cstring>
#include <exception>
#include <string>
#include <vector>

#include "runtime/design.hpp"
#include "runtime/device.hpp"
#include "runtime/model.hpp"
#include "runtime/pool.hpp"
#include "vit/encoder.hpp"
#include "vit/geometry.hpp"

void nebw_oracle_describe_design(const npue::File &f);  // oracle/ref_stub.cpp

namespace {
void set_err(char *err, int32_t errlen, const char *msg) {
  if (!err || errlen <= 0) return;
  std::strncpy(err, msg, static_cast<size_t>(errlen) - 1);
  err[errlen - 1] = '\0';
}

// image.cpp:732-755: patch row p*n + q, column (c*P + i)*P + j.
std::vector<float> patches_of(const float *chw, const npue::vit::Geometry &g) {
  const int64_t n = g.image_size / g.patch_size;
  std::vector<float> out(static_cast<size_t>(g.n_patches * g.patch_dim));
  for (int64_t p = 0; p < n; ++p)
    for (int64_t q = 0; q < n; ++q) {
      float *dst = out.data() + (p * n + q) * g.patch_dim;
      for (int64_t c = 0; c < g.num_channels; ++c)
        for (int64_t i = 0; i < g.patch_size; ++i)
          for (int64_t j = 0; j < g.patch_size; ++j)
            dst[(c * g.patch_size + i) * g.patch_size + j] =
                chw[(c * g.image_size + p * g.patch_size + i) * g.image_size + q * g.patch_size +
                    j];
    }
  return out;
}
}  // namespace

extern "C" {

// images [n, C, S, S] fp32 (already normalised) -> cls_out [n, hidden], the
// CLS row of VitEncoder::run's output; hidden_out optional [n, n_pos, hidden].
int nebw_ref_vit_encode(const char *npue_path, const float *images, int32_t n_images,
                        int32_t threads, float *cls_out, float *hidden_out, char *err,
                        int32_t errlen) {
  try {
    npue::File f(npue_path);
    nebw_oracle_describe_design(f);
    const npue::vit::Geometry g = npue::vit::read_geometry(f, npue_path);
    app::Pool pool(threads > 0 ? threads : 1);
    npu::Device dev;
    npu::Design d(dev, "oracle-host");
    npue::vit::VitEncoder enc(f, d, pool, g);
    npue::vit::EncoderStreams st;
    st.rows = g.n_pos;
    enc.set_streams(st);
    enc.stage_all();
    const int64_t img_elems = g.num_channels * g.image_size * g.image_size;
    for (int64_t i = 0; i < n_images; ++i) {
      const std::vector<float> x = enc.run(patches_of(images + i * img_elems, g));
      std::memcpy(cls_out + i * g.d_model, x.data(), static_cast<size_t>(g.d_model) * sizeof(float));
      if (hidden_out)
        std::memcpy(hidden_out + i * g.n_pos * g.d_model, x.data(), x.size() * sizeof(float));
    }
    return 0;
  } catch (const std::exception &e) {
    set_err(err, errlen, e.what());
    return 1;
  }
}

// A persistent reference ViT encoder over one container, for timing:
// open() stages it once (VitEncoder::stage_all), run() is the reference's
// steady-state per-image cost (im2col + VitEncoder::run).
struct RefVitSession {
  npue::File f;
  npue::vit::Geometry g;
  app::Pool pool;
  npu::Device dev;
  npu::Design design;
  npue::vit::VitEncoder enc;
  RefVitSession(const char *path, int threads)
      : f(path), g((nebw_oracle_describe_design(f), npue::vit::read_geometry(f, path))),
        pool(threads > 0 ? threads : 1),
        design(dev, "oracle-host"), enc(f, design, pool, g) {
    npue::vit::EncoderStreams st;
    st.rows = g.n_pos;
    enc.set_streams(st);
    enc.stage_all();
  }
};

void *nebw_ref_vit_session_open(const char *npue_path, int32_t threads, char *err,
                                int32_t errlen) {
  try {
    return new RefVitSession(npue_path, threads);
  } catch (const std::exception &e) {
    set_err(err, errlen, e.what());
    return nullptr;
  }
}

int nebw_ref_vit_session_run(void *handle, const float *images, int32_t n_images, float *cls_out,
                             char *err, int32_t errlen) {
  try {
    auto *s = static_cast<RefVitSession *>(handle);
    const int64_t img_elems = s->g.num_channels * s->g.image_size * s->g.image_size;
    for (int64_t i = 0; i < n_images; ++i) {
      const std::vector<float> x = s->enc.run(patches_of(images + i * img_elems, s->g));
      std::memcpy(cls_out + i * s->g.d_model, x.data(),
                  static_cast<size_t>(s->g.d_model) * sizeof(float));
    }
    return 0;
  } catch (const std::exception &e) {
    set_err(err, errlen, e.what());
    return 1;
  }
}

void nebw_ref_vit_session_close(void *handle) { delete static_cast<RefVitSession *>(handle); }

}  // extern "C"
