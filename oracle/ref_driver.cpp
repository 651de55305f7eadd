// TEST INFRASTRUCTURE ONLY -- part of the parity oracle, never shipped.
//
// A C-ABI front for the reference's OWN host-CPU encoder, compiled from the
// reference tree (see oracle/Makefile).  It drives exactly the call sequence
// the reference's embedding service uses:
//
//   EmbedService::chunk          runtime/src/server/embed_service.cpp:29-64
//     x[b,s,:] = (word[id] + pos[s]) + type[0]      (:51-57, order kept)
//     add_mask  = 0 / -1e30 from the 1/0 attention mask (:49)
//     h = BertEncoder::run(x)    runtime/src/encoders/bert_encoder.cpp:1419-1598
//     pool_rows(h, mask)         runtime/include/common/app_state.hpp:335-374
//
// with the encoder set up the way setup_encoder() does for an all-host run:
// set_model_shape (app_state.hpp:380), set_design_seq (:637), host_ln /
// host_sm / host_gelu true, stage_all() (bert_encoder.cpp:41-172), so every
// GEMM is hostconv::gemm_nt over the operand as fp32 [K,N]: a
// `gemm_layout:"host"` container's F32 operand, or a pre-tiled container's
// panel untiled by host_b.hpp (int8 dequantised by .wscale, A divided by
// .asmooth), the stand-in design describing that container's operands.
//
// It also exposes a few of the reference's inline host kernels one by one
// (gemm_nt, gelu8, to_bf16, exp2_avx2, pool_rows) so the CPU restatement in
// oracle/bert_oracle.c can be pinned op by op as well as end to end.

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <exception>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "common/app_state.hpp"
#include "common/conv_host.hpp"
#include "common/host_b.hpp"
#include "common/host_kernels.hpp"
#include "common/npu_ops_flag.hpp"
#include "encoders/bert_encoder.hpp"
#include "runtime/design.hpp"
#include "runtime/device.hpp"
#include "runtime/model.hpp"
#include "runtime/pool.hpp"
#include "ref_array.hpp"
#include "tokenizers/wordpiece.hpp"

void nebw_oracle_describe_design(const npue::File &f);  // oracle/ref_stub.cpp
extern size_t nebw_oracle_a_elem_bytes;                 // oracle/ref_stub.cpp

namespace {
void set_err(char *err, int32_t errlen, const char *msg) {
  if (!err || errlen <= 0) return;
  std::strncpy(err, msg, static_cast<size_t>(errlen) - 1);
  err[errlen - 1] = '\0';
}

// The EmbedService::chunk gather into x, the encoder's add_mask and the
// pooling mask, for `batch` sequences of `seq` ids (embed_service.cpp:29-64).
void gather_rows(const npue::File &f, int64_t seq, const int32_t *ids, const int32_t *attn_mask,
                 int64_t batch, std::vector<float> &x, std::vector<float> &cmask,
                 std::vector<float> &cam) {
  const int64_t H = app::g_hidden;
  const float *w_word = f.raw("embeddings.word").as<float>();
  const float *w_pos = f.raw("embeddings.position").as<float>();
  const float *w_typ = f.raw("embeddings.token_type").as<float>();
  x.assign(static_cast<size_t>(batch) * seq * H, 0.f);
  cmask.assign(static_cast<size_t>(batch) * seq, -1.0e30f);
  cam.assign(static_cast<size_t>(batch) * seq, 0.f);
  for (int64_t b = 0; b < batch; ++b)
    for (int64_t s = 0; s < seq; ++s) {
      const int32_t id = ids[b * seq + s];
      const float m = static_cast<float>(attn_mask[b * seq + s]);
      cam[b * seq + s] = m;
      cmask[b * seq + s] = m > 0 ? 0.f : -1.0e30f;
      float *dst = x.data() + (b * seq + s) * H;
      const float *wv = w_word + static_cast<size_t>(id) * H;
      const float *pv = w_pos + static_cast<size_t>(s) * H;
      for (int64_t c = 0; c < H; ++c) dst[c] = wv[c] + pv[c] + w_typ[c];
    }
}

// Switches the stand-in design's array emulation on for one encode and off
// again however the encode ends.
struct ArrayEmulation {
  ArrayEmulation() {
    nebw_array_registry.clear();
    app::g_npu_ops = {"gemm"};
  }
  ~ArrayEmulation() {
    nebw_array_on = false;
    nebw_array_registry.clear();
    nebw_array_a.clear();
    nebw_array_c.clear();
    app::g_npu_ops.clear();
  }
};

}  // namespace

extern "C" {

// Encode `batch` sequences of `seq` token ids through the reference host path.
//   ids        [batch, seq] int32, tokenizer output (pad id in padded slots)
//   attn_mask  [batch, seq] int32 1/0
//   out        [batch, hidden] fp32, pooled (+L2 as the container says)
//   hidden_out optional [batch*seq, hidden] fp32: BertEncoder::run's output
// Returns 0, or 1 with `err` holding the reference's exception text.
int nebw_ref_encode(const char *npue_path, int32_t seq, const int32_t *ids,
                    const int32_t *attn_mask, int32_t batch, int32_t threads,
                    float *out, float *hidden_out, char *err, int32_t errlen) {
  try {
    npue::File f(npue_path);
    nebw_oracle_describe_design(f);
    app::set_model_shape(f);
    app::set_design_seq(seq);
    app::Pool pool(threads > 0 ? threads : 1);
    npu::Device dev;
    npu::Design d(dev, "oracle-host");
    npue::BertEncoder enc(f, d, d, d, d, d, d, d, pool);
    enc.host_ln = enc.host_sm = enc.host_gelu = true;
    enc.batch = batch;
    enc.rows = static_cast<int64_t>(batch) * seq;
    enc.stage_all();

    const int64_t H = app::g_hidden;
    const float *w_word = f.raw("embeddings.word").as<float>();
    const float *w_pos = f.raw("embeddings.position").as<float>();
    const float *w_typ = f.raw("embeddings.token_type").as<float>();
    std::vector<float> buf(static_cast<size_t>(batch) * seq * H, 0.f);
    std::vector<float> cmask(static_cast<size_t>(batch) * seq, -1.0e30f);
    std::vector<float> cam(static_cast<size_t>(batch) * seq, 0.f);
    for (int64_t b = 0; b < batch; ++b) {
      for (int64_t s = 0; s < seq; ++s) {
        const int32_t id = ids[b * seq + s];
        const float m = static_cast<float>(attn_mask[b * seq + s]);
        cam[b * seq + s] = m;
        cmask[b * seq + s] = m > 0 ? 0.f : -1.0e30f;
        float *dst = buf.data() + (b * seq + s) * H;
        const float *wv = w_word + static_cast<size_t>(id) * H;
        const float *pv = w_pos + static_cast<size_t>(s) * H;
        for (int64_t c = 0; c < H; ++c) dst[c] = wv[c] + pv[c] + w_typ[c];
      }
    }
    enc.add_mask = cmask;
    std::vector<float> h = enc.run(buf);
    if (hidden_out) std::memcpy(hidden_out, h.data(), h.size() * sizeof(float));
    app::pool_rows(h.data(), cam.data(), batch, out);
    return 0;
  } catch (const std::exception &e) {
    set_err(err, errlen, e.what());
    return 1;
  }
}

// The reference's int8 ARRAY path on an int8 container (a_dtype "i8", int8
// block panels with .wscale / .asmooth): BertEncoder::run as `--npu-ops gemm`
// runs it (bert_encoder.cpp:741-923, 1419-1598) -- each of the four GEMMs a
// dispatch on the array, everything else on the host, the fused epilogues on
// (fuse_ffn_epilogue's default, run_setup.hpp:694):
//   QKV   quantise_a_int8(x) (layer 0) or the previous add_norm_quant's rows,
//         int32 product, dequantise_c -> fp32 qkv; host attention -> fp32 ctx
//   AO    quantise_a_int8(ctx), int32 product, dequantise_c -> proj;
//         add_norm_quant(x, proj) quantises FFN-up's A
//   UP    int32 product, dequant_act_quant (gelu8, FFN-down's A)
//   DOWN  int32 product, dequantise_c; add_norm_quant quantises the next
//         layer's QKV A (the last layer: LayerNorm only)
// The dispatches are the stand-in design's emulation (ref_stub.cpp): the
// exact int32 product of the int8 rows and the operand, recovered as int8
// [K, N] from the reference's own untiler (host_b_kn hands back
// float(q) * wscale, and rint(that / wscale) = q exactly for |q| <= 127).
// Arguments and result as nebw_ref_encode.
int nebw_ref_encode_array(const char *npue_path, int32_t seq, const int32_t *ids,
                          const int32_t *attn_mask, int32_t batch, int32_t threads, float *out,
                          float *hidden_out, char *err, int32_t errlen) {
  try {
    ArrayEmulation emu;
    npue::File f(npue_path);
    nebw_oracle_describe_design(f);
    if (nebw_oracle_a_elem_bytes != 1)
      throw std::runtime_error("the array emulation runs int8 containers (a_dtype i8) only");
    app::set_model_shape(f);
    app::set_design_seq(seq);
    const int64_t rows = static_cast<int64_t>(batch) * seq;
    int64_t max_k = 0, max_n = 0;
    for (int64_t L = 0; L < app::g_layers; ++L)
      for (const char *g : {"qkv", "attn_out", "ffn_up", "ffn_down"}) {
        const std::string name = "layer." + std::to_string(L) + "." + g;
        const npue::TensorInfo &t = f.info(name);
        if (t.dtype != "I8") throw std::runtime_error(name + ": the emulation takes I8 panels");
        const npue::Panel panel = npue::gemm_b_panel(f, name, 1);
        const std::vector<float> w = npue::hostb::host_b_kn(f, name);
        const float *ws = f.raw(name + ".wscale").as<float>();
        NebwArrayOperand op;
        op.K = t.padded_shape[0];
        op.N = t.padded_shape[1];
        op.kn.resize(static_cast<size_t>(op.K * op.N));
        for (int64_t k = 0; k < op.K; ++k)
          for (int64_t n = 0; n < op.N; ++n) {
            const float v = w[k * op.N + n];
            const float q = ws[n] != 0.f ? std::rint(v / ws[n]) : 0.f;
            if (!(q >= -127.f && q <= 127.f) || (ws[n] == 0.f && v != 0.f))
              throw std::runtime_error(name + ": operand does not recover as int8");
            op.kn[k * op.N + n] = static_cast<int8_t>(q);
          }
        max_k = std::max(max_k, op.K);
        max_n = std::max(max_n, op.N);
        nebw_array_registry[panel.bytes.data] = std::move(op);
      }
    nebw_array_rows = rows;
    nebw_array_a.assign(static_cast<size_t>(rows * max_k + 64), 0);
    nebw_array_c.assign(static_cast<size_t>(rows * max_n + 16), 0);
    nebw_array_on = true;

    app::Pool pool(threads > 0 ? threads : 1);
    npu::Device dev;
    npu::Design d(dev, "oracle-array");
    npue::BertEncoder enc(f, d, d, d, d, d, d, d, pool);
    enc.host_ln = enc.host_sm = enc.host_gelu = true;
    enc.batch = batch;
    enc.rows = rows;
    enc.stage_all();
    std::vector<float> x, cmask, cam;
    gather_rows(f, seq, ids, attn_mask, batch, x, cmask, cam);
    enc.add_mask = cmask;
    std::vector<float> h = enc.run(x);
    if (hidden_out) std::memcpy(hidden_out, h.data(), h.size() * sizeof(float));
    app::pool_rows(h.data(), cam.data(), batch, out);
    return 0;
  } catch (const std::exception &e) {
    set_err(err, errlen, e.what());
    return 1;
  }
}

// A persistent reference encoder, for timing: the container is mapped, the
// encoder constructed and its weights staged (stage_all; the first run()
// also builds host_b.hpp's fp32 weight cache) once, and every
// nebw_ref_session_run() is then the reference's steady-state per-request
// work -- the gather, BertEncoder::run and pool_rows of EmbedService::chunk.
struct RefSession {
  npue::File file;
  app::Pool pool;
  npu::Device dev;
  npu::Design design;
  npue::BertEncoder enc;
  int32_t seq;
  RefSession(const char *path, int32_t s, int32_t threads)
      : file(path), pool(threads > 0 ? threads : 1), design(dev, "oracle-host"),
        enc(file, design, design, design, design, design, design, design, pool), seq(s) {}
};

void *nebw_ref_session_open(const char *npue_path, int32_t seq, int32_t threads, char *err,
                            int32_t errlen) {
  try {
    // geometry globals first: the encoder's constructor and stage_all read them
    {
      npue::File probe(npue_path);
      nebw_oracle_describe_design(probe);
      app::set_model_shape(probe);
      app::set_design_seq(seq);
    }
    auto *s = new RefSession(npue_path, seq, threads);
    s->enc.host_ln = s->enc.host_sm = s->enc.host_gelu = true;
    s->enc.stage_all();
    return s;
  } catch (const std::exception &e) {
    set_err(err, errlen, e.what());
    return nullptr;
  }
}

int nebw_ref_session_run(void *handle, const int32_t *ids, const int32_t *attn_mask,
                         int32_t batch, float *out, char *err, int32_t errlen) {
  try {
    auto *s = static_cast<RefSession *>(handle);
    const int64_t seq = s->seq, H = app::g_hidden;
    s->enc.batch = batch;
    s->enc.rows = static_cast<int64_t>(batch) * seq;
    const float *w_word = s->file.raw("embeddings.word").as<float>();
    const float *w_pos = s->file.raw("embeddings.position").as<float>();
    const float *w_typ = s->file.raw("embeddings.token_type").as<float>();
    std::vector<float> buf(static_cast<size_t>(batch) * seq * H, 0.f);
    std::vector<float> cmask(static_cast<size_t>(batch) * seq, -1.0e30f);
    std::vector<float> cam(static_cast<size_t>(batch) * seq, 0.f);
    for (int64_t b = 0; b < batch; ++b)
      for (int64_t t = 0; t < seq; ++t) {
        const int32_t id = ids[b * seq + t];
        const float m = static_cast<float>(attn_mask[b * seq + t]);
        cam[b * seq + t] = m;
        cmask[b * seq + t] = m > 0 ? 0.f : -1.0e30f;
        float *dst = buf.data() + (b * seq + t) * H;
        const float *wv = w_word + static_cast<size_t>(id) * H;
        const float *pv = w_pos + static_cast<size_t>(t) * H;
        for (int64_t c = 0; c < H; ++c) dst[c] = wv[c] + pv[c] + w_typ[c];
      }
    s->enc.add_mask = cmask;
    std::vector<float> h = s->enc.run(buf);
    app::pool_rows(h.data(), cam.data(), batch, out);
    return 0;
  } catch (const std::exception &e) {
    set_err(err, errlen, e.what());
    return 1;
  }
}

void nebw_ref_session_close(void *handle) { delete static_cast<RefSession *>(handle); }

// npue::hostconv::gemm_nt (runtime/include/common/conv_host.hpp:150-181):
// C[M,N] = A[M,K] . B[K,N] + bias, fp32.
int nebw_ref_gemm_nt(const float *A, int64_t M, const float *B, int64_t K,
                     int64_t N, const float *bias, float *C, int32_t threads) {
  app::Pool pool(threads > 0 ? threads : 1);
  npue::hostconv::gemm_nt(A, M, B, K, N, bias, C, pool);
  return 0;
}

// app::gelu8, scalar form (runtime/include/common/host_kernels.hpp:340-352),
// and the 8-wide AVX2 form gelu_cpu() uses for all but the tail
// (bert_encoder.cpp:532-580).
void nebw_ref_gelu8(float *x, int64_t n) {
  int64_t i = 0;
#if defined(__AVX2__)
  for (; i + 8 <= n; i += 8)
    _mm256_storeu_ps(x + i, app::gelu8(_mm256_loadu_ps(x + i)));
#endif
  for (; i < n; ++i) x[i] = app::gelu8(x[i]);
}

// app::exp2_avx2 (host_kernels.hpp:354-380), 8 lanes at a time; n % 8 == 0.
void nebw_ref_exp2(float *x, int64_t n) {
#if defined(__AVX2__)
  for (int64_t i = 0; i + 8 <= n; i += 8)
    _mm256_storeu_ps(x + i, app::exp2_avx2(_mm256_loadu_ps(x + i)));
#else
  (void)x; (void)n;
#endif
}

// app::to_bf16 (host_kernels.hpp:157-161), fp32 -> bf16 RNE bit pattern.
void nebw_ref_to_bf16(const float *x, uint16_t *out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = app::to_bf16(x[i]);
}

// app::pool_rows (app_state.hpp:335-374) with the geometry globals it reads
// set from the arguments.
int nebw_ref_pool_rows(const float *h, const float *am, int64_t take,
                       int64_t seq, int64_t hidden, int32_t cls, int32_t l2,
                       float *out, char *err, int32_t errlen) {
  try {
    app::g_seq = seq;
    app::g_hidden = hidden;
    app::g_cls_pool = cls != 0;
    app::g_l2_normalize = l2 != 0;
    app::pool_rows(h, am, take, out);
    return 0;
  } catch (const std::exception &e) {
    set_err(err, errlen, e.what());
    return 1;
  }
}

// The reference's WordPiece (runtime/src/tokenizers/wordpiece.cpp) on one
// text: ids and the 1/0 mask padded to max_len, as EmbedService::chunk gets
// them.  Returns 0, or 1 with `err` set.
int nebw_ref_wordpiece(const char *vocab_path, const char *text, int32_t max_len, int32_t *ids,
                       int32_t *mask, char *err, int32_t errlen) {
  try {
    const npue::WordPiece wp = npue::WordPiece::from_vocab_file(vocab_path);
    const npue::Encoded e = wp.encode(text, max_len);
    for (int32_t i = 0; i < max_len; ++i) {
      ids[i] = e.input_ids[static_cast<size_t>(i)];
      mask[i] = e.attention_mask[static_cast<size_t>(i)];
    }
    return 0;
  } catch (const std::exception &ex) {
    set_err(err, errlen, ex.what());
    return 1;
  }
}

}  // extern "C"
