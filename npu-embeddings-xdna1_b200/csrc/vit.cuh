// The ViT encoder (container arch "vit_patch16_prenorm_gelu"), C ABI part of
// include/nebw.h.  This file is part of the nebw.cu translation unit (it is
// included at its end): it uses that file's device handle, weight staging,
// tensor maps, GEMM and attention launchers and error reporting.
//
// The pass mirrors VitEncoder::run (runtime/src/vit/encoder.cpp:222-431)
// over a batch of images, every image one unmasked sequence of n_pos rows:
//
//   vit_im2col      patches = bf16(im2col(image))         (image.cpp:732-755)
//   gemm PATCH      pe = patches . W_patch + b            (fp32)
//   vit_assemble    x = [cls; pe] + pos                   (encoder.cpp:267-281)
//   ln_rows         a = bf16(LN1_0(x))                    (x unchanged: pre-LN)
//   per layer L:
//     gemm QKV      qkv = bf16(a . Wqkv + b)
//     attention     ctx = softmax(Q K^T) V               (per image, per head)
//     gemm AO       y = bf16(ctx . Wao + b)
//     ln_rows       x += y;  a = bf16(LN2(x))
//     gemm UP       h = bf16(gelu_erf(a . Wup + b))
//     gemm DOWN     y = bf16(h . Wdn + b)
//     ln_rows       x += y;  a = bf16(LN1_L+1(x))          (last layer: the
//                   final LayerNorm of the CLS rows only, out = LN(x + y), fp32)
//
// The residual adds keep the reference's order -- the GEMM's (acc + bias)
// first, then + x (encoder.cpp:395-399, :408-411) -- with the sublayer output
// narrowed to bf16 RNE in between, as the reference's array path narrows
// every GEMM C tile (kernels/narrow_f32_bf16.cc:50-90); the residual stream
// and the LayerNorm arithmetic stay fp32.

#include "vitops.cuh"

struct VitLayerW {
  Weight qkv, ao, up, dn;
  float *b_qkv = nullptr, *b_ao = nullptr, *b_up = nullptr, *b_dn = nullptr;
  float *ln1_g = nullptr, *ln1_b = nullptr, *ln2_g = nullptr, *ln2_b = nullptr;
};

struct nebw_vit {
  nebw_dev *dev = nullptr;
  nebw_vit_config cfg{};
  int n_patches = 0, n_pos = 0, patch_dim = 0;
  Weight patch;
  float *patch_b = nullptr, *cls = nullptr, *pos = nullptr, *lnf_g = nullptr, *lnf_b = nullptr;
  std::vector<VitLayerW> layers;
  std::map<std::string, bool> staged;
  // workspace for img_cap images (rows_cap = img_cap * n_pos)
  int64_t img_cap = 0;
  float *x = nullptr;                                      // residual stream fp32 [R, H]
  __nv_bfloat16 *y = nullptr;                              // sublayer output bf16 [R, H]
  __nv_bfloat16 *a = nullptr, *qkv = nullptr, *ctx = nullptr, *h = nullptr;
  int *len = nullptr, *off = nullptr, *att_items = nullptr;
  float *images = nullptr, *out = nullptr;                 // staging for nebw_vit_encode
  // GEMM operand / output maps; the patches (bf16 [n*np, pd]) live in the
  // qkv buffer and the patch GEMM's fp32 output in the h buffer, both dead
  // at that point of the pass
  CUtensorMap map_a, map_ctx, map_h, map_patches;
  CUtensorMap out_qkv, out_h, out_y, out_pe, map_qkv_att, map_kv_att;
  // nebw_vit_encode: the stream its host->device chunk copies run on, and
  // one "chunk landed" event per chunk
  cudaStream_t copy_st = nullptr;
  std::vector<cudaEvent_t> chunk_ev;
  bool prof = false;
  std::vector<std::pair<cudaEvent_t, int>> marks;
  std::vector<cudaEvent_t> ev_pool;
  size_t ev_used = 0;
};

namespace {

void vit_free_workspace(nebw_vit *m) {
  for (void *p : {static_cast<void *>(m->x), static_cast<void *>(m->y), static_cast<void *>(m->a),
                  static_cast<void *>(m->qkv), static_cast<void *>(m->ctx),
                  static_cast<void *>(m->h), static_cast<void *>(m->len),
                  static_cast<void *>(m->off), static_cast<void *>(m->att_items),
                  static_cast<void *>(m->images), static_cast<void *>(m->out)})
    cudaFree(p);
  m->x = nullptr;
  m->y = nullptr;
  m->a = m->qkv = m->ctx = m->h = nullptr;
  m->len = m->off = m->att_items = nullptr;
  m->images = m->out = nullptr;
  m->img_cap = 0;
}

int vit_ensure_workspace(nebw_vit *m, int64_t n) {
  if (n <= m->img_cap) return NEBW_OK;
  NEBW_CUDA(cudaStreamSynchronize(m->dev->stream));
  vit_free_workspace(m);
  const nebw_vit_config &c = m->cfg;
  const int64_t H = c.hidden, F = c.intermediate, R = n * m->n_pos, NP = n * m->n_patches;
  const int64_t img_elems =
      static_cast<int64_t>(c.num_channels) * c.image_size * c.image_size;
  auto alloc = [&](void **p, size_t bytes) -> int {
    if (cudaMalloc(p, bytes) != cudaSuccess) {
      cudaGetLastError();
      return set_error(NEBW_ENOMEM, "ViT workspace allocation of %zu bytes failed", bytes);
    }
    return NEBW_OK;
  };
  int rc = 0;
  rc = rc ? rc : alloc(reinterpret_cast<void **>(&m->x), R * H * 4);
  rc = rc ? rc : alloc(reinterpret_cast<void **>(&m->y), R * H * 2);
  rc = rc ? rc : alloc(reinterpret_cast<void **>(&m->a), R * H * 2);
  rc = rc ? rc : alloc(reinterpret_cast<void **>(&m->qkv), R * 3 * H * 2);
  rc = rc ? rc : alloc(reinterpret_cast<void **>(&m->ctx), R * H * 2);
  rc = rc ? rc : alloc(reinterpret_cast<void **>(&m->h), R * F * 2);
  rc = rc ? rc : alloc(reinterpret_cast<void **>(&m->len), n * 4);
  rc = rc ? rc : alloc(reinterpret_cast<void **>(&m->off), (n + 1) * 4);
  rc = rc ? rc : alloc(reinterpret_cast<void **>(&m->att_items), (R / 128 + n + 1) * 4);
  rc = rc ? rc : alloc(reinterpret_cast<void **>(&m->images), n * img_elems * 4);
  rc = rc ? rc : alloc(reinterpret_cast<void **>(&m->out), n * H * 4);
  if (rc) {
    vit_free_workspace(m);
    return rc;
  }
  m->img_cap = n;
  if ((rc = make_tmap_kmajor(&m->map_a, m->a, R, H, nebw::kGemmBM))) return rc;
  if ((rc = make_tmap_kmajor(&m->map_ctx, m->ctx, R, H, nebw::kGemmBM))) return rc;
  if ((rc = make_tmap_kmajor(&m->map_h, m->h, R, F, nebw::kGemmBM))) return rc;
  if ((rc = make_tmap_kmajor(&m->map_patches, m->qkv, NP, m->patch_dim, nebw::kGemmBM))) return rc;
  if ((rc = make_tmap_out(&m->out_qkv, m->qkv, R, 3 * H, true))) return rc;
  if ((rc = make_tmap_out(&m->out_h, m->h, R, F, true))) return rc;
  if ((rc = make_tmap_out(&m->out_y, m->y, R, H, true))) return rc;
  if ((rc = make_tmap_out(&m->out_pe, m->h, NP, H, false))) return rc;
  if (nebw::attn_tc_head_dim(m->cfg.head_dim)) {
    if ((rc = make_tmap_head(&m->map_qkv_att, m->qkv, R, 3 * H, m->cfg.head_dim, 128))) return rc;
    if ((rc = make_tmap_head(&m->map_kv_att, m->qkv, R, 3 * H, m->cfg.head_dim, 64))) return rc;
  }
  return NEBW_OK;
}

std::vector<std::string> vit_required_names(const nebw_vit_config &c) {
  std::vector<std::string> v = {"frontend.patch_embed", "frontend.patch_embed.bias",
                                "frontend.cls_token", "frontend.position_embeddings",
                                "layernorm.weight", "layernorm.bias"};
  for (int L = 0; L < c.num_layers; ++L) {
    const std::string p = "layer." + std::to_string(L) + ".";
    for (const char *s : {"qkv", "qkv.bias", "attn_out", "attn_out.bias", "ln1.weight", "ln1.bias",
                          "ffn_up", "ffn_up.bias", "ffn_down", "ffn_down.bias", "ln2.weight",
                          "ln2.bias"})
      v.push_back(p + s);
  }
  return v;
}

int vit_ready(const nebw_vit *m) {
  for (const auto &n : vit_required_names(m->cfg))
    if (!m->staged.count(n))
      return set_error(NEBW_ESTATE, "ViT tensor '%s' has not been staged", n.c_str());
  return NEBW_OK;
}

int vit_mark(nebw_vit *m, int kind, cudaStream_t st) {
  if (!m->prof) return NEBW_OK;
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

template <int NV>
void launch_ln_rows_nv(float *x, const __nv_bfloat16 *y, int64_t stride, int rows,
                       const float *g, const float *b, float eps, int write_x, float *out_f32,
                       __nv_bfloat16 *out_a, cudaStream_t st) {
  const int grid = (rows + nebw::kRowWarps - 1) / nebw::kRowWarps;
  nebw::ln_rows_kernel<NV><<<grid, nebw::kRowWarps * 32, 0, st>>>(x, y, stride, rows, g, b, eps,
                                                                   write_x, out_f32, out_a);
}

// ln_rows_kernel: v = x (+ y), optionally written back to x; LN(v) to
// out_f32 and/or out_a.
int launch_ln_rows(float *x, const __nv_bfloat16 *y, int64_t stride, int64_t rows, int64_t H,
                   const float *g, const float *b, float eps, bool write_x, float *out_f32,
                   __nv_bfloat16 *out_a, cudaStream_t st) {
  NEBW_REQUIRE(H % 128 == 0 && H >= 128 && H <= 2048, "LayerNorm width %lld refused",
               static_cast<long long>(H));
  if (rows <= 0) return NEBW_OK;
  const int r = static_cast<int>(rows);
  switch (H / 128) {
#define NEBW_LNR_CASE(n) \
  case n: launch_ln_rows_nv<n>(x, y, stride, r, g, b, eps, write_x, out_f32, out_a, st); break;
    NEBW_LNR_CASE(1) NEBW_LNR_CASE(2) NEBW_LNR_CASE(3) NEBW_LNR_CASE(4) NEBW_LNR_CASE(5)
    NEBW_LNR_CASE(6) NEBW_LNR_CASE(7) NEBW_LNR_CASE(8) NEBW_LNR_CASE(9) NEBW_LNR_CASE(10)
    NEBW_LNR_CASE(11) NEBW_LNR_CASE(12) NEBW_LNR_CASE(13) NEBW_LNR_CASE(14) NEBW_LNR_CASE(15)
    NEBW_LNR_CASE(16)
#undef NEBW_LNR_CASE
    default: break;
  }
  NEBW_CUDA(cudaGetLastError());
  return NEBW_OK;
}

bool vit_tc_attention(const nebw_vit *m) {
  return m->dev->attn_kind == NEBW_ATTN_TCGEN05 && nebw::attn_tc_head_dim(m->cfg.head_dim);
}

int vit_encode_device(nebw_vit *m, const float *images, int n, float *out, cudaStream_t st) {
  nebw_dev *d = m->dev;
  const nebw_vit_config &c = m->cfg;
  if (int rc = vit_ready(m)) return rc;
  NEBW_REQUIRE(n > 0 && n <= 65535, "image count %d refused: 1..65535", n);
  NEBW_REQUIRE(reinterpret_cast<uintptr_t>(images) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(out) % 16 == 0,
               "images and output must be 16-byte aligned");
  if (int rc = vit_ensure_workspace(m, n)) return rc;
  const int64_t H = c.hidden, F = c.intermediate, R = static_cast<int64_t>(n) * m->n_pos;
  const int64_t NP = static_cast<int64_t>(n) * m->n_patches;
  NEBW_REQUIRE(R < (1ll << 30), "ViT batch of %lld rows refused", static_cast<long long>(R));
  const bool tc = vit_tc_attention(m);
  int rc;
  // image -> patches (bf16, in the qkv buffer)
  if ((rc = vit_mark(m, NEBW_K_PACK, st))) return rc;
  {
    const int64_t units = NP * c.num_channels * c.patch_size * (c.patch_size / 8);
    nebw::vit_im2col_kernel<<<static_cast<unsigned>((units + 255) / 256), 256, 0, st>>>(
        images, units, c.num_channels, c.image_size, c.patch_size, m->qkv);
    NEBW_CUDA(cudaGetLastError());
  }
  // patch embedding (fp32, in the h buffer), then x = [cls; pe] + pos
  if ((rc = vit_mark(m, NEBW_K_EMBED_LN, st))) return rc;
  GemmArgs a{};
  a.M = static_cast<int>(NP);
  a.M_dev = nullptr;
  a.N = static_cast<int>(H);
  a.K = m->patch_dim;
  a.bias = m->patch_b;
  a.resid = nullptr;
  a.out = m->h;
  a.err = d->d_err;
  if ((rc = launch_gemm(d, m->patch, m->map_patches, m->out_pe, nebw::kEpiF32, a, st))) return rc;
  {
    const int64_t v = R * (H / 4);
    nebw::vit_assemble_kernel<<<static_cast<unsigned>((v + 255) / 256), 256, 0, st>>>(
        reinterpret_cast<const float *>(m->h), m->cls, m->pos, n, m->n_pos, static_cast<int>(H),
        m->x);
    NEBW_CUDA(cudaGetLastError());
    nebw::uniform_seqs_kernel<<<(n + 1 + 255) / 256, 256, 0, st>>>(n, m->n_pos, m->len, m->off);
    NEBW_CUDA(cudaGetLastError());
    if (tc) {
      // with the work list, zero the Q|K|V and A rows just past this batch's
      // rows (inside the workspace's maps when an earlier batch was larger)
      nebw::attn_work_kernel<<<1 + nebw::kAttnTailBlocks, 1024, 0, st>>>(
          m->len, n, m->att_items + 1, m->att_items, m->off + n, m->img_cap * m->n_pos, m->qkv,
          static_cast<int>(3 * H), m->a, static_cast<int>(H));
      NEBW_CUDA(cudaGetLastError());
    }
  }
  a.M = static_cast<int>(R);
  // LN1 of layer 0; every later LayerNorm site is fused with the residual add
  // before it
  if ((rc = vit_mark(m, NEBW_K_LN, st))) return rc;
  if ((rc = launch_ln_rows(m->x, nullptr, 1, R, H, m->layers[0].ln1_g, m->layers[0].ln1_b,
                           c.layer_norm_eps, false, nullptr, m->a, st)))
    return rc;
  for (int L = 0; L < c.num_layers; ++L) {
    const VitLayerW &w = m->layers[L];
    // x += attn_out(attention(qkv(LN1(x))))
    a.N = static_cast<int>(3 * H);
    a.K = static_cast<int>(H);
    a.bias = w.b_qkv;
    a.resid = nullptr;
    a.out = m->qkv;
    if ((rc = vit_mark(m, NEBW_K_GEMM_QKV, st))) return rc;
    if ((rc = launch_gemm(d, w.qkv, m->map_a, m->out_qkv, nebw::kEpiBf16, a, st))) return rc;
    if ((rc = vit_mark(m, NEBW_K_ATTENTION, st))) return rc;
    if (tc)
      rc = launch_attention_tc(d, m->map_qkv_att, m->map_kv_att, m->off, m->len, m->att_items + 1,
                               m->att_items, n, m->n_pos, c.num_heads, c.head_dim, m->ctx, st);
    else
      rc = launch_attention(m->qkv, m->off, m->len, n, m->n_pos, c.num_heads, c.head_dim, m->ctx,
                            st);
    if (rc) return rc;
    a.N = static_cast<int>(H);
    a.K = static_cast<int>(H);
    a.bias = w.b_ao;
    a.out = m->y;
    if ((rc = vit_mark(m, NEBW_K_GEMM_AO, st))) return rc;
    if ((rc = launch_gemm(d, w.ao, m->map_ctx, m->out_y, nebw::kEpiBf16, a, st))) return rc;
    if ((rc = vit_mark(m, NEBW_K_LN, st))) return rc;
    if ((rc = launch_ln_rows(m->x, m->y, 1, R, H, w.ln2_g, w.ln2_b, c.layer_norm_eps, true,
                             nullptr, m->a, st)))
      return rc;
    // x += ffn_down(gelu_erf(ffn_up(LN2(x))))
    a.N = static_cast<int>(F);
    a.K = static_cast<int>(H);
    a.bias = w.b_up;
    a.out = m->h;
    if ((rc = vit_mark(m, NEBW_K_GEMM_UP, st))) return rc;
    if ((rc = launch_gemm(d, w.up, m->map_a, m->out_h, nebw::kEpiBf16Erf, a, st))) return rc;
    a.N = static_cast<int>(H);
    a.K = static_cast<int>(F);
    a.bias = w.b_dn;
    a.out = m->y;
    if ((rc = vit_mark(m, NEBW_K_GEMM_DOWN, st))) return rc;
    if ((rc = launch_gemm(d, w.dn, m->map_h, m->out_y, nebw::kEpiBf16, a, st))) return rc;
    if (L + 1 < c.num_layers) {
      if ((rc = vit_mark(m, NEBW_K_LN, st))) return rc;
      if ((rc = launch_ln_rows(m->x, m->y, 1, R, H, m->layers[L + 1].ln1_g,
                               m->layers[L + 1].ln1_b, c.layer_norm_eps, true, nullptr, m->a,
                               st)))
        return rc;
    } else {
      // the last residual add and the final LayerNorm, CLS rows only
      if ((rc = vit_mark(m, NEBW_K_POOL, st))) return rc;
      if ((rc = launch_ln_rows(m->x, m->y, m->n_pos, n, H, m->lnf_g, m->lnf_b, c.layer_norm_eps,
                               false, out, nullptr, st)))
        return rc;
    }
  }
  return vit_mark(m, -1, st);
}

}  // namespace

extern "C" int nebw_vit_create(nebw_dev *d, const nebw_vit_config *cfg, nebw_vit **out) {
  if (int rc = use_dev(d)) return rc;
  NEBW_REQUIRE(cfg && out, "null argument");
  const nebw_vit_config &c = *cfg;
  NEBW_REQUIRE(c.num_layers > 0 && c.hidden > 0 && c.num_heads > 0 && c.intermediate > 0 &&
                   c.image_size > 0 && c.patch_size > 0 && c.num_channels > 0,
               "the ViT model reports a non-positive shape");
  NEBW_REQUIRE(c.head_dim * c.num_heads == c.hidden, "head_dim * heads != hidden");
  NEBW_REQUIRE(c.head_dim == 32 || c.head_dim == 64, "head_dim %d refused: 32 or 64", c.head_dim);
  NEBW_REQUIRE(c.hidden % 128 == 0 && c.hidden <= 2048, "hidden %d refused: multiple of 128, <= 2048",
               c.hidden);
  NEBW_REQUIRE(c.intermediate % 64 == 0, "intermediate %d refused: multiple of 64", c.intermediate);
  NEBW_REQUIRE(c.image_size % c.patch_size == 0,
               "image_size %d is not a whole number of %d-pixel patches", c.image_size,
               c.patch_size);
  NEBW_REQUIRE(c.patch_size % 8 == 0, "patch_size %d refused: a multiple of 8", c.patch_size);
  NEBW_REQUIRE(c.num_channels * c.patch_size * c.patch_size == c.hidden,
               "patch_dim %d (channels x patch^2) is not hidden %d",
               c.num_channels * c.patch_size * c.patch_size, c.hidden);
  const int side = c.image_size / c.patch_size;
  NEBW_REQUIRE(side * side + 1 <= 4096, "%d patches refused", side * side);
  std::unique_ptr<nebw_vit> m(new nebw_vit());
  m->dev = d;
  m->cfg = c;
  m->n_patches = side * side;
  m->n_pos = side * side + 1;
  m->patch_dim = c.num_channels * c.patch_size * c.patch_size;
  m->layers.resize(c.num_layers);
  *out = m.release();
  return NEBW_OK;
}

extern "C" int nebw_vit_set_tensor(nebw_vit *m, const char *name, const void *host, int dtype,
                                   int64_t rows, int64_t cols) {
  NEBW_REQUIRE(m && name && host, "null argument");
  if (int rc = use_dev(m->dev)) return rc;
  const nebw_vit_config &c = m->cfg;
  const std::string n(name);
  const int64_t H = c.hidden, F = c.intermediate;
  auto expect = [&](int64_t r, int64_t cc) -> int {
    if (rows != r || cols != cc)
      return set_error(NEBW_EINVAL, "tensor '%s' is [%lld, %lld], expected [%lld, %lld]", name,
                       static_cast<long long>(rows), static_cast<long long>(cols),
                       static_cast<long long>(r), static_cast<long long>(cc));
    return NEBW_OK;
  };
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
  int rc = NEBW_OK;
  if (n == "frontend.patch_embed") rc = gemm_w(&m->patch, m->patch_dim, H);
  else if (n == "frontend.patch_embed.bias") rc = vec(&m->patch_b, H);
  else if (n == "frontend.cls_token") rc = vec(&m->cls, H);
  else if (n == "frontend.position_embeddings") {
    if (!(rc = expect(m->n_pos, H))) rc = upload_f32(m->dev, &m->pos, host, dtype, m->n_pos * H);
  } else if (n == "layernorm.weight") rc = vec(&m->lnf_g, H);
  else if (n == "layernorm.bias") rc = vec(&m->lnf_b, H);
  else if (n.rfind("layer.", 0) == 0) {
    const size_t dot = n.find('.', 6);
    NEBW_REQUIRE(dot != std::string::npos, "malformed tensor name '%s'", name);
    const int L = std::atoi(n.substr(6, dot - 6).c_str());
    NEBW_REQUIRE(L >= 0 && L < c.num_layers, "tensor '%s' names a layer outside [0, %d)", name,
                 c.num_layers);
    const std::string leaf = n.substr(dot + 1);
    VitLayerW &w = m->layers[L];
    if (leaf == "qkv") rc = gemm_w(&w.qkv, H, 3 * H);
    else if (leaf == "qkv.bias") rc = vec(&w.b_qkv, 3 * H);
    else if (leaf == "attn_out") rc = gemm_w(&w.ao, H, H);
    else if (leaf == "attn_out.bias") rc = vec(&w.b_ao, H);
    else if (leaf == "ffn_up") rc = gemm_w(&w.up, H, F);
    else if (leaf == "ffn_up.bias") rc = vec(&w.b_up, F);
    else if (leaf == "ffn_down") rc = gemm_w(&w.dn, F, H);
    else if (leaf == "ffn_down.bias") rc = vec(&w.b_dn, H);
    else if (leaf == "ln1.weight") rc = vec(&w.ln1_g, H);
    else if (leaf == "ln1.bias") rc = vec(&w.ln1_b, H);
    else if (leaf == "ln2.weight") rc = vec(&w.ln2_g, H);
    else if (leaf == "ln2.bias") rc = vec(&w.ln2_b, H);
    else return set_error(NEBW_EINVAL, "unknown ViT tensor '%s'", name);
  } else {
    return set_error(NEBW_EINVAL, "unknown ViT tensor '%s'", name);
  }
  if (rc == NEBW_OK) m->staged[n] = true;
  return rc;
}

extern "C" int nebw_vit_destroy(nebw_vit *m) {
  if (!m) return NEBW_OK;
  cudaSetDevice(m->dev->device);
  cudaStreamSynchronize(m->dev->stream);
  vit_free_workspace(m);
  for (cudaEvent_t e : m->ev_pool) cudaEventDestroy(e);
  for (cudaEvent_t e : m->chunk_ev) cudaEventDestroy(e);
  if (m->copy_st) cudaStreamDestroy(m->copy_st);
  cudaFree(m->patch.ptr);
  for (float *p : {m->patch_b, m->cls, m->pos, m->lnf_g, m->lnf_b}) cudaFree(p);
  for (auto &w : m->layers) {
    for (Weight *x : {&w.qkv, &w.ao, &w.up, &w.dn}) cudaFree(x->ptr);
    for (float *p : {w.b_qkv, w.b_ao, w.b_up, w.b_dn, w.ln1_g, w.ln1_b, w.ln2_g, w.ln2_b})
      cudaFree(p);
  }
  delete m;
  return NEBW_OK;
}

extern "C" int nebw_vit_get_config(const nebw_vit *m, nebw_vit_config *cfg) {
  NEBW_REQUIRE(m && cfg, "null argument");
  *cfg = m->cfg;
  return NEBW_OK;
}

// The container is read and checked before the device is touched
// (nebw_vit_create uses it), so a refused container is refused on any host.
extern "C" int nebw_vit_load_npue(nebw_dev *d, const char *path, nebw_vit **out) {
  NEBW_REQUIRE(path && out, "null argument");
  *out = nullptr;
  try {
    nebw::NpueFile f(path);
    const std::string arch = f.config_string("arch");
    if (arch != "vit_patch16_prenorm_gelu")
      return set_error(NEBW_EINVAL, "container architecture '%s' is not vit_patch16_prenorm_gelu",
                       arch.c_str());
    std::string layout = "pretiled_bf16";
    if (f.has_config("gemm_layout")) layout = f.config_string("gemm_layout");
    if (layout != "host" && layout != "pretiled_bf16")
      return set_error(NEBW_EINVAL,
                       "container gemm_layout '%s' refused: this library reads \"host\" (F32 "
                       "[K, N]) and the reference's pre-tiled block panels (\"pretiled_bf16\", "
                       "a_dtype bf16 or i8)", layout.c_str());
    const bool panels = layout == "pretiled_bf16";
    std::string a_dtype = "bf16";
    if (panels && f.has_config("a_dtype")) a_dtype = f.config_string("a_dtype");
    for (char &ch : a_dtype) ch = static_cast<char>(std::tolower(static_cast<unsigned char>(ch)));
    // (the BERT packer writes "bf16" / "i8", the ViT packer "BF16" / "I8")
    if (panels && a_dtype != "bf16" && a_dtype != "i8")
      return set_error(NEBW_EINVAL, "pre-tiled container with a_dtype '%s' refused: bf16 or i8 "
                       "(int4 panels are not read)", a_dtype.c_str());
    if (f.has_config("qkv_scale_folded") && f.config_string("qkv_scale_folded") == "false")
      return set_error(NEBW_EINVAL,
                       "container has qkv_scale_folded false: this library expects "
                       "1/sqrt(head_dim) folded into the Q operand, as the packer folds it");
    nebw_vit_config c{};
    c.num_layers = static_cast<int32_t>(f.config_int("num_layers"));
    c.hidden = static_cast<int32_t>(f.config_int("hidden"));
    c.num_heads = static_cast<int32_t>(f.config_int("num_heads"));
    c.head_dim = static_cast<int32_t>(f.config_int("head_dim"));
    c.intermediate = static_cast<int32_t>(f.config_int("intermediate"));
    c.image_size = static_cast<int32_t>(f.config_int("image_size"));
    c.patch_size = static_cast<int32_t>(f.config_int("patch_size"));
    c.num_channels = static_cast<int32_t>(f.config_int("num_channels"));
    c.layer_norm_eps = static_cast<float>(f.config_double("layer_norm_eps"));
    if (f.config_int("patch_dim") != static_cast<int64_t>(c.num_channels) * c.patch_size *
                                         c.patch_size ||
        f.config_int("max_seq_len") !=
            static_cast<int64_t>(c.image_size / c.patch_size) * (c.image_size / c.patch_size) + 1)
      return set_error(NEBW_EINVAL, "container patch_dim / max_seq_len disagree with its image "
                       "geometry");
    nebw_vit *m = nullptr;
    if (int rc = nebw_vit_create(d, &c, &m)) return rc;
    for (const auto &n : vit_required_names(c)) {
      const auto &t = f.tensor(n);
      const bool gemm_operand = t.shape.size() == 2 && !t.layout_kind.empty();
      if (t.dtype != "F32" && t.dtype != "BF16" && !(panels && gemm_operand && t.dtype == "I8")) {
        nebw_vit_destroy(m);
        return set_error(NEBW_EINVAL, "tensor '%s' has dtype %s; F32 or BF16 expected",
                         n.c_str(), t.dtype.c_str());
      }
      const int64_t r = t.shape.size() >= 1 ? t.shape[0] : 1;
      const int64_t cc = t.shape.size() >= 2 ? t.shape[1] : 1;
      const int dt = t.dtype == "F32" ? NEBW_F32 : NEBW_BF16;
      int rc;
      if (panels && gemm_operand) {
        // untiled on the host and staged as F32 [K, N]; an int8 operand's
        // optional .asmooth becomes a per-row factor 1/asmooth (1 where it is
        // not positive), as NpuGemm::run_host scales A (runtime/src/whisper/
        // npu_ops.cpp:96-116, 158-190), moved onto W
        std::vector<float> kn;
        rc = panel_to_kn(f, n, kn);
        const std::string an = n + ".asmooth";
        if (!rc && a_dtype == "i8" && f.has(an)) {
          const auto &at = f.tensor(an);
          if (at.dtype != "F32" || at.nbytes != static_cast<uint64_t>(r) * 4) {
            nebw_vit_destroy(m);
            return set_error(NEBW_EINVAL, "%s must be F32 [%lld]", an.c_str(),
                             static_cast<long long>(r));
          }
          std::vector<float> as(static_cast<size_t>(r));
          std::memcpy(as.data(), at.data, as.size() * 4);
          for (int64_t k = 0; k < r; ++k) {
            const float inv = as[static_cast<size_t>(k)] > 0.f ? 1.0f / as[static_cast<size_t>(k)]
                                                                : 1.0f;
            for (int64_t j = 0; j < cc; ++j) kn[static_cast<size_t>(k * cc + j)] *= inv;
          }
        }
        if (!rc) rc = nebw_vit_set_tensor(m, n.c_str(), kn.data(), NEBW_F32, r, cc);
      } else {
        rc = nebw_vit_set_tensor(m, n.c_str(), t.data, dt, r, cc);
      }
      if (rc) {
        const std::string msg = g_last_error;
        nebw_vit_destroy(m);
        return set_error(rc, "%s", msg.c_str());
      }
    }
    *out = m;
    return NEBW_OK;
  } catch (const std::exception &e) {
    return set_error(NEBW_EIO, "%s", e.what());
  }
}

extern "C" int nebw_vit_encode_device(nebw_vit *m, const float *images, int32_t n, float *out,
                                      void *stream) {
  NEBW_REQUIRE(m && images && out, "null argument");
  if (int rc = use_dev(m->dev)) return rc;
  return vit_encode_device(m, images, n, out, pick_stream(m->dev, stream));
}

// Host buffers: the batch is split into up to kVitChunks chunks whose
// host->device copies run on a second stream, so that chunk i + 1 crosses
// PCIe while the encoder runs on chunk i (only the first chunk's copy is
// exposed); the pass over each chunk is the device pass above.  With
// pageable host memory the copies are synchronous and nothing overlaps,
// with the same results.
constexpr int kVitChunks = 8;
constexpr int kVitMinChunk = 256;  // images; smaller batches go in one piece

extern "C" int nebw_vit_encode(nebw_vit *m, const float *images, int32_t n, float *out) {
  NEBW_REQUIRE(m && images && out, "null argument");
  if (int rc = use_dev(m->dev)) return rc;
  NEBW_REQUIRE(n > 0, "empty batch refused");
  if (int rc = vit_ready(m)) return rc;
  if (int rc = vit_ensure_workspace(m, n)) return rc;
  const nebw_vit_config &c = m->cfg;
  cudaStream_t st = m->dev->stream;
  if (!m->copy_st) NEBW_CUDA(cudaStreamCreateWithFlags(&m->copy_st, cudaStreamNonBlocking));
  while (static_cast<int>(m->chunk_ev.size()) < kVitChunks) {
    cudaEvent_t e;
    NEBW_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    m->chunk_ev.push_back(e);
  }
  const size_t per_img = static_cast<size_t>(c.num_channels) * c.image_size * c.image_size;
  const int chunk = n < 2 * kVitMinChunk
                        ? n
                        : std::max(kVitMinChunk, (n + kVitChunks - 1) / kVitChunks);
  const int nchunks = (n + chunk - 1) / chunk;
  // the copies may start once the previous call's work on the stream is done
  NEBW_CUDA(cudaEventRecord(m->chunk_ev[0], st));
  NEBW_CUDA(cudaStreamWaitEvent(m->copy_st, m->chunk_ev[0], 0));
  for (int i = 0; i < nchunks; ++i) {
    const int i0 = i * chunk, cnt = std::min(chunk, n - i0);
    NEBW_CUDA(cudaMemcpyAsync(m->images + i0 * per_img, images + i0 * per_img,
                              static_cast<size_t>(cnt) * per_img * 4, cudaMemcpyHostToDevice,
                              m->copy_st));
    NEBW_CUDA(cudaEventRecord(m->chunk_ev[i], m->copy_st));
  }
  for (int i = 0; i < nchunks; ++i) {
    const int i0 = i * chunk, cnt = std::min(chunk, n - i0);
    NEBW_CUDA(cudaStreamWaitEvent(st, m->chunk_ev[i], 0));
    if (int rc = vit_encode_device(m, m->images + i0 * per_img, cnt,
                                   m->out + static_cast<size_t>(i0) * c.hidden, st))
      return rc;
  }
  NEBW_CUDA(cudaMemcpyAsync(out, m->out, static_cast<size_t>(n) * c.hidden * 4,
                            cudaMemcpyDeviceToHost, st));
  return nebw_sync(m->dev);
}

extern "C" int nebw_vit_launch_count(const nebw_vit *m) {
  if (!m) return set_error(NEBW_EINVAL, "null model"), -1;
  const bool tc = vit_tc_attention(m);
  return 5 + (tc ? 1 : 0) + m->cfg.num_layers * (6 + attention_launches(tc ? 64 : 0, m->n_pos));
}

extern "C" int nebw_vit_profile(nebw_vit *m, int enable) {
  NEBW_REQUIRE(m != nullptr, "null model");
  m->prof = enable != 0;
  return NEBW_OK;
}

extern "C" int nebw_vit_profile_collect(nebw_vit *m, int64_t launches[NEBW_K_COUNT],
                                        double ms[NEBW_K_COUNT]) {
  NEBW_REQUIRE(m && launches && ms, "null argument");
  if (int rc = use_dev(m->dev)) return rc;
  for (int k = 0; k < NEBW_K_COUNT; ++k) {
    launches[k] = 0;
    ms[k] = 0.0;
  }
  for (size_t i = 0; i + 1 < m->marks.size(); ++i) {
    const int kind = m->marks[i].second;
    if (kind < 0) continue;
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
