/* TEST INFRASTRUCTURE ONLY -- the parity oracle, never shipped.
 *
 * Plain-C restatement of the reference's host-CPU BERT path.  Each function
 * names the reference code it follows.  The reference build is
 * -O2 -march=x86-64-v3 (runtime/CMakeLists.txt:297-302), so its host kernels
 * take their AVX2 branches; this file restates the ARITHMETIC ORDER of those
 * branches in scalar C -- eight-lane partial sums reduced the way hsum256
 * reduces them, fused multiply-adds exactly where _mm256_fmadd_ps stands --
 * so that it reproduces the compiled reference closely (bit-exactly where the
 * compiler contracts the same way; tests/test_oracle_pin.py measures it).
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load
 * this library.
 */
#define _GNU_SOURCE
#include "bert_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

static __thread char g_err[512];

const char *nebw_oracle_last_error(void) { return g_err; }

static int fail(const char *msg) {
  snprintf(g_err, sizeof g_err, "%s", msg);
  return 1;
}

/* ---- a tiny static-chunk parallel-for (stands in for app::Pool) ---------- */

typedef void (*range_fn)(void *ctx, int64_t lo, int64_t hi);
typedef struct {
  range_fn fn;
  void *ctx;
  int64_t lo, hi;
} job_t;

static void *job_main(void *p) {
  job_t *j = (job_t *)p;
  if (j->lo < j->hi) j->fn(j->ctx, j->lo, j->hi);
  return NULL;
}

static void parallel_for(int64_t n, int32_t threads, range_fn fn, void *ctx) {
  if (threads <= 1 || n <= 1) {
    fn(ctx, 0, n);
    return;
  }
  if (threads > 256) threads = 256;
  if ((int64_t)threads > n) threads = (int32_t)n;
  pthread_t tid[256];
  job_t jobs[256];
  const int64_t chunk = (n + threads - 1) / threads;
  for (int32_t w = 0; w < threads; ++w) {
    int64_t lo = chunk * w, hi = lo + chunk;
    if (lo > n) lo = n;
    if (hi > n) hi = n;
    jobs[w] = (job_t){fn, ctx, lo, hi};
    if (w > 0) pthread_create(&tid[w], NULL, job_main, &jobs[w]);
  }
  job_main(&jobs[0]);
  for (int32_t w = 1; w < threads; ++w) pthread_join(tid[w], NULL);
}

/* ---- arithmetic primitives ----------------------------------------------- */

/* hsum256 (runtime/include/common/host_kernels.hpp:617-623): lo = v[0:4] +
 * v[4:8], then two horizontal adds. */
static inline float hsum8(const float s[8]) {
  const float lo0 = s[0] + s[4], lo1 = s[1] + s[5];
  const float lo2 = s[2] + s[6], lo3 = s[3] + s[7];
  return (lo0 + lo1) + (lo2 + lo3);
}

/* exp2_avx2 (host_kernels.hpp:354-380): k = trunc(x), f = x - k, degree-7
 * Horner polynomial in f with the reference's own coefficients, times 2^k
 * built from the exponent bits. */
static inline float exp2_ref(float x) {
  const int32_t k = (int32_t)x;
  const float f = x - (float)k;
  float pl = fmaf(1.5483275463e-05f, f, 1.5669833174e-04f);
  pl = fmaf(pl, f, 1.3331825236e-03f);
  pl = fmaf(pl, f, 9.6164605538e-03f);
  pl = fmaf(pl, f, 5.5504156855e-02f);
  pl = fmaf(pl, f, 2.4022684109e-01f);
  pl = fmaf(pl, f, 6.9314717694e-01f);
  pl = fmaf(pl, f, 9.9999998955e-01f);
  const uint32_t bits = (uint32_t)(k + 127) << 23;
  float p2;
  memcpy(&p2, &bits, sizeof p2);
  return pl * p2;
}

/* gelu8 (host_kernels.hpp:322-352; gelu_cpu bert_encoder.cpp:532-580):
 * max(v,0) + P(min(|v|,4)), degree-8 Horner with fused multiply-adds. */
static inline float gelu8_ref(float v) {
  const float u = fminf(fabsf(v), 4.0f);
  float pl = fmaf(-7.2340282171e-05f, u, 1.8179518005e-03f);
  pl = fmaf(pl, u, -1.7707383379e-02f);
  pl = fmaf(pl, u, 8.4577147641e-02f);
  pl = fmaf(pl, u, -1.9228671834e-01f);
  pl = fmaf(pl, u, 9.8431124458e-02f);
  pl = fmaf(pl, u, 3.6137852062e-01f);
  pl = fmaf(pl, u, -4.9454128936e-01f);
  pl = fmaf(pl, u, -1.3007010117e-04f);
  return (v > 0.0f ? v : 0.0f) + pl;
}

/* app::gelu_erf_exact (app_state.hpp:116-120): erf GELU in double, one
 * rounding at the end. */
static inline float gelu_erf_ref(float x) {
  const double xd = (double)x;
  return (float)(0.5 * xd * (1.0 + erf(xd * 0.70710678118654752440)));
}

/* app::to_bf16 (host_kernels.hpp:157-161): round-to-nearest-even. */
static inline uint16_t to_bf16_ref(float x) {
  uint32_t u;
  memcpy(&u, &x, sizeof u);
  return (uint16_t)((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}

/* ---- GEMM: hostconv::gemm_nt (conv_host.hpp:150-181) ---------------------
 * C[M,N] = A[M,K] . B[K,N] + bias.  Per output element the products are
 * accumulated in k order (the k-outer, n-inner axpy) and the bias is added
 * last. */
typedef struct {
  const float *A, *B, *bias;
  float *C;
  int64_t K, N;
} gemm_ctx;

static void gemm_rows(void *p, int64_t lo, int64_t hi) {
  const gemm_ctx *g = (const gemm_ctx *)p;
  const int64_t K = g->K, N = g->N;
  float *acc = (float *)malloc((size_t)N * sizeof(float));
  for (int64_t r = lo; r < hi; ++r) {
    memset(acc, 0, (size_t)N * sizeof(float));
    const float *a = g->A + r * K;
    for (int64_t k = 0; k < K; ++k) {
      const float av = a[k];
      const float *brow = g->B + k * N;
      for (int64_t n = 0; n < N; ++n) acc[n] = fmaf(av, brow[n], acc[n]);
    }
    float *crow = g->C + r * N;
    for (int64_t n = 0; n < N; ++n) crow[n] = acc[n] + g->bias[n];
  }
  free(acc);
}

void nebw_oracle_gemm_nt(const float *A, int64_t M, const float *B, int64_t K,
                         int64_t N, const float *bias, float *C,
                         int32_t threads) {
  gemm_ctx g = {A, B, bias, C, K, N};
  parallel_for(M, threads, gemm_rows, &g);
}

/* ---- LayerNorm: layer_norm_cpu, AVX2 branch (bert_encoder.cpp:416-463) ---
 * Eight-lane partial sums of x, mean = hsum/H; eight-lane fma sums of
 * (x-mean)^2, var = hsum/H (biased); y = fma((x-mean)*is, g, b) with
 * is = 1/sqrt(var + eps). */
static void ln_row(float *row, int64_t H, const float *g, const float *b,
                   float eps) {
  float s[8] = {0};
  for (int64_t j = 0; j < H; j += 8)
    for (int l = 0; l < 8; ++l) s[l] = s[l] + row[j + l];
  const float mean = hsum8(s) / (float)H;
  float v[8] = {0};
  for (int64_t j = 0; j < H; j += 8)
    for (int l = 0; l < 8; ++l) {
      const float d = row[j + l] - mean;
      v[l] = fmaf(d, d, v[l]);
    }
  const float var = hsum8(v) / (float)H;
  const float is = 1.0f / sqrtf(var + eps);
  for (int64_t j = 0; j < H; ++j) {
    const float d = row[j] - mean;
    row[j] = fmaf(d * is, g[j], b[j]);
  }
}

typedef struct {
  float *x;
  int64_t H;
  const float *g, *b;
  float eps;
} ln_ctx;

static void ln_rows(void *p, int64_t lo, int64_t hi) {
  const ln_ctx *c = (const ln_ctx *)p;
  for (int64_t r = lo; r < hi; ++r) ln_row(c->x + r * c->H, c->H, c->g, c->b, c->eps);
}

void nebw_oracle_layer_norm(float *x, int64_t rows, int64_t hidden,
                            const float *g, const float *b, float eps) {
  ln_ctx c = {x, hidden, g, b, eps};
  ln_rows(&c, 0, rows);
}

/* ---- attention: qk_impl / softmax_cpu / av_impl, AVX2 branches -----------
 * (bert_encoder.cpp:995-1135, :481-530).  Scores are not scaled: the packer
 * folded 1/sqrt(head_dim) into Q (pack_npue.py:2742-2750). */
typedef struct {
  const float *qkv;
  const float *add_mask; /* [batch, seq] of 0 / -1e30 */
  float *ctx;
  int64_t seq, H, heads, hd;
} attn_ctx;

static void attn_pairs(void *p, int64_t lo, int64_t hi) {
  const attn_ctx *a = (const attn_ctx *)p;
  const int64_t S = a->seq, H = a->H, hd = a->hd, nv = hd / 8;
  float *sc = (float *)malloc((size_t)S * sizeof(float));
  for (int64_t pr = lo; pr < hi; ++pr) {
    const int64_t b = pr / a->heads, h = pr % a->heads;
    const float *mk = a->add_mask + b * S;
    for (int64_t i = 0; i < S; ++i) {
      const float *q = a->qkv + (b * S + i) * 3 * H + h * hd;
      /* qk_impl: lane l holds q[l]*k[l] + sum_v q[8v+l]*k[8v+l] (fma). */
      for (int64_t j = 0; j < S; ++j) {
        const float *k = a->qkv + (b * S + j) * 3 * H + H + h * hd;
        float s[8];
        for (int l = 0; l < 8; ++l) s[l] = q[l] * k[l];
        for (int64_t v = 1; v < nv; ++v)
          for (int l = 0; l < 8; ++l) s[l] = fmaf(q[8 * v + l], k[8 * v + l], s[l]);
        sc[j] = hsum8(s);
      }
      /* softmax_cpu: add mask, row max, exp2((x-max)*log2e floored at -120),
       * eight-lane sum, multiply by 1/sum. */
      for (int64_t j = 0; j < S; ++j) sc[j] += mk[j];
      float mx = sc[0];
      for (int64_t j = 1; j < S; ++j) mx = sc[j] > mx ? sc[j] : mx;
      float sum[8] = {0};
      for (int64_t j = 0; j < S; j += 8)
        for (int l = 0; l < 8; ++l) {
          float t = (sc[j + l] - mx) * 1.4426950408889634f;
          t = t > -120.0f ? t : -120.0f;
          const float e = exp2_ref(t);
          sc[j + l] = e;
          sum[l] = sum[l] + e;
        }
      const float inv = 1.0f / hsum8(sum);
      for (int64_t j = 0; j < S; ++j) sc[j] = sc[j] * inv;
      /* av_impl: per output element, fma over j in order. */
      float *o = a->ctx + (b * S + i) * H + h * hd;
      for (int64_t d = 0; d < hd; ++d) o[d] = 0.0f;
      for (int64_t j = 0; j < S; ++j) {
        const float *v = a->qkv + (b * S + j) * 3 * H + 2 * H + h * hd;
        const float pj = sc[j];
        for (int64_t d = 0; d < hd; ++d) o[d] = fmaf(pj, v[d], o[d]);
      }
    }
  }
  free(sc);
}

/* ---- pooling: app::pool_rows (app_state.hpp:335-374) -------------------- */
int nebw_oracle_pool_rows(const float *h, const float *am, int64_t take,
                          int64_t seq, int64_t hidden, int32_t cls, int32_t l2,
                          float *out) {
  double *acc = (double *)malloc((size_t)hidden * sizeof(double));
  for (int64_t b = 0; b < take; ++b) {
    const float *amb = am + b * seq;
    const float *hb = h + b * seq * hidden;
    if (cls) {
      if (amb[0] == 0.f) {
        free(acc);
        return fail("CLS pooling on a sequence whose first token is masked");
      }
      for (int64_t c = 0; c < hidden; ++c) acc[c] = hb[c];
    } else {
      float denom = 0.f;
      for (int64_t s = 0; s < seq; ++s) denom += amb[s];
      denom = denom > 1e-9f ? denom : 1e-9f;
      for (int64_t c = 0; c < hidden; ++c) acc[c] = 0.0;
      for (int64_t s = 0; s < seq; ++s) {
        const float m = amb[s];
        if (m == 0.f) continue;
        const float *hr = hb + s * hidden;
        for (int64_t c = 0; c < hidden; ++c) acc[c] += hr[c] * m;
      }
      for (int64_t c = 0; c < hidden; ++c) acc[c] /= denom;
    }
    float *o = out + b * hidden;
    if (l2) {
      double nrm = 0.0;
      for (int64_t c = 0; c < hidden; ++c) nrm += acc[c] * acc[c];
      nrm = sqrt(nrm > 1e-24 ? nrm : 1e-24);
      for (int64_t c = 0; c < hidden; ++c) o[c] = (float)(acc[c] / nrm);
    } else {
      for (int64_t c = 0; c < hidden; ++c) o[c] = (float)acc[c];
    }
  }
  free(acc);
  return 0;
}

/* ---- elementwise passes --------------------------------------------------- */
typedef struct {
  float *x;
  int erf;
} act_ctx;

static void act_range(void *p, int64_t lo, int64_t hi) {
  const act_ctx *c = (const act_ctx *)p;
  if (c->erf)
    for (int64_t i = lo; i < hi; ++i) c->x[i] = gelu_erf_ref(c->x[i]);
  else
    for (int64_t i = lo; i < hi; ++i) c->x[i] = gelu8_ref(c->x[i]);
}

void nebw_oracle_gelu8(float *x, int64_t n) {
  act_ctx c = {x, 0};
  act_range(&c, 0, n);
}

void nebw_oracle_exp2(float *x, int64_t n) {
  for (int64_t i = 0; i < n; ++i) x[i] = exp2_ref(x[i]);
}

void nebw_oracle_to_bf16(const float *x, uint16_t *out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = to_bf16_ref(x[i]);
}

/* swiglu_cpu (bert_encoder.cpp:582-627), the AVX2 form every width that is
 * a multiple of 8 takes: SiLU = x / (1 + exp2(max(-x * log2e, -120))) with
 * the reference's exp2 polynomial, or the exact erf GELU in double; out[j] =
 * up[j] * act(gate[j]) over rows of [up | gate]. */
typedef struct {
  const float *in;
  float *out;
  int64_t F;
  int32_t gated;
} glu_ctx;

static void glu_rows(void *p, int64_t lo, int64_t hi) {
  const glu_ctx *c = (const glu_ctx *)p;
  for (int64_t r = lo; r < hi; ++r) {
    const float *up = c->in + r * 2 * c->F, *gate = up + c->F;
    float *dst = c->out + r * c->F;
    for (int64_t j = 0; j < c->F; ++j) {
      const float xv = gate[j];
      float act;
      if (c->gated == 2) {
        act = gelu_erf_ref(xv);
      } else {
        float a = (0.0f - xv) * 1.4426950408889634f;
        if (a < -120.0f) a = -120.0f;
        act = xv / (1.0f + exp2_ref(a));
      }
      dst[j] = up[j] * act;
    }
  }
}

/* apply_rope_qkv (bert_encoder.cpp:926-993): tables cos/sin [S, d] from
 * angle s * inv_freq[j] in double rounded to float, the same value in
 * columns j and j + d/2; each head of Q and K rotated pairwise.  The
 * reference's AVX2 rotation, as its own build (g++ -O2 -march=x86-64-v3)
 * compiles it, fuses the second product of each line into the sum:
 *   o1 = fma(-x2, s, x1 c),  o2 = fma(x1, s, x2 c)
 * (measured: an intrinsic form of that shape, built with those flags, gives
 * exactly these values; pinned against oracle/_ref by the tests). */
typedef struct {
  float *qkv;
  const float *cs, *sn;
  int64_t S, H, heads, hd;
} rope_ctx;

static void rope_rows(void *p, int64_t lo, int64_t hi) {
  const rope_ctx *c = (const rope_ctx *)p;
  const int64_t half = c->hd / 2;
  for (int64_t row = lo; row < hi; ++row) {
    const int64_t s = row % c->S;
    const float *cs = c->cs + s * c->hd, *sn = c->sn + s * c->hd;
    float *base = c->qkv + row * 3 * c->H;
    for (int64_t h = 0; h < c->heads; ++h)
      for (int qk = 0; qk < 2; ++qk) {
        float *v = base + qk * c->H + h * c->hd;
        for (int64_t d = 0; d < half; ++d) {
          const float x1 = v[d], x2 = v[d + half];
          v[d] = fmaf(-x2, sn[d], x1 * cs[d]);
          v[d + half] = fmaf(x1, sn[d], x2 * cs[d]);
        }
      }
  }
}

/* ---- the encoder: BertEncoder::run (bert_encoder.cpp:1419-1598) ----------
 * host_ln/host_sm/host_gelu, no --npu-ops:
 *   x = LN(emb)
 *   per layer: residual = x; qkv = gemm(x); ctx = attention(qkv)
 *              proj = gemm(ctx); x = proj + residual; x = LN1(x); residual = x
 *              up = gelu(gemm(x)); down = gemm(up); x = down + residual;
 *              x = LN2(x) */
int nebw_oracle_encode(const nebw_oracle_model *m, const int32_t *ids,
                       const int32_t *mask, int32_t batch, int32_t seq,
                       int32_t threads, float *out, float *hidden_out) {
  const int64_t H = m->hidden, F = m->ffn, S = seq, B = batch;
  const int64_t rows = B * S;
  if (seq <= 0 || seq % 8) return fail("seq must be positive and a multiple of 8");
  if (H % 8 || m->head_dim % 8 || m->head_dim * m->heads != H)
    return fail("hidden/head_dim geometry refused (multiples of 8, heads*head_dim == hidden)");

  float *x = (float *)malloc((size_t)rows * H * sizeof(float));
  float *res = (float *)malloc((size_t)rows * H * sizeof(float));
  float *qkv = (float *)malloc((size_t)rows * 3 * H * sizeof(float));
  float *ctx = (float *)malloc((size_t)rows * H * sizeof(float));
  float *tmp = (float *)malloc((size_t)rows * H * sizeof(float));
  const int64_t FW = m->gated ? 2 * F : F;
  float *up = (float *)malloc((size_t)rows * FW * sizeof(float));
  float *gl = m->gated ? (float *)malloc((size_t)rows * F * sizeof(float)) : NULL;
  float *rcs = NULL, *rsn = NULL;
  if (m->rope_inv_freq) {
    const int64_t hd = m->head_dim, half = hd / 2;
    rcs = (float *)malloc((size_t)S * hd * sizeof(float));
    rsn = (float *)malloc((size_t)S * hd * sizeof(float));
    if (rcs && rsn)
      for (int64_t s = 0; s < S; ++s)
        for (int64_t j = 0; j < half; ++j) {
          const double ang = (double)s * m->rope_inv_freq[j];
          const float cv = (float)cos(ang), sv = (float)sin(ang);
          rcs[s * hd + j] = rcs[s * hd + half + j] = cv;
          rsn[s * hd + j] = rsn[s * hd + half + j] = sv;
        }
  }
  float *amask = (float *)malloc((size_t)rows * sizeof(float));
  float *cam = (float *)malloc((size_t)rows * sizeof(float));
  if (!x || !res || !qkv || !ctx || !tmp || !up || !amask || !cam ||
      (m->gated && !gl) || (m->rope_inv_freq && (!rcs || !rsn))) {
    free(x); free(res); free(qkv); free(ctx); free(tmp); free(up); free(amask); free(cam);
    free(gl); free(rcs); free(rsn);
    return fail("out of host memory");
  }

  /* EmbedService::chunk (embed_service.cpp:29-64). */
  for (int64_t b = 0; b < B; ++b)
    for (int64_t s = 0; s < S; ++s) {
      const int32_t id = ids[b * S + s];
      const float mk = (float)mask[b * S + s];
      cam[b * S + s] = mk;
      amask[b * S + s] = mk > 0 ? 0.f : -1.0e30f;
      float *dst = x + (b * S + s) * H;
      const float *wv = m->word + (int64_t)id * H;
      const float *pv = m->pos + s * H;
      for (int64_t c = 0; c < H; ++c) dst[c] = wv[c] + pv[c] + m->typ[c];
    }

  ln_ctx lc = {x, H, m->emb_ln_g, m->emb_ln_b, m->ln_eps};
  parallel_for(rows, threads, ln_rows, &lc);

  for (int32_t L = 0; L < m->layers; ++L) {
    memcpy(res, x, (size_t)rows * H * sizeof(float));
    nebw_oracle_gemm_nt(x, rows, m->w_qkv[L], H, 3 * H, m->b_qkv[L], qkv, threads);
    if (m->rope_inv_freq) {
      rope_ctx rc = {qkv, rcs, rsn, S, H, m->heads, m->head_dim};
      parallel_for(rows, threads, rope_rows, &rc);
    }
    attn_ctx ac = {qkv, amask, ctx, S, H, m->heads, m->head_dim};
    parallel_for(B * m->heads, threads, attn_pairs, &ac);
    nebw_oracle_gemm_nt(ctx, rows, m->w_ao[L], H, H, m->b_ao[L], tmp, threads);
    for (int64_t i = 0; i < rows * H; ++i) x[i] = tmp[i] + res[i];
    lc.g = m->ln1_g[L];
    lc.b = m->ln1_b[L];
    parallel_for(rows, threads, ln_rows, &lc);
    memcpy(res, x, (size_t)rows * H * sizeof(float));
    nebw_oracle_gemm_nt(x, rows, m->w_up[L], H, FW, m->b_up[L], up, threads);
    if (m->gated) {
      glu_ctx gg = {up, gl, F, m->gated};
      parallel_for(rows, threads, glu_rows, &gg);
    } else {
      act_ctx gc = {up, m->gelu_erf};
      parallel_for(rows * F, threads, act_range, &gc);
    }
    nebw_oracle_gemm_nt(m->gated ? gl : up, rows, m->w_dn[L], F, H, m->b_dn[L], tmp, threads);
    for (int64_t i = 0; i < rows * H; ++i) x[i] = tmp[i] + res[i];
    lc.g = m->ln2_g[L];
    lc.b = m->ln2_b[L];
    parallel_for(rows, threads, ln_rows, &lc);
  }

  if (hidden_out) memcpy(hidden_out, x, (size_t)rows * H * sizeof(float));
  const int rc = nebw_oracle_pool_rows(x, cam, B, S, H, m->cls_pool, m->l2_normalize, out);
  free(x); free(res); free(qkv); free(ctx); free(tmp); free(up); free(amask); free(cam);
  free(gl); free(rcs); free(rsn);
  return rc;
}

/* ======================================================================== *
 * ViT (arch vit_patch16_prenorm_gelu): VitEncoder::run, host path
 * (runtime/src/vit/encoder.cpp:222-431) with the whisper host ops it calls
 * (runtime/src/whisper/npu_ops.cpp:449-620) and the im2col of
 * runtime/src/vit/image.cpp:732-755.
 * ======================================================================== */

/* im2col_patches (image.cpp:732-755): patch row p*n + q, column
 * (c*P + i)*P + j  <-  chw[(c*S + p*P + i)*S + q*P + j]. */
/* ---- int8 datapath: the array path of a --dtype i8 container --------------
 * Each GEMM input is quantised per row to int8 with the SmoothQuant divisor
 * folded in, the array multiplies int8 x int8 into int32, and the host
 * dequantises C with the row scale, the column scale and the bias.  The int32
 * product is exact, so these steps pin bit-exactly.  Only an int32 C (the
 * designs' c_elem_bytes 4) is restated, and N % 8 == 0 (every BERT width),
 * the widths on which the reference's AVX2 bodies cover whole rows. */

/* app::quantise_a_int8 (host_kernels.hpp:263-315), one row:
 *   mx = max_j |x_j * ias_j|, sc = mx > 0 ? mx / 127 : 1,
 *   q_j = rne(clamp((x_j * ias_j) * (1 / sc), -127, 127)). */
static void quant_row(const float *x, int64_t K, const float *ias, int8_t *q, float *scale) {
  float mx = 0.0f;
  for (int64_t j = 0; j < K; ++j) {
    const float a = fabsf(x[j] * ias[j]);
    if (a > mx) mx = a;
  }
  const float sc = mx > 0.0f ? mx / 127.0f : 1.0f;
  *scale = sc;
  const float inv = 1.0f / sc;
  for (int64_t j = 0; j < K; ++j) {
    const float t = fminf(fmaxf((x[j] * ias[j]) * inv, -127.0f), 127.0f);
    q[j] = (int8_t)nearbyintf(t);
  }
}

void nebw_oracle_quantise_rows(const float *a, int64_t rows, int64_t K, const float *ias,
                               int8_t *q, float *scale) {
  for (int64_t r = 0; r < rows; ++r) quant_row(a + r * K, K, ias, q + r * K, scale + r);
}

typedef struct {
  const int8_t *A, *B;
  int32_t *C;
  int64_t K, N;
} gemm_i8_ctx;

static void gemm_i8_rows(void *p, int64_t lo, int64_t hi) {
  const gemm_i8_ctx *c = (const gemm_i8_ctx *)p;
  for (int64_t m = lo; m < hi; ++m) {
    int32_t *row = c->C + m * c->N;
    for (int64_t n = 0; n < c->N; ++n) row[n] = 0;
    for (int64_t k = 0; k < c->K; ++k) {
      const int32_t a = c->A[m * c->K + k];
      const int8_t *b = c->B + k * c->N;
      for (int64_t n = 0; n < c->N; ++n) row[n] += a * (int32_t)b[n];
    }
  }
}

/* The array's int8 GEMM: C[M, N] = A[M, K] . B[K, N] in int32 (exact). */
void nebw_oracle_gemm_i8(const int8_t *A, int64_t M, const int8_t *B, int64_t K, int64_t N,
                         int32_t *C, int32_t threads) {
  gemm_i8_ctx c = {A, B, C, K, N};
  parallel_for(M, threads, gemm_i8_rows, &c);
}

/* app::dequantise_c, int32 C (host_kernels.hpp:575-613): y = fma(float(c) *
 * sa[row], ws[col], bias[col]) -- the float conversion rounds to nearest even,
 * the product rounds, the multiply-add rounds once. */
static inline float dequant_one(int32_t c, float sa, float ws, float b) {
  return fmaf((float)c * sa, ws, b);
}

int nebw_oracle_dequantise(const int32_t *C, int64_t rows, int64_t N, const float *sa,
                           const float *ws, const float *bias, float *out) {
  if (N % 8) return fail("dequantise: N must be a multiple of 8");
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t j = 0; j < N; ++j)
      out[r * N + j] = dequant_one(C[r * N + j], sa[r], ws[j], bias[j]);
  return 0;
}

/* app::dequant_act_quant with the BERT FFN's GELU (host_kernels.hpp:404-526;
 * the act of bert_encoder.cpp:821-829): per row, dequantise as above, gelu8,
 * then quantise for the next GEMM with its divisor ias_next. */
int nebw_oracle_dequant_gelu_quant(const int32_t *C, int64_t rows, int64_t N, const float *sa,
                                   const float *ws, const float *bias, const float *ias_next,
                                   int8_t *q, float *sa_next) {
  if (N % 8) return fail("dequant_gelu_quant: N must be a multiple of 8");
  float *v = (float *)malloc((size_t)N * sizeof(float));
  if (!v) return fail("dequant_gelu_quant: out of memory");
  for (int64_t r = 0; r < rows; ++r) {
    for (int64_t j = 0; j < N; ++j)
      v[j] = gelu8_ref(dequant_one(C[r * N + j], sa[r], ws[j], bias[j]));
    quant_row(v, N, ias_next, q + r * N, sa_next + r);
  }
  free(v);
  return 0;
}

/* ---- int8 encoder pass: BertEncoder::run's array path -------------------
 * (bert_encoder.cpp:1419-1598 with gemm_on_array() and the fused epilogues,
 * fuse_ffn_epilogue's default; gemm()'s array branch :763-923;
 * add_norm_quant :1196-1302).  Per layer:
 *   QKV  A = quantise(x, ias_qkv) on layer 0, else the rows the previous
 *        layer's add_norm_quant wrote; C = A.W; qkv = dequantise(C) (fp32)
 *   attention on the host (qk_impl / softmax_cpu / av_impl) -> ctx
 *   AO   A = quantise(ctx, ias_ao); proj = dequantise(A.W)
 *   x = LN1(proj + residual); residual = x; A = quantise(x, ias_up)
 *   UP   A' = dequant_act_quant(A.W): gelu8, quantised with ias_dn
 *   DOWN down = dequantise(A'.W)
 *   x = LN2(down + residual); residual = x; A = quantise(x, ias_qkv of the
 *        next layer) unless this is the last
 * add_norm_quant's LayerNorm is layer_norm_cpu's arithmetic (ln_row), its
 * quantisation quantise_a_int8's (quant_row). */
int nebw_oracle_encode_i8(const nebw_oracle_model *m, const nebw_oracle_i8_gemm *gq,
                          const nebw_oracle_i8_gemm *ga, const nebw_oracle_i8_gemm *gu,
                          const nebw_oracle_i8_gemm *gd, const int32_t *ids,
                          const int32_t *mask, int32_t batch, int32_t seq, int32_t threads,
                          float *out, float *hidden_out) {
  const int64_t H = m->hidden, F = m->ffn, S = seq, B = batch;
  const int64_t rows = B * S;
  if (seq <= 0 || seq % 8) return fail("seq must be positive and a multiple of 8");
  if (H % 8 || F % 8 || m->head_dim % 8 || m->head_dim * m->heads != H)
    return fail("hidden/ffn/head_dim geometry refused (multiples of 8, heads*head_dim == hidden)");
  if (m->gated || m->rope_inv_freq) return fail("the int8 pass restates plain BERT only");
  const int64_t KM = F > H ? F : H, NM = 3 * H > F ? 3 * H : F;
  float *x = (float *)malloc((size_t)rows * H * sizeof(float));
  float *res = (float *)malloc((size_t)rows * H * sizeof(float));
  float *qkv = (float *)malloc((size_t)rows * 3 * H * sizeof(float));
  float *ctx = (float *)malloc((size_t)rows * H * sizeof(float));
  float *y = (float *)malloc((size_t)rows * H * sizeof(float));
  int8_t *aq = (int8_t *)malloc((size_t)rows * KM);
  float *sa = (float *)malloc((size_t)rows * sizeof(float));
  int32_t *c = (int32_t *)malloc((size_t)rows * NM * sizeof(int32_t));
  float *amask = (float *)malloc((size_t)rows * sizeof(float));
  float *cam = (float *)malloc((size_t)rows * sizeof(float));
  int rc = 0;
  if (!x || !res || !qkv || !ctx || !y || !aq || !sa || !c || !amask || !cam) {
    rc = fail("out of host memory");
    goto done;
  }

  /* EmbedService::chunk (embed_service.cpp:29-64), then LN of the embeddings */
  for (int64_t b = 0; b < B; ++b)
    for (int64_t s2 = 0; s2 < S; ++s2) {
      const int32_t id = ids[b * S + s2];
      const float mk = (float)mask[b * S + s2];
      cam[b * S + s2] = mk;
      amask[b * S + s2] = mk > 0 ? 0.f : -1.0e30f;
      float *dst = x + (b * S + s2) * H;
      const float *wv = m->word + (int64_t)id * H;
      const float *pv = m->pos + s2 * H;
      for (int64_t j = 0; j < H; ++j) dst[j] = wv[j] + pv[j] + m->typ[j];
    }
  ln_ctx lc = {x, H, m->emb_ln_g, m->emb_ln_b, m->ln_eps};
  parallel_for(rows, threads, ln_rows, &lc);

  for (int32_t L = 0; L < m->layers; ++L) {
    if (L == 0) {
      memcpy(res, x, (size_t)rows * H * sizeof(float));
      nebw_oracle_quantise_rows(x, rows, H, gq[0].ias, aq, sa);
    }
    nebw_oracle_gemm_i8(aq, rows, gq[L].w, H, 3 * H, c, threads);
    if ((rc = nebw_oracle_dequantise(c, rows, 3 * H, sa, gq[L].ws, m->b_qkv[L], qkv))) goto done;
    attn_ctx ac = {qkv, amask, ctx, S, H, m->heads, m->head_dim};
    parallel_for(B * m->heads, threads, attn_pairs, &ac);

    nebw_oracle_quantise_rows(ctx, rows, H, ga[L].ias, aq, sa);
    nebw_oracle_gemm_i8(aq, rows, ga[L].w, H, H, c, threads);
    if ((rc = nebw_oracle_dequantise(c, rows, H, sa, ga[L].ws, m->b_ao[L], y))) goto done;
    /* add_norm_quant(x, proj, ln1, 1 / asmooth of FFN-up) */
    for (int64_t i = 0; i < rows * H; ++i) x[i] = y[i] + res[i];
    lc.g = m->ln1_g[L];
    lc.b = m->ln1_b[L];
    lc.eps = 1e-12f;
    parallel_for(rows, threads, ln_rows, &lc);
    memcpy(res, x, (size_t)rows * H * sizeof(float));
    nebw_oracle_quantise_rows(x, rows, H, gu[L].ias, aq, sa);

    nebw_oracle_gemm_i8(aq, rows, gu[L].w, H, F, c, threads);
    if ((rc = nebw_oracle_dequant_gelu_quant(c, rows, F, sa, gu[L].ws, m->b_up[L], gd[L].ias, aq,
                                             sa)))
      goto done;
    nebw_oracle_gemm_i8(aq, rows, gd[L].w, F, H, c, threads);
    if ((rc = nebw_oracle_dequantise(c, rows, H, sa, gd[L].ws, m->b_dn[L], y))) goto done;
    /* add_norm_quant(x, down, ln2, 1 / asmooth of the next QKV, or none) */
    for (int64_t i = 0; i < rows * H; ++i) x[i] = y[i] + res[i];
    lc.g = m->ln2_g[L];
    lc.b = m->ln2_b[L];
    parallel_for(rows, threads, ln_rows, &lc);
    memcpy(res, x, (size_t)rows * H * sizeof(float));
    if (L + 1 < m->layers) nebw_oracle_quantise_rows(x, rows, H, gq[L + 1].ias, aq, sa);
  }

  if (hidden_out) memcpy(hidden_out, x, (size_t)rows * H * sizeof(float));
  rc = nebw_oracle_pool_rows(x, cam, B, S, H, m->cls_pool, m->l2_normalize, out);
done:
  free(x); free(res); free(qkv); free(ctx); free(y); free(aq); free(sa); free(c); free(amask);
  free(cam);
  return rc;
}

void nebw_oracle_vit_im2col(const float *chw, int32_t channels, int32_t image,
                            int32_t patch, float *out) {
  const int64_t n = image / patch, pd = (int64_t)channels * patch * patch;
  for (int64_t p = 0; p < n; ++p)
    for (int64_t q = 0; q < n; ++q) {
      float *dst = out + (p * n + q) * pd;
      for (int64_t c = 0; c < channels; ++c)
        for (int64_t i = 0; i < patch; ++i)
          for (int64_t j = 0; j < patch; ++j)
            dst[(c * patch + i) * patch + j] =
                chw[(c * image + p * patch + i) * image + q * patch + j];
    }
}

/* layernorm_rows (npu_ops.cpp:449-468): mean and variance summed in double
 * in row order; y = ((x - mean) * is) * gamma + beta with is =
 * 1/sqrt(var + eps) in float (the reference build contracts the last
 * multiply-add into one fused operation). */
static void ln_row_vit(float *row, int64_t d, const float *g, const float *b,
                       float eps) {
  double sm = 0.0;
  for (int64_t j = 0; j < d; ++j) sm += row[j];
  const float mean = (float)(sm / (double)d);
  double sv = 0.0;
  for (int64_t j = 0; j < d; ++j) {
    const double dd = (double)row[j] - (double)mean;
    sv = fma(dd, dd, sv);
  }
  const float var = (float)(sv / (double)d);
  const float is = 1.0f / sqrtf(var + eps);
  for (int64_t j = 0; j < d; ++j) row[j] = fmaf((row[j] - mean) * is, g[j], b[j]);
}

typedef struct {
  const float *src;
  float *dst;
  int64_t d;
  const float *g, *b;
  float eps;
} ln_vit_ctx;

static void ln_vit_rows(void *p, int64_t lo, int64_t hi) {
  const ln_vit_ctx *c = (const ln_vit_ctx *)p;
  for (int64_t r = lo; r < hi; ++r) {
    float *row = c->dst + r * c->d;
    if (c->src != c->dst) memcpy(row, c->src + r * c->d, (size_t)c->d * sizeof(float));
    ln_row_vit(row, c->d, c->g, c->b, c->eps);
  }
}

/* whisper attention, no softmax operator (npu_ops.cpp:478-600): per (query
 * i, head h) scores q.k (eight-lane fused partial sums, hsum256) times the
 * scale, softmax with the row max subtracted and std::exp, sum in key order,
 * inverse sum; ctx = sum_j (p_j * inv) * v_j with fused multiply-adds. */
typedef struct {
  const float *qkv;
  float *ctx;
  int64_t n_pos, H, heads, hd;
  float scale;
} vit_attn_ctx;

static void vit_attn_pairs(void *p, int64_t lo, int64_t hi) {
  const vit_attn_ctx *a = (const vit_attn_ctx *)p;
  const int64_t S = a->n_pos, H = a->H, hd = a->hd, nv = hd / 8;
  float *sc = (float *)malloc((size_t)S * sizeof(float));
  for (int64_t pr = lo; pr < hi; ++pr) {
    const int64_t img = pr / (S * a->heads), rem = pr % (S * a->heads);
    const int64_t i = rem / a->heads, h = rem % a->heads;
    const float *base = a->qkv + img * S * 3 * H;
    const float *q = base + i * 3 * H + h * hd;
    for (int64_t j = 0; j < S; ++j) {
      const float *k = base + j * 3 * H + H + h * hd;
      float s[8];
      for (int l = 0; l < 8; ++l) s[l] = q[l] * k[l];
      for (int64_t v = 1; v < nv; ++v)
        for (int l = 0; l < 8; ++l) s[l] = fmaf(q[8 * v + l], k[8 * v + l], s[l]);
      sc[j] = hsum8(s) * a->scale;
    }
    float mx = sc[0];
    for (int64_t j = 1; j < S; ++j) mx = sc[j] > mx ? sc[j] : mx;
    float sum = 0.f;
    for (int64_t j = 0; j < S; ++j) {
      sc[j] = expf(sc[j] - mx);
      sum += sc[j];
    }
    const float inv = sum > 0.f ? 1.0f / sum : 0.f;
    float *o = a->ctx + (img * S + i) * H + h * hd;
    for (int64_t d = 0; d < hd; ++d) o[d] = 0.0f;
    for (int64_t j = 0; j < S; ++j) {
      const float w = sc[j] * inv;
      const float *v = base + j * 3 * H + 2 * H + h * hd;
      for (int64_t d = 0; d < hd; ++d) o[d] = fmaf(w, v[d], o[d]);
    }
  }
  free(sc);
}

/* VitEncoder::run (encoder.cpp:222-431), image by image:
 *   patches = im2col(image); pe = gemm(patches, patch_embed) + bias
 *   x[0] = cls + pos[0]; x[1+p] = pe[p] + pos[1+p]
 *   per layer: x += attn_out(attention(qkv(LN1(x))))
 *              x += ffn_down(gelu_erf(ffn_up(LN2(x))))
 *   x = LN_final(x); the CLS row is x[0]. */
int nebw_oracle_vit_encode(const nebw_oracle_vit *m, const float *images, int32_t n_images,
                           int32_t threads, float *cls_out, float *hidden_out) {
  const int64_t H = m->hidden, F = m->ffn, P = m->patch_size, C = m->channels;
  const int64_t side = m->image_size / P, np = side * side, S = np + 1, pd = C * P * P;
  if (m->image_size % P || pd != H)
    return fail("ViT geometry refused: image_size % patch and channels*patch^2 == hidden");
  if (H % 8 || m->head_dim % 8 || m->head_dim * m->heads != H)
    return fail("ViT head geometry refused (multiples of 8, heads*head_dim == hidden)");
  const int64_t rows = (int64_t)n_images * S;
  float *x = (float *)malloc((size_t)rows * H * sizeof(float));
  float *nrm = (float *)malloc((size_t)rows * H * sizeof(float));
  float *qkv = (float *)malloc((size_t)rows * 3 * H * sizeof(float));
  float *ctx = (float *)malloc((size_t)rows * H * sizeof(float));
  float *tmp = (float *)malloc((size_t)rows * H * sizeof(float));
  float *up = (float *)malloc((size_t)rows * F * sizeof(float));
  float *pat = (float *)malloc((size_t)np * pd * sizeof(float));
  float *pe = (float *)malloc((size_t)np * H * sizeof(float));
  if (!x || !nrm || !qkv || !ctx || !tmp || !up || !pat || !pe) {
    free(x); free(nrm); free(qkv); free(ctx); free(tmp); free(up); free(pat); free(pe);
    return fail("out of host memory");
  }
  for (int64_t img = 0; img < n_images; ++img) {
    nebw_oracle_vit_im2col(images + img * C * m->image_size * m->image_size, (int32_t)C,
                           m->image_size, (int32_t)P, pat);
    nebw_oracle_gemm_nt(pat, np, m->patch_w, pd, H, m->patch_b, pe, threads);
    float *xi = x + img * S * H;
    for (int64_t c = 0; c < H; ++c) xi[c] = m->cls[c];
    memcpy(xi + H, pe, (size_t)np * H * sizeof(float));
    for (int64_t t = 0; t < S; ++t)
      for (int64_t c = 0; c < H; ++c) xi[t * H + c] += m->pos[t * H + c];
  }
  for (int32_t L = 0; L < m->layers; ++L) {
    ln_vit_ctx lc = {x, nrm, H, m->ln1_g[L], m->ln1_b[L], m->ln_eps};
    parallel_for(rows, threads, ln_vit_rows, &lc);
    nebw_oracle_gemm_nt(nrm, rows, m->w_qkv[L], H, 3 * H, m->b_qkv[L], qkv, threads);
    vit_attn_ctx ac = {qkv, ctx, S, H, m->heads, m->head_dim, m->attn_scale};
    parallel_for(rows * m->heads, threads, vit_attn_pairs, &ac);
    nebw_oracle_gemm_nt(ctx, rows, m->w_ao[L], H, H, m->b_ao[L], tmp, threads);
    for (int64_t i = 0; i < rows * H; ++i) x[i] += tmp[i];
    lc.g = m->ln2_g[L];
    lc.b = m->ln2_b[L];
    parallel_for(rows, threads, ln_vit_rows, &lc);
    nebw_oracle_gemm_nt(nrm, rows, m->w_up[L], H, F, m->b_up[L], up, threads);
    act_ctx gc = {up, 1};
    parallel_for(rows * F, threads, act_range, &gc);
    nebw_oracle_gemm_nt(up, rows, m->w_dn[L], F, H, m->b_dn[L], tmp, threads);
    for (int64_t i = 0; i < rows * H; ++i) x[i] += tmp[i];
  }
  ln_vit_ctx lf = {x, x, H, m->lnf_g, m->lnf_b, m->ln_eps};
  parallel_for(rows, threads, ln_vit_rows, &lf);
  for (int64_t img = 0; img < n_images; ++img)
    memcpy(cls_out + img * H, x + img * S * H, (size_t)H * sizeof(float));
  if (hidden_out) memcpy(hidden_out, x, (size_t)rows * H * sizeof(float));
  free(x); free(nrm); free(qkv); free(ctx); free(tmp); free(up); free(pat); free(pe);
  return 0;
}
