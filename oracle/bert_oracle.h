/* TEST INFRASTRUCTURE ONLY -- the parity oracle, never shipped.
 *
 * A plain-C restatement of the reference's host-CPU BERT encoder path
 * (runtime/src/encoders/bert_encoder.cpp:1419-1598 with --npu-ops empty) and
 * of its pooling (runtime/include/common/app_state.hpp:335-374).  It exists so
 * that the GPU build can be checked where the reference tree is absent (the
 * GPU box); it is itself pinned against the reference compiled from source
 * (oracle/_ref, tests/test_oracle_pin.py) and against committed golden
 * vectors made by that compiled reference (tests/golden/).
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
 * load this library.
 */
#ifndef NEBW_BERT_ORACLE_H
#define NEBW_BERT_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Weights in the reference container's layout (tools/pack/pack_npue.py
 * BERT branch :2684-2790): GEMM operands fp32 row-major [K, N] with Q|K|V
 * fused along N and 1/sqrt(head_dim) already folded into the Q columns;
 * biases and LayerNorm parameters fp32. */
typedef struct nebw_oracle_model {
  int32_t layers, hidden, heads, head_dim, ffn;
  int32_t cls_pool;      /* 1: CLS row, 0: masked mean                       */
  int32_t l2_normalize;  /* 1: L2-normalise the pooled vector                */
  int32_t gelu_erf;      /* 0: gelu8 polynomial (the BERT host path);
                            1: exact erf GELU in double (app::gelu_erf_exact) */
  float ln_eps;          /* the BERT host path hard-codes 1e-12              */
  const float *word, *pos, *typ, *emb_ln_g, *emb_ln_b;
  /* per layer, arrays of `layers` pointers */
  const float *const *w_qkv, *const *b_qkv;   /* [H, 3H], [3H] */
  const float *const *w_ao, *const *b_ao;     /* [H, H],  [H]  */
  const float *const *ln1_g, *const *ln1_b;   /* [H]           */
  const float *const *w_up, *const *b_up;     /* [H, F],  [F]  */
  const float *const *w_dn, *const *b_dn;     /* [F, H],  [H]  */
  const float *const *ln2_g, *const *ln2_b;   /* [H]           */
  /* The gated / rotary families (arch nomic_bert_rope_swiglu,
   * gte_new_rope_geglu): gated 0 = plain FFN, 1 = up * SiLU(gate), 2 = up *
   * erf-GELU(gate) over a w_up of [H, 2F] = [up | gate] (swiglu_cpu,
   * bert_encoder.cpp:582-627); rope_inv_freq non-NULL: head_dim/2 rotary
   * frequencies applied to Q and K after the QKV GEMM (apply_rope_qkv,
   * bert_encoder.cpp:926-993). */
  int32_t gated;
  const double *rope_inv_freq;
} nebw_oracle_model;

/* Encode `batch` padded sequences of `seq` token ids.
 *   ids [batch, seq] int32, mask [batch, seq] int32 1/0
 *   out [batch, hidden] fp32; hidden_out optional [batch*seq, hidden].
 * seq must be a multiple of 8 and hidden a multiple of 8 (the reference's
 * set_design_seq / set_model_shape refusals).  Returns 0, or a nonzero code
 * with a message available from nebw_oracle_last_error(). */
int nebw_oracle_encode(const nebw_oracle_model *m, const int32_t *ids,
                       const int32_t *mask, int32_t batch, int32_t seq,
                       int32_t threads, float *out, float *hidden_out);

/* Single ops, exposed so each can be pinned against the reference. */
void nebw_oracle_gemm_nt(const float *A, int64_t M, const float *B, int64_t K,
                         int64_t N, const float *bias, float *C,
                         int32_t threads);
void nebw_oracle_gelu8(float *x, int64_t n);
void nebw_oracle_exp2(float *x, int64_t n);
void nebw_oracle_to_bf16(const float *x, uint16_t *out, int64_t n);
void nebw_oracle_layer_norm(float *x, int64_t rows, int64_t hidden,
                            const float *g, const float *b, float eps);
int nebw_oracle_pool_rows(const float *h, const float *am, int64_t take,
                          int64_t seq, int64_t hidden, int32_t cls, int32_t l2,
                          float *out);
const char *nebw_oracle_last_error(void);

/* The int8 datapath of a --dtype i8 container (the array's quantised
 * operands): per-row quantisation with the SmoothQuant divisor (ias =
 * 1/asmooth), the exact int32 GEMM, dequantisation, and the FFN-up epilogue
 * that dequantises, applies gelu8 and quantises for FFN-down.  int32 C only;
 * N % 8 == 0. */
void nebw_oracle_quantise_rows(const float *a, int64_t rows, int64_t K, const float *ias,
                               int8_t *q, float *scale);
void nebw_oracle_gemm_i8(const int8_t *A, int64_t M, const int8_t *B, int64_t K, int64_t N,
                         int32_t *C, int32_t threads);
int nebw_oracle_dequantise(const int32_t *C, int64_t rows, int64_t N, const float *sa,
                           const float *ws, const float *bias, float *out);
int nebw_oracle_dequant_gelu_quant(const int32_t *C, int64_t rows, int64_t N, const float *sa,
                                   const float *ws, const float *bias, const float *ias_next,
                                   int8_t *q, float *sa_next);

/* ViT (arch vit_patch16_prenorm_gelu): pre-LN encoder over image patches. */
/* One GEMM of an int8 container on the array path: the int8 operand [K, N]
 * (the panel untiled), its column scales (.wscale) and the reciprocal of its
 * SmoothQuant divisor (1 / .asmooth, as the encoder computes it). */
typedef struct nebw_oracle_i8_gemm {
  const int8_t *w;    /* [K, N] */
  const float *ws;    /* [N]    */
  const float *ias;   /* [K]    */
} nebw_oracle_i8_gemm;

/* BertEncoder::run's array path for an int8 container (every GEMM on the
 * array, the fused host epilogues).  `m` supplies the geometry, embeddings,
 * biases and LayerNorm parameters (its fp32 GEMM operands are not read);
 * qkv / ao / up / dn hold `layers` operands each.  Plain BERT only (m->gated
 * 0, no rotary). */
int nebw_oracle_encode_i8(const nebw_oracle_model *m, const nebw_oracle_i8_gemm *qkv,
                          const nebw_oracle_i8_gemm *ao, const nebw_oracle_i8_gemm *up,
                          const nebw_oracle_i8_gemm *dn, const int32_t *ids,
                          const int32_t *mask, int32_t batch, int32_t seq, int32_t threads,
                          float *out, float *hidden_out);

typedef struct nebw_oracle_vit {
  int32_t layers, hidden, heads, head_dim, ffn;
  int32_t image_size, patch_size, channels;  /* hidden == channels*patch^2 */
  float ln_eps;
  float attn_scale;  /* 1 when 1/sqrt(head_dim) is folded into the Q operand */
  const float *patch_w, *patch_b;            /* [C*P*P, H], [H]          */
  const float *cls, *pos;                    /* [H], [n_patches + 1, H]  */
  const float *lnf_g, *lnf_b;                /* final LayerNorm          */
  const float *const *w_qkv, *const *b_qkv;
  const float *const *w_ao, *const *b_ao;
  const float *const *ln1_g, *const *ln1_b;
  const float *const *w_up, *const *b_up;
  const float *const *w_dn, *const *b_dn;
  const float *const *ln2_g, *const *ln2_b;
} nebw_oracle_vit;

/* images [n, C, S, S] fp32 (normalised pixels) -> cls_out [n, H] (the CLS
 * row after the final LayerNorm); hidden_out [n, n_pos, H] or NULL. */
int nebw_oracle_vit_encode(const nebw_oracle_vit *m, const float *images, int32_t n_images,
                           int32_t threads, float *cls_out, float *hidden_out);
void nebw_oracle_vit_im2col(const float *chw, int32_t channels, int32_t image,
                            int32_t patch, float *out);

#ifdef __cplusplus
}
#endif
#endif
