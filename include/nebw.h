/* nebw -- the B200 (sm_100a) BERT-encoder library behind a plain C ABI.
 *
 * This is the device side of the reference's embedding runtime, rebuilt for
 * the GPU: everything the reference dispatches to its NPU (or runs on the
 * host when --npu-ops is empty) for a BERT-family encoder pass.  The entry
 * points are the ones the reference's op funnels would bind; each comment
 * names the reference interface it replaces (paths inside the reference
 * project).
 *
 * Conventions
 *   - Every function returns 0 (NEBW_OK) or a nebw_status; the message for
 *     the calling thread's last failure is nebw_last_error().  Nothing falls
 *     back to the CPU: a missing device, a refused shape or a device-side
 *     fault is an error by name (the reference's "fail loudly" rule,
 *     README.md:2111-2140).
 *   - Pointers named *_dev / documented "device" are CUDA device pointers;
 *     "host" pointers are ordinary memory.  `stream` is a cudaStream_t passed
 *     as void*: NULL means the device handle's own stream, so a caller that
 *     wants the legacy default stream passes cudaStreamLegacy ((void*)0x1).
 *   - One nebw_dev per GPU.  Calls on different nebw_dev handles may run
 *     concurrently from different host threads; calls on one handle must not
 *     overlap.  Staged weights are immutable after staging.
 */
#ifndef NEBW_H
#define NEBW_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NEBW_ABI_VERSION 5

typedef enum nebw_status {
  NEBW_OK = 0,
  NEBW_EINVAL = 1,   /* an argument or shape is refused                     */
  NEBW_ECUDA = 2,    /* a CUDA runtime call failed (message names it)       */
  NEBW_ENOMEM = 3,   /* device or pinned-host allocation failed             */
  NEBW_ESTATE = 4,   /* the object is not in a state to do this (e.g. a
                        model with unstaged tensors)                         */
  NEBW_EDEVICE = 5,  /* a kernel reported an error (bad token id, bad
                        length, a bounded wait that timed out)              */
  NEBW_EIO = 6,      /* a container file could not be read or is malformed */
  NEBW_ECOMM = 7     /* NCCL is missing, or a collective failed or did not
                        finish within the communicator's timeout (the
                        communicator is then aborted)                      */
} nebw_status;

enum { NEBW_F32 = 0, NEBW_BF16 = 1 };
enum { NEBW_ACT_NONE = 0, NEBW_ACT_GELU8 = 1, NEBW_ACT_GELU_ERF = 2 };
/* The activation of a gated FFN's gate half (GatedAct, app_state.hpp:109):
 * SiLU ("silu", nomic_bert_rope_swiglu) or exact-erf GELU ("gelu",
 * gte_new_rope_geglu). */
enum { NEBW_GATE_SILU = 0, NEBW_GATE_GELU_ERF = 1 };
enum { NEBW_POOL_MEAN = 0, NEBW_POOL_CLS = 1 };

typedef struct nebw_dev nebw_dev;
typedef struct nebw_model nebw_model;

/* Message of the calling thread's last failure ("" if none). */
const char *nebw_last_error(void);
int nebw_abi_version(void);

/* ---- device ------------------------------------------------------------
 * Replaces npu::Device (runtime/include/runtime/device.hpp:29-38) and the
 * XRT buffer plumbing of npu::Design (runtime/include/runtime/design.hpp:
 * 199-263).  nebw_open refuses a GPU that is not sm_100 by name. */
int nebw_open(int device, nebw_dev **out);
int nebw_close(nebw_dev *dev);
/* Wait for the handle's stream, then report (and clear) any error a kernel
 * recorded since the last check. */
int nebw_sync(nebw_dev *dev);
/* Self-check of the kernels' bounded waits (no counterpart in the
 * reference): one warp waits on an mbarrier that nothing arrives on, for
 * limit_ns (1 us .. 1 s) of the GPU's global timer, with no copy or
 * tensor-core product in flight.  *expired = 1 when the wait ran out as it
 * should; the kernel then has recorded the wait-timeout code in the device
 * error word, so the next nebw_sync returns NEBW_EDEVICE (and clears it).
 * Every wait of the GEMM and attention kernels takes this path, bounded at
 * 2 s, before unwinding.  Synchronous. */
int nebw_check_bounded_wait(nebw_dev *dev, int64_t limit_ns, int32_t *expired);
int nebw_alloc(nebw_dev *dev, size_t bytes, void **dptr);
int nebw_free(nebw_dev *dev, void *dptr);
int nebw_copy_h2d(nebw_dev *dev, void *dst_dev, const void *src_host, size_t bytes);
int nebw_copy_d2h(nebw_dev *dev, void *dst_host, const void *src_dev, size_t bytes);
int nebw_device_info(nebw_dev *dev, int *sm_count, int *cc_major, int *cc_minor);

/* Which attention kernel a device handle uses (no
 * counterpart in the reference, which has one host path):
 * NEBW_ATTN_TCGEN05 -- S and P.V on tcgen05 UMMA with TMEM accumulators,
 *   persistent CTAs over a longest-first work list (the default);
 * NEBW_ATTN_MMA -- flash attention on mma.sync.
 * Both give results within the same parity tolerance, at head_dim 64 and
 * 32; other head_dims are refused. */
enum { NEBW_ATTN_MMA = 0, NEBW_ATTN_TCGEN05 = 1 };
int nebw_set_attention_kernel(nebw_dev *dev, int kind);

/* ---- weights -------------------------------------------------------------
 * Replaces npu::Design::stage(arg, data, bytes) (design.hpp:199-263,
 * design.cpp:394) for a GEMM operand.  `host_kn` is the container's operand
 * layout, row-major [K, N] (tools/pack/pack_npue.py add_gemm_b_host
 * :411-428), fp32 or bf16; it is staged once as bf16 RNE [N, K] (K-major,
 * the tensor-core B layout).  K % 8 == 0 and N % 8 == 0 are required. */
int nebw_stage_weight(nebw_dev *dev, const void *host_kn, int dtype, int64_t K, int64_t N,
                      uint64_t *handle);
int nebw_release_weight(nebw_dev *dev, uint64_t handle);

/* ---- ops (device pointers, asynchronous on `stream`) ---------------------- */

/* The unified GEMM.  Replaces BertEncoder::gemm / host_gemm
 * (runtime/src/encoders/bert_encoder.cpp:714-924, bert_encoder.hpp:269-274)
 * and the gemm_rtp design set, with the elementwise passes that follow a
 * GEMM fused in:
 *   C = A . W + bias                  (hostconv::gemm_nt, conv_host.hpp:150-181)
 *   act: NEBW_ACT_GELU8 / _GELU_ERF   (gelu_cpu :532-580; gelu_erf_exact,
 *                                      app_state.hpp:116-120)
 *   residual (fp32, may alias C):     C = (A.W + bias) + residual  (add_into :1183-1194)
 *   c_dtype NEBW_BF16: RNE narrow     (kernels/narrow_f32_bf16.cc)
 * A is bf16 [M, K] device; C is [M, N] device, bf16 or fp32.  `residual`
 * requires c_dtype NEBW_F32 and act NONE; act requires NEBW_BF16. */
int nebw_gemm(nebw_dev *dev, uint64_t weight, const void *A, int64_t M, int64_t K, int64_t N,
              const float *bias, const float *residual, int act, void *C, int c_dtype,
              void *stream);

/* LayerNorm over rows of width H, in place: x = LN(x + y) (y may be NULL).
 * Replaces layer_norm / layer_norm_cpu / add_norm_bf16
 * (bert_encoder.cpp:370-463, :1304-1361; kernels/layernorm{,_rne}.cc):
 * two-pass fp32, biased variance, eps inside the square root.  y is fp32
 * (y_dtype NEBW_F32) or a bf16 GEMM output (NEBW_BF16), widened exactly;
 * x is fp32.  If a_bf16 is not NULL the normalised rows are also written as
 * bf16 RNE (the next GEMM's A).  H % 128 == 0, H <= 2048. */
int nebw_layernorm(nebw_dev *dev, float *x, const void *y, int y_dtype, const float *gamma,
                   const float *beta, float eps, int64_t rows, int64_t H, void *a_bf16,
                   void *stream);

/* Fused masked attention over packed sequences.  Replaces qk / softmax_cpu /
 * av and attention_npu (bert_encoder.cpp:481-530, :995-1181).
 *   qkv_bf16 [rows, 3H] device (Q|K|V per row, Q pre-scaled by 1/sqrt(d));
 *   rows = the buffer's row count (>= every seq_off[b] + seq_len[b]); the
 *   rows past a sequence up to its next 16-row boundary (and below rows)
 *   must hold finite values: head_dim 64 multiplies them by exactly zero
 *   seq_off [B+1], seq_len [B] int32 device: sequence b owns packed rows
 *   [seq_off[b], seq_off[b] + seq_len[b])
 *   ctx_bf16 [rows, H] device.  head_dim in {32, 64}; max_len bounds
 *   seq_len.  Runs on tcgen05 (S and P.V on the 5th-generation tensor cores)
 *   unless nebw_set_attention_kernel chose mma.sync. */
int nebw_attention(nebw_dev *dev, const void *qkv_bf16, int64_t rows, const int32_t *seq_off,
                   const int32_t *seq_len, int32_t B, int32_t max_len, int32_t heads,
                   int32_t head_dim, void *ctx_bf16, void *stream);

/* Packing scan: seq_off[0..B] = exclusive prefix sum of seq_len (device).
 * Lengths outside [1, S] are an NEBW_EDEVICE error at the next sync. */
int nebw_pack_offsets(nebw_dev *dev, const int32_t *seq_len_in, int32_t B, int32_t S,
                      int32_t *seq_len_out, int32_t *seq_off, void *stream);

/* Embedding gather + LayerNorm into packed rows.  Replaces the gather of
 * EmbedService::chunk (runtime/src/server/embed_service.cpp:29-64,
 * x = (word[id] + pos[s]) + type[0]) and the embedding LayerNorm
 * (BertEncoder::run :1429).  ids [B, S] int32 device (padded tokenizer
 * output); x fp32 [T, H] and a_bf16 [T, H] device outputs. */
int nebw_embed_ln(nebw_dev *dev, const int32_t *ids, const int32_t *seq_off,
                  const int32_t *seq_len, int32_t B, int32_t S, const float *word,
                  int32_t vocab, const float *pos, const float *typ, const float *gamma,
                  const float *beta, float eps, int32_t H, float *x, void *a_bf16,
                  void *stream);

/* Pooling + L2 normalisation.  Replaces app::pool_rows
 * (runtime/include/common/app_state.hpp:335-374): NEBW_POOL_CLS takes each
 * sequence's first packed row, NEBW_POOL_MEAN the masked mean; both
 * accumulate in double.  out fp32 [B, H] device. */
int nebw_pool_l2(nebw_dev *dev, const float *h, const int32_t *seq_off, const int32_t *seq_len,
                 int32_t B, int32_t H, int pooling, int l2, float *out, void *stream);

/* fp32 -> bf16 RNE narrow (kernels/narrow_f32_bf16.cc; app::to_bf16,
 * host_kernels.hpp:157-161). */
int nebw_narrow_bf16(nebw_dev *dev, const float *x, int64_t n, void *y_bf16, void *stream);

/* ---- the int8 datapath (the reference's --dtype i8 array path) ------------
 * The array path of an int8 container quantises each GEMM input per row,
 * multiplies int8 x int8 into int32 and dequantises C on the host
 * (host_kernels.hpp:263-614).  These run those steps on the GPU and return
 * the reference's bits (the product is exact; each floating-point step is
 * the reference's single IEEE operation). */

/* app::quantise_a_int8 (host_kernels.hpp:263-315), per row of x [rows, K]
 * fp32 with the SmoothQuant divisor ias [K]: sc = max|x * ias| / 127 (1 for
 * an all-zero row), q = rne(clamp(x * ias * (1 / sc), -127, 127)).  q int8
 * [rows, K], scale fp32 [rows]; device buffers, asynchronous. */
int nebw_quantise_rows(nebw_dev *dev, const float *x, int64_t rows, int64_t K, const float *ias,
                       int8_t *q, float *scale, void *stream);
/* An int8 GEMM operand, the container's int8 panel untiled to row-major
 * [K, N] (host), staged once as [N, K] (the tensor-core B layout).
 * K % 16 == 0, N % 8 == 0.  Released with nebw_release_weight. */
int nebw_stage_weight_i8(nebw_dev *dev, const int8_t *host_kn, int64_t K, int64_t N,
                         uint64_t *handle);
/* C = dequant(A . W) on tcgen05.mma kind::i8: A int8 [M, K] device (rows
 * quantised with scale sa [M]), int32 accumulation, then app::dequantise_c
 * (host_kernels.hpp:575-613) y = fma(float(acc) * sa[row], ws[col], bias[col])
 * (bias NULL: 0), act NEBW_ACT_GELU8 applies gelu8 after it (the FFN-up step
 * of app::dequant_act_quant, host_kernels.hpp:404-526, whose quantisation for
 * the next GEMM is then nebw_quantise_rows).  C fp32 [M, N] device; C, ws and
 * bias 16-byte aligned.  Asynchronous on `stream`. */
int nebw_gemm_i8(nebw_dev *dev, uint64_t weight, const int8_t *A, const float *sa, int64_t M,
                 int64_t K, int64_t N, const float *ws, const float *bias, int act, float *C,
                 void *stream);
/* nebw_gemm_i8 with the output type chosen: c_dtype NEBW_F32 (as above) or
 * NEBW_BF16, the dequantised value narrowed RNE (app::to_bf16,
 * host_kernels.hpp:157-161) -- the form the int8 pass feeds the tensor-core
 * attention with.  C 16-byte (F32) or 8-byte (BF16) aligned. */
int nebw_gemm_i8_ex(nebw_dev *dev, uint64_t weight, const int8_t *A, const float *sa, int64_t M,
                    int64_t K, int64_t N, const float *ws, const float *bias, int act, void *C,
                    int c_dtype, void *stream);
/* nebw_quantise_rows over bf16 rows (x_bf16 [rows, K] bf16 bits, widened
 * exactly): the attention output's quantisation for the attention-out GEMM
 * in the int8 pass. */
int nebw_quantise_rows_bf16(nebw_dev *dev, const void *x_bf16, int64_t rows, int64_t K,
                            const float *ias, int8_t *q, float *scale, void *stream);
/* BertEncoder::add_norm_quant (runtime/src/encoders/bert_encoder.cpp:
 * 1196-1302): x = LN(x + y) in place (y fp32 [rows, H], or NULL), then, when
 * q is not NULL, the normalised rows quantised for the next int8 GEMM with
 * its divisor ias [H]: the steps of nebw_quantise_rows on the rows in
 * registers.  x, y, gamma, beta, ias 16-byte aligned; H a multiple of 128
 * up to 2048. */
int nebw_layernorm_quant(nebw_dev *dev, float *x, const float *y, const float *gamma,
                         const float *beta, float eps, int64_t rows, int64_t H, const float *ias,
                         int8_t *q, float *scale, void *stream);

/* ---- the whole encoder -------------------------------------------------- */

/* Geometry a container's config carries (set_model_shape,
 * app_state.hpp:380-631). */
typedef struct nebw_config {
  int32_t num_layers;
  int32_t hidden;
  int32_t num_heads;
  int32_t head_dim;
  int32_t intermediate;
  int32_t vocab_size;
  int32_t max_seq_len;     /* position-table rows                        */
  int32_t type_vocab_size;
  int32_t pooling;         /* NEBW_POOL_MEAN / NEBW_POOL_CLS             */
  int32_t l2_normalize;    /* 0 / 1                                      */
  int32_t activation;      /* NEBW_ACT_GELU8 (the reference BERT host
                              path) or NEBW_ACT_GELU_ERF                 */
  float layer_norm_eps;    /* the reference BERT host path uses 1e-12    */
  /* The gated / rotary families (set_model_shape, app_state.hpp:440-560):
   * arch nomic_bert_rope_swiglu and gte_new_rope_geglu.  Zero for BERT. */
  int32_t gated_ffn;       /* 1: ffn_up is [hidden, 2*intermediate] = [up | gate]
                              along N and the FFN is up * act(gate)
                              (swiglu_cpu, bert_encoder.cpp:582-627)      */
  int32_t gated_act;       /* NEBW_GATE_SILU / NEBW_GATE_GELU_ERF         */
  int32_t rope;            /* 1: rotary positions on Q and K (rotate-half,
                              position 0 at each sequence's first token;
                              apply_rope_qkv, bert_encoder.cpp:926-993); a
                              position table, if set, is added as the
                              reference adds its zero placeholder         */
  int32_t reserved0;
  double rope_theta;       /* inv_freq_j = theta^(-2j / head_dim) unless
                              nebw_model_set_rope_freq gives the set      */
} nebw_config;

/* Model = npue::BertEncoder's staged state (stage_all,
 * bert_encoder.cpp:41-172) on one GPU.  Tensors are set by their container
 * names ("embeddings.word", "layer.3.qkv", "layer.3.qkv.bias", ...,
 * pack_npue.py:2684-2790); GEMM operands are [K, N] as in the container. */
int nebw_model_create(nebw_dev *dev, const nebw_config *cfg, nebw_model **out);
int nebw_model_set_tensor(nebw_model *m, const char *name, const void *host, int dtype,
                          int64_t rows, int64_t cols);
/* A GEMM operand ("layer.{i}.{qkv,attn_out,ffn_up,ffn_down}") already in the
 * device layout: bf16 bits, row-major [N, K] (K-major), as the packer's
 * gemm_layout "tma_bf16" containers store it -- uploaded as is, no
 * re-tiling.  Replaces the pre-tiled operand staging of Design::stage
 * (runtime/src/design.cpp:394) for the array's block-panel layout. */
int nebw_model_set_gemm_nk(nebw_model *m, const char *name, const uint16_t *host_bf16_nk,
                           int64_t n_rows, int64_t k_cols);
/* An int8 GEMM operand for the int8 datapath: "layer.{i}.{qkv,attn_out,
 * ffn_up,ffn_down}" as the container's int8 panel untiled to [K, N] (host),
 * its per-column scale wscale [N] (.wscale) and the activation's SmoothQuant
 * divisor asmooth [K] (.asmooth; the pass multiplies by 1 / asmooth taken in
 * float, bert_encoder.cpp:767-772).  K and N as the model's GEMM.
 * nebw_model_load_npue sets these for an int8 container. */
int nebw_model_set_int8_operand(nebw_model *m, const char *name, const int8_t *host_kn,
                                const float *wscale, const float *asmooth, int64_t K, int64_t N);
/* Which arithmetic the encoder passes run.  NEBW_DATAPATH_BF16 (the
 * default): bf16 tensor-core GEMMs over the staged operands -- for an int8
 * container, its weights dequantised, as the reference's default host path
 * multiplies them (--npu-ops empty).  NEBW_DATAPATH_I8: the reference's
 * array path for an int8 container (`--npu-ops gemm`, BertEncoder::run,
 * bert_encoder.cpp:1419-1598 with gemm()'s array branch :763-923): every
 * GEMM int8 x int8 -> int32 on tcgen05.mma kind::i8 between the reference's
 * host steps -- quantise the A rows, dequantise C, gelu8 + quantise after
 * FFN-up, add + LayerNorm + quantise (add_norm_quant) -- with the attention
 * on the bf16 tensor cores.  Needs every layer's four int8 operands and a
 * plain BERT model (no gated FFN, no rotary); refused otherwise.  The static
 * entry point (nebw_encode_device_static) runs the bf16 datapath only and
 * refuses a model set to NEBW_DATAPATH_I8. */
enum { NEBW_DATAPATH_BF16 = 0, NEBW_DATAPATH_I8 = 1 };
int nebw_model_set_datapath(nebw_model *m, int32_t datapath);
/* on != 0: the model's passes are replayed as CUDA graphs instead of
 * launching their ~7 kernels per layer one by one -- by nebw_encode (between
 * its input and output copies), nebw_encode_device and the sharded passes of
 * the several-GPU entry points.  A graph is captured (on a stream of the
 * library's own) on the first pass of a (B, S) shape with given device input
 * / output buffers (and the model's datapath and the device's attention
 * kernel), then launched in one call, on the caller's stream, whenever they
 * recur; the packed row count is computed
 * on the device inside the pass, so one graph serves every length pattern of
 * its shape.  Up to 16 are kept; setting a tensor, the datapath or growing
 * the workspace drops them.  Off by default; profiling (nebw_model_profile)
 * launches directly.  The results are the direct launches' bit for bit.  The
 * static entry point launches directly. */
int nebw_model_set_graphs(nebw_model *m, int32_t on);
/* The rotary frequency set as data (gte_new_rope_geglu's rope_inv_freq):
 * n = head_dim / 2 values, angle(s, j) = s * inv_freq[j] in double, as
 * apply_rope_qkv builds its tables (bert_encoder.cpp:929-945). */
int nebw_model_set_rope_freq(nebw_model *m, const double *inv_freq, int32_t n);
/* Stage every tensor of a `.npue` container -- the reference's npue::File +
 * set_model_shape + stage_all (runtime/src/model.cpp:214-380).  gemm_layout
 * "host" (F32 [K,N] operands, the reference packer's --dtype f32) or
 * "tma_bf16" (bf16 [N,K] operands, nebw.pack) or "pretiled_bf16" (the
 * reference's default block panels, a_dtype bf16, or int8 panels with
 * .wscale and .asmooth, a_dtype i8: see nebw_npue_gemm_kn).  Architectures
 * bert_abs_gelu_postln, nomic_bert_rope_swiglu and gte_new_rope_geglu, with
 * set_model_shape's refusals for the latter two (position encoding, gating,
 * the order of the fused FFN-up halves, the gate's activation).  A tma_bf16
 * GEMM operand whose layout_hash is not nebw_tma_layout_hash() is refused,
 * as the reference refuses a design whose b_layout_hash differs from the
 * model's (runtime/src/runtime.cpp:190-222).  The container is checked before
 * the device is used, so refusals need no GPU. */
int nebw_model_load_npue(nebw_dev *dev, const char *path, nebw_model **out);
/* One GEMM operand of a pre-tiled container (gemm_layout "pretiled_bf16",
 * block_panel BF16 or I8) as fp32 row-major [K, N], I8 dequantised per
 * column by its .wscale -- the reference's host_b_kn (runtime/include/common/
 * host_b.hpp:74-224).  Host only: no device is used.  nebw_model_load_npue
 * stages such operands this way, an int8 one further divided row by row by
 * its .asmooth (the activation's SmoothQuant divisor, moved onto the
 * weights). */
int nebw_npue_gemm_kn(const char *path, const char *name, float *out_kn, int64_t K, int64_t N);
/* The layout hash this library reads tma_bf16 GEMM operands in: sha256 (hex)
 * of the canonical JSON {"dtype":"BF16","kind":"dense","order":"n,k"}
 * (tools/lib/npue.py:777-785's scheme).  No reference counterpart as a
 * function: the reference reads it from a design's design.json. */
const char *nebw_tma_layout_hash(void);
/* The weight packer: a Hugging Face BERT checkpoint directory (config.json,
 * 1_Pooling/config.json, model.safetensors, optional vocab.txt and
 * CHECKPOINT.json) -> a `.npue` container at out_path.  layout "tma_bf16"
 * (NULL: the default) stores GEMM operands as bf16 [N, K] for
 * nebw_model_load_npue to upload as they are; "host" writes the reference
 * packer's --dtype f32 container (F32 [K, N]).  QKV fused, weights
 * transposed to [K, N], 1/sqrt(head_dim) folded into Q unless fold_scale is
 * 0, the position table cut to max_seq (<= 0: 256).  Replaces the BERT
 * branch of tools/pack/pack_npue.py (:2620-2835) and the runtime's
 * --prepare-model (runtime/src/common/npue_pack.cpp).  Host only; *bytes
 * (may be NULL) gets the file size.  NEBW_EIO names what is missing or
 * refused. */
int nebw_pack_checkpoint(const char *model_dir, const char *out_path, const char *layout,
                         int32_t max_seq, int32_t fold_scale, uint64_t *bytes);
int nebw_model_destroy(nebw_model *m);
int nebw_model_get_config(const nebw_model *m, nebw_config *cfg);

/* Encode B padded sequences end to end: host ids [B, S] int32 and host
 * lengths [B] (the attention mask as a prefix length; the tokenizer's mask is
 * always a prefix, wordpiece.cpp:354-378) in, host fp32 [B, hidden] pooled
 * (+L2) embeddings out.  Synchronous.  Replaces EmbedService::chunk's
 * run + pool_rows (embed_service.cpp:29-64; BertEncoder::run
 * bert_encoder.cpp:1419-1598). */
int nebw_encode(nebw_model *m, const int32_t *ids, const int32_t *lens, int32_t B, int32_t S,
                float *out);

/* The same pass with everything device-resident and asynchronous on
 * `stream`: ids_dev [B, S], lens_dev [B], out_dev [B, hidden].  No host
 * synchronisation inside; call nebw_sync (or synchronise the stream and call
 * nebw_sync) to collect device-side errors. */
int nebw_encode_device(nebw_model *m, const int32_t *ids_dev, const int32_t *lens_dev,
                       int32_t B, int32_t S, float *out_dev, void *stream);

/* Number of kernel launches one nebw_encode_device call makes for a model
 * at padded sequence length `seq` (<= 0: the model's max_seq_len), for
 * launch accounting. */
int nebw_encode_launch_count(const nebw_model *m, int32_t seq);

/* ---- per-kernel timing (the reference's BertEncoder::Timings,
 * bert_encoder.hpp:67-87, measured on the device) ------------------------
 * While enabled, every encoder pass brackets each kernel launch with CUDA
 * events on the launching stream.  nebw_model_profile_collect synchronises,
 * and returns, per kernel kind, the number of launches and their summed
 * device time since the last collect. */
enum {
  NEBW_K_PACK = 0, NEBW_K_EMBED_LN = 1, NEBW_K_GEMM_QKV = 2, NEBW_K_ATTENTION = 3,
  NEBW_K_GEMM_AO = 4, NEBW_K_LN = 5, NEBW_K_GEMM_UP = 6, NEBW_K_GEMM_DOWN = 7,
  NEBW_K_POOL = 8, NEBW_K_COUNT = 9
};
int nebw_model_profile(nebw_model *m, int enable);
int nebw_model_profile_collect(nebw_model *m, int64_t launches[NEBW_K_COUNT],
                               double ms[NEBW_K_COUNT]);

/* nebw_encode_device without any allocation at call time.  This entry point
 * has no counterpart in the reference.  It is for callers that cannot
 * allocate device memory when a request arrives: a serving process that
 * claims its whole GPU-memory budget at start-up, or a program sharing the
 * GPU under a fixed partition.  (nebw_encode_device may cudaMalloc a larger
 * workspace the first time it sees a larger batch.)  All intermediates live
 * in one static 64 MiB device array that every GPU loading the library holds
 * until exit.  A batch needs B * S * (16 * hidden + 2 * F) bytes of it (F the
 * FFN width; 2F for a gated FFN without CTA pairs; plus 4 per row for a
 * rotary head_dim-64 model), plus about 12 * B + B * S / 32 bytes and up to
 * 2.5 KB of alignment; a batch that does not fit is refused with NEBW_EINVAL
 * (bge-large: about 2730 padded rows fit; MiniLM: about 7280).  The first
 * call on a device looks the array's address up and should come before any
 * stream capture.  All calls share the array and it keeps the last call's
 * contents (a pass clears what it reads before writing it): calls that
 * overlap on the GPU race, so the caller serialises them.  The pass launches
 * the same kernels as nebw_encode_device and returns the same bits; static
 * calls record no per-kernel profiling events.  Arguments and results as
 * nebw_encode_device. */
int nebw_encode_device_static(nebw_model *m, const int32_t *ids_dev, const int32_t *lens_dev,
                              int32_t B, int32_t S, float *out_dev, void *stream);

/* ---- ViT encoder (container arch "vit_patch16_prenorm_gelu") --------------
 * Replaces npue::vit::VitEncoder (runtime/include/vit/encoder.hpp:87-289):
 * its stage_all() (runtime/src/vit/encoder.cpp:23-189) becomes
 * nebw_vit_create + nebw_vit_set_tensor or nebw_vit_load_npue, and its run()
 * (:222-431) becomes nebw_vit_encode / nebw_vit_encode_device, which also
 * take over the image -> patch step im2col_patches
 * (runtime/src/vit/image.cpp:732-755).  Schedule (pre-LN):
 *   patches = im2col(image); x = [cls; patches . W_patch + b] + pos
 *   per layer: x += attn_out(attention(qkv(LN1(x))))
 *              x += ffn_down(gelu_erf(ffn_up(LN2(x))))
 *   out = LN_final(x[CLS row])            (the reference's run() returns every
 *                                          row; the head reads the CLS row)
 * Q's 1/sqrt(head_dim) must already be folded into the qkv operand, as
 * containers with qkv_scale_folded (the packer's default) have it.  Every
 * image is one unmasked sequence of (image_size/patch_size)^2 + 1 rows.
 * GEMM operands bf16 (RNE), fp32 accumulation, every GEMM output narrowed
 * to bf16 RNE (as the reference's array path narrows each C tile), the
 * residual add fused into the next LayerNorm, fp32 residual stream, exact-erf
 * GELU in the FFN-up epilogue, attention on the same kernels as the BERT
 * pass, LayerNorm fp32 two-pass. */
typedef struct nebw_vit_config {
  int32_t num_layers, hidden, num_heads, head_dim, intermediate;
  int32_t image_size, patch_size, num_channels;  /* hidden == channels * patch^2 */
  float layer_norm_eps;
} nebw_vit_config;

typedef struct nebw_vit nebw_vit;

int nebw_vit_create(nebw_dev *dev, const nebw_vit_config *cfg, nebw_vit **out);
/* Tensor names of the ViT container (encoder.cpp:125-139): frontend.patch_embed
 * [C*P*P, hidden] (+ .bias), frontend.cls_token [hidden],
 * frontend.position_embeddings [n_pos, hidden], layer.{i}.{qkv, attn_out,
 * ffn_up, ffn_down}[.bias], layer.{i}.{ln1,ln2}.{weight,bias},
 * layernorm.{weight,bias}.  GEMM operands [K, N] F32 or BF16; the rest F32. */
int nebw_vit_set_tensor(nebw_vit *m, const char *name, const void *host, int dtype, int64_t rows,
                        int64_t cols);
/* A gemm_layout "host" container; its classifier head is not loaded (the
 * reference runs the head on the host, encoder.cpp:433-444). */
int nebw_vit_load_npue(nebw_dev *dev, const char *path, nebw_vit **out);
int nebw_vit_get_config(const nebw_vit *m, nebw_vit_config *cfg);
int nebw_vit_destroy(nebw_vit *m);
/* images [n, C, S, S] fp32 (normalised pixels, 16-byte aligned) -> out [n,
 * hidden] fp32, the CLS row after the final LayerNorm.  Device buffers,
 * asynchronous on `stream` (NULL: the device's stream). */
int nebw_vit_encode_device(nebw_vit *m, const float *images_dev, int32_t n, float *out_dev,
                           void *stream);
/* The same with host buffers: copies in, the pass, copies out, synchronous. */
int nebw_vit_encode(nebw_vit *m, const float *images_host, int32_t n, float *out_host);
/* Kernel launches one nebw_vit_encode_device makes. */
int nebw_vit_launch_count(const nebw_vit *m);
/* Per-kernel device time, as nebw_model_profile: im2col under NEBW_K_PACK,
 * the patch GEMM and the row assembly under NEBW_K_EMBED_LN, the LayerNorm
 * sites (each fused with the residual add before it) under NEBW_K_LN, the
 * last residual add with the final CLS-row LayerNorm under NEBW_K_POOL. */
int nebw_vit_profile(nebw_vit *m, int enable);
int nebw_vit_profile_collect(nebw_vit *m, int64_t launches[NEBW_K_COUNT],
                             double ms[NEBW_K_COUNT]);

/* ---- several GPUs: the batch sharded, the embeddings gathered -------------
 * The reference has no multi-device code; its only concurrency is host
 * threads sharing one NPU (the --pipeline lanes of EmbedService::embed,
 * runtime/src/server/embed_service.cpp:66-108, run_setup.hpp:465-480).  Every
 * sequence is an independent encoder pass (conv_host.hpp:154-158,
 * bert_encoder.cpp:1001-1004), so a batch splits across GPUs with one weight
 * replica per GPU (one nebw_model per GPU) and no exchange on the data path;
 * the pooled [b_r, hidden] fp32 rows of every rank are gathered to rank 0
 * over NCCL (NVLink / NVSwitch) and put back in request order there.
 *
 * NCCL (libnccl.so.2, or the file $NEBW_NCCL_LIB names) is loaded on first
 * use, or the copy the process already holds is used; without it these calls
 * return NEBW_ECOMM.  A process that also uses another NCCL (PyTorch's)
 * loads that one before the first call here.  Communicators are non-blocking and every wait on one is
 * bounded by its timeout_s: on expiry (a rank that never joins, a peer that
 * died) the communicator is aborted, the call returns NEBW_ECOMM, and later
 * calls on it return NEBW_ESTATE.  Collective calls must be made by every
 * rank in the same order. */
#define NEBW_COMM_ID_BYTES 128
typedef struct nebw_comm nebw_comm;

/* A fresh communicator id: made by one rank and handed to the others over
 * the host (a socket, a file, a key-value store). */
int nebw_comm_unique_id(uint8_t id[NEBW_COMM_ID_BYTES]);
/* Join communicator `id` as `rank` of `nranks` (one process per GPU).
 * Collective. */
int nebw_comm_init_rank(nebw_dev *dev, int32_t nranks, int32_t rank,
                        const uint8_t id[NEBW_COMM_ID_BYTES], double timeout_s,
                        nebw_comm **out);
/* One process driving n GPUs: comms[i] is rank i, on devs[i]. */
int nebw_comm_init_all(int32_t n, nebw_dev *const *devs, double timeout_s, nebw_comm **comms);
/* Flush and free (bounded by the timeout; an aborted communicator is only
 * freed). */
int nebw_comm_destroy(nebw_comm *c);
int nebw_comm_size(const nebw_comm *c, int32_t *nranks, int32_t *rank);
/* Wait (bounded) for `stream` to drain -- the collectives enqueued on it
 * included -- then report device errors as nebw_sync does. */
int nebw_comm_sync(nebw_comm *c, void *stream);

/* The shard plan, host only and deterministic (every rank computes the same
 * plan from the same lengths): sequences in decreasing cost l + l^2 / 2048
 * (the GEMMs grow with l, attention with l^2), each to the rank with the
 * least cost so far.  owner[B] gets each sequence's rank, counts[nranks]
 * the sequences per rank; a rank's shard is its sequences in ascending
 * order. */
int nebw_shard_plan(const int32_t *lens, int32_t B, int32_t nranks, int32_t *owner,
                    int32_t *counts);
/* order[k] = the request index of row k of the rank-major gather (each
 * rank's sequences ascending). */
int nebw_shard_order(const int32_t *owner, int32_t B, int32_t nranks, int32_t *order);
/* Gather counts[r] rows of H fp32 from every rank r (rows_dev, device) to
 * rank `root`'s out_dev [sum(counts), H] in rank order.  Asynchronous on
 * `stream`; collective. */
int nebw_gather_rows(nebw_comm *c, const float *rows_dev, const int32_t *counts, int32_t H,
                     float *out_dev, int32_t root, void *stream);

/* The sharded encoder pass with the shard already on this rank's GPU: encode
 * this rank's b_r sequences (ids_dev [b_r, S], lens_dev [b_r]), gather the
 * pooled rows to rank 0, and there write out_dev [B, hidden] (B =
 * sum(counts)) in request order through order_dev [B] (nebw_shard_order;
 * NULL keeps rank order).  Asynchronous on `stream`; nebw_comm_sync waits.
 * Collective. */
int nebw_encode_shard_gather(nebw_model *m, nebw_comm *c, const int32_t *ids_dev,
                             const int32_t *lens_dev, int32_t b_r, int32_t S,
                             const int32_t *counts, const int32_t *order_dev, float *out_dev,
                             void *stream);
/* The sharded pass with host buffers, as nebw_encode: every rank passes the
 * whole batch (ids [B, S], lens [B]) and encodes its share of the plan; rank
 * 0 receives [B, hidden] in request order in `out` (other ranks may pass
 * NULL).  Synchronous; collective. */
int nebw_encode_sharded(nebw_model *m, nebw_comm *c, const int32_t *ids, const int32_t *lens,
                        int32_t B, int32_t S, float *out);
/* One process, n GPUs: models[i] on comms[i] (nebw_comm_init_all), one host
 * thread per GPU running nebw_encode_sharded; `out` [B, hidden] in request
 * order.  Synchronous.  (The reference's lane-parallel EmbedService::embed,
 * embed_service.cpp:66-108, over GPUs instead of one NPU.) */
int nebw_encode_multi(int32_t n, nebw_model *const *models, nebw_comm *const *comms,
                      const int32_t *ids, const int32_t *lens, int32_t B, int32_t S, float *out);

#ifdef __cplusplus
}
#endif
#endif /* NEBW_H */
