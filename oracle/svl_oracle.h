/*
 * svl_oracle.h — CPU restatement of semantic-voice-local's streaming LM step.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the parity checker for the CUDA path and the
 * timed CPU baseline. Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
 * --impl reference legs may load it. The product (semantic-ai_b200/) never links it.
 *
 * Parity status: the restatement is pinned to the reference's own unit-test bounds
 * (activations within 8 ulp of f64, attention vs generic masked softmax within 1e-5, matvec
 * vs matmul within 1e-5*k, streaming == full sequence within 1e-4) through torch-f64
 * fixtures in tests/golden/. The reference is Rust on candle 0.11.1 and cannot be built in
 * this image, so the candle-internal pieces (Q8_0 QMatMul, rope_i, rms_norm/layer_norm
 * reduction order, argmax tie rule) are restated from their published algorithms and are
 * "parity unpinned" against candle itself.
 */
#ifndef SVL_ORACLE_H
#define SVL_ORACLE_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same field layout as svl_transformer_config in include/svl_cuda.h. */
typedef struct {
  int32_t d_model, num_layers, num_heads, num_kv_heads, head_dim;
  int32_t ffn_kind;   /* 0 plain gelu-tanh, 1 plain gelu-erf, 2 gated silu */
  int32_t ffn_hidden;
  int32_t norm_kind;  /* 0 layer norm, 1 rms norm */
  float norm_eps;
  int32_t layer_scale;
  int32_t context;    /* 0 = unlimited */
  int32_t weight_dtype; /* 0 f32, 1 bf16, 2 q8_0, 3 q4_1 */
  int32_t kv_dtype;     /* 0 f32, 1 bf16 */
  int32_t _pad;
  double max_period;
} orc_tcfg;

typedef struct {
  int32_t card, n_q, text_card, extra_heads_num, extra_heads_dim, _pad;
} orc_stt_extra;

typedef struct {
  int32_t latent_dim, flow_dim, flow_depth, flow_kind, text_bins, _pad;
} orc_tts_extra;

typedef struct {
  const char* name;
  const float* data; /* host f32, row-major */
  int64_t numel;
} orc_tensor;

typedef struct orc_lm orc_lm;
typedef struct orc_state orc_state;

/* Builds a model from named f32 tensors. kind 0 = STT LanguageModel, 1 = Pocket-TTS FlowLm.
 * Weights are converted like the reference's loader: quantised to Q8_0/Q4_1 or rounded to
 * bf16 per cfg->weight_dtype. Returns NULL and sets orc_last_error() on failure. */
orc_lm* orc_lm_create(int kind, const orc_tcfg* cfg, const orc_stt_extra* stt,
                      const orc_tts_extra* tts, const orc_tensor* tensors, int n_tensors);
/* A bare transformer (kind 2) whose tensors are named under `prefix` (Mimi's transformers). */
orc_lm* orc_transformer_create(const orc_tcfg* cfg, const char* prefix, const orc_tensor* tensors,
                               int n_tensors);
void orc_lm_free(orc_lm*);
orc_state* orc_state_create(orc_lm*);
orc_state* orc_state_duplicate(const orc_state*);
void orc_state_free(orc_state*);
int orc_state_position(const orc_state*);
const char* orc_last_error(void);
void orc_set_threads(int n);
/* Test-only: 1 = RMS-norm sum of squares in reverse order (sensitivity envelope). */
void orc_set_reduction_variant(int v);

/* LanguageModel::step (svl/stt/model.rs:239-277). logits (text_card) and extra
 * (extra_heads_num) may be NULL. Returns 0 on success. */
int orc_stt_step(orc_lm*, orc_state*, uint32_t text_token, const uint32_t* audio_tokens,
                 uint32_t* out_token, float* logits, float* extra);

/* Transformer::forward (svl/nn/transformer.rs:139-186) on xs[t][d] in place. */
int orc_transformer_forward(orc_lm*, orc_state*, float* xs, int t);

/* FlowLm::step (svl/tts/flow_lm.rs:162-185): latent_in NULL means BOS. noise is the
 * already-sampled [latent_dim] noise (the reference draws it on the host). */
int orc_tts_step(orc_lm*, orc_state*, const float* latent_in, const float* noise,
                 float decode_steps_f, float* latent_out, float* eos_logit);
/* FlowLm::prompt_text (svl/tts/flow_lm.rs:150-158). */
int orc_tts_prompt_text(orc_lm*, orc_state*, const uint32_t* tokens, int n);

/* Kernel-level restatements, exposed for the known-answer tests. */
float orc_dot(const float* a, const float* b, int n);
float orc_exp(float x);
float orc_silu(float x);
float orc_gelu_tanh(float x);
void orc_matvec(const float* x, const float* w, const float* bias, int n, int k, float* out);
void orc_attention(const float* q, const float* k, const float* v, int heads, int kv_heads,
                   int t, int n, int d, int64_t k_head_stride, int64_t k_row_stride,
                   int position, int first_key, int context, float* out);
void orc_rms_norm(const float* x, const float* alpha, int d, float eps, float* out);
void orc_layer_norm(const float* x, const float* w, const float* b, int d, float eps,
                    float* out);
/* Q8_0 / Q4_1 blocks in the ggml layout: Q8_0 {f16 d; i8 qs[32]} (34 B),
 * Q4_1 {f16 d; f16 m; u8 qs[16]} (20 B). */
void orc_quantize_q8_0(const float* x, int64_t n, uint8_t* blocks);
void orc_quantize_q4_1(const float* x, int64_t n, uint8_t* blocks);
void orc_matvec_q8_0(const float* x, const uint8_t* wblocks, int n, int k, float* out);
void orc_matvec_q4_1(const float* x, const uint8_t* wblocks, int n, int k, float* out);
uint16_t orc_f32_to_f16(float x);
float orc_f16_to_f32(uint16_t h);
float orc_round_bf16(float x);

/* ---- Mimi codec and residual vector quantizer (svl_codec_oracle.c) ---------------------- */

/* Activation::Elu (nn/kernels/activation.rs:60-67). */
float orc_elu(float x);

/* Same layouts as svl_seanet_config / svl_projected_transformer_config / svl_mimi_config in
 * include/svl_cuda.h. */
typedef struct {
  int32_t dimension, channels, n_filters, n_residual_layers;
  int32_t kernel_size, residual_kernel_size, last_kernel_size, dilation_base;
  int32_t pad_mode, compress, n_ratios;
  int32_t ratios[8];
  int32_t _pad;
} orc_seanet_cfg;
typedef struct {
  int32_t d_model, input_dimension, output_dimension, num_heads, num_layers, context;
  int32_t dim_feedforward, _pad;
  double max_period;
} orc_ptrans_cfg;
typedef struct {
  int32_t sample_rate, inner_dim, outer_dim, exact_gelu, parts, _pad;
  double frame_rate;
  orc_seanet_cfg encoder, decoder;
  orc_ptrans_cfg encoder_transformer, decoder_transformer;
} orc_mimi_cfg;
typedef struct orc_mimi orc_mimi;
typedef struct orc_mimi_state orc_mimi_state;
typedef struct orc_rvq orc_rvq;

/* StreamingConv1d::forward (nn/conv.rs:122-179) of one stream, state passed explicitly: w
 * [cout][cin][k], bias [cout] or NULL, prev [cin][ctx] with ctx = max(0, (k-1) dil + 1 - stride)
 * and *started (0 before the first chunk; set to 1), x [cin][t] (ELU applied first when elu
 * is set), skip [cout][t/stride] or NULL (added after the bias), out [cout][t/stride]. */
int orc_conv1d_stream(int cin, int cout, int k, int stride, int dil, int replicate, const float* w,
                      const float* bias, float* prev, int* started, const float* x, int t, int elu,
                      const float* skip, float* out);
/* StreamingConvTranspose1d::forward (nn/conv.rs:265-335) of one stream: w [cin][cout/groups][k]
 * (groups 1 or depthwise), partial [cout][k - stride] (zeros at the start), x [cin][t], out
 * [cout][t * stride]. */
int orc_convtr1d_stream(int cin, int cout, int k, int stride, int depthwise, const float* w,
                        const float* bias, float* partial, const float* x, int t, int elu,
                        float* out);

/* MimiEncoder / MimiDecoder (nn/mimi.rs:133-272) for one stream. */
orc_mimi* orc_mimi_create(const orc_mimi_cfg* cfg, const orc_tensor* tensors, int n_tensors);
void orc_mimi_free(orc_mimi*);
int orc_mimi_frame_size(const orc_mimi*);
orc_mimi_state* orc_mimi_state_create(orc_mimi*);
void orc_mimi_state_free(orc_mimi_state*);
/* pcm [channels][frames * frame_size] -> latent [inner_dim][frames]. */
int orc_mimi_encode_step(orc_mimi*, orc_mimi_state*, const float* pcm, int frames, float* latent);
/* latent [outer_dim][frames] -> pcm [channels][frames * frame_size]. */
int orc_mimi_decode_step(orc_mimi*, orc_mimi_state*, const float* latent, int frames, float* pcm);

/* Tts::decode_latent (tts/mod.rs:441-447): latent [frames][latent_dim], emb_std / emb_mean
 * [latent_dim] (both NULL to skip), through "quantizer.output_proj.weight", then decode_step. */
int orc_mimi_decode_latent(orc_mimi*, orc_mimi_state*, const float* latent, int frames,
                           const float* emb_std, const float* emb_mean, float* pcm);

/* Quantizer (stt/model.rs:84-170): latent [512][frames] -> codes [frames][n_q]. */
orc_rvq* orc_rvq_create(int n_q, int bins, const orc_tensor* tensors, int n_tensors);
void orc_rvq_free(orc_rvq*);
int orc_rvq_encode(orc_rvq*, const float* latent, int frames, uint32_t* codes);
/* The distances of one codebook for a residual (test support): dist[bins]. */
int orc_rvq_distances(orc_rvq*, int codebook, const float* residual, float* dist);

#ifdef __cplusplus
}
#endif
#endif
