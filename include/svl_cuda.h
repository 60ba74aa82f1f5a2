/*
 * svl_cuda.h — C ABI of the B200 (sm_100a) streaming language-model step.
 *
 * This is the drop-in boundary for semantic-voice-local's per-frame StreamingTransformer
 * step (Kyutai STT LanguageModel, Pocket-TTS FlowLm) on `--device cuda`. Every entry point
 * names the reference interface it replaces; paths are relative to
 * crates/semantic-voice-local/src/ in semantiverse/semantic-ai.
 *
 * Conventions
 *  - Plain pointers and sizes only. Host pointers unless the name ends in _device.
 *  - Every call returns an svl_status; svl_last_error() holds the message of the last
 *    failure on the calling thread. The codes mirror the reference's Error enum
 *    (error.rs:2-31): CONFIG = Error::Config, INVALID_INPUT = Error::InvalidInput,
 *    CUDA/OOM/TIMEOUT = Error::Candle raised by the device.
 *  - A model is immutable after creation and may be shared by threads (the reference's
 *    Stt/Tts are Send + Sync, stt/mod.rs:159). A state is owned by one thread at a time
 *    (the reference mutates TransformerState through &mut).
 *  - There is no CPU fallback: without a B200 every call that touches the device fails with
 *    SVL_ERR_CUDA.
 */
#ifndef SVL_CUDA_H
#define SVL_CUDA_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define SVL_API __attribute__((visibility("default")))
#else
#define SVL_API
#endif

typedef enum svl_status {
  SVL_OK = 0,
  SVL_ERR_CONFIG = 1,        /* Error::Config: bad config or weight shapes */
  SVL_ERR_INVALID_INPUT = 2, /* Error::InvalidInput: token ids, batch, lengths */
  SVL_ERR_CUDA = 3,          /* a CUDA runtime error (no device, launch failure) */
  SVL_ERR_OOM = 4,           /* device allocation failed */
  SVL_ERR_TIMEOUT = 5,       /* a bounded device-side wait expired */
  SVL_ERR_UNSUPPORTED = 6    /* a config this build does not implement */
} svl_status;

/* FeedForward (nn/transformer.rs:19-24). */
typedef enum { SVL_FFN_PLAIN_GELU_TANH = 0, SVL_FFN_PLAIN_GELU_ERF = 1, SVL_FFN_GATED_SILU = 2 } svl_ffn_kind;
/* Norm (nn/transformer.rs:13-16). */
typedef enum { SVL_NORM_LAYER = 0, SVL_NORM_RMS = 1 } svl_norm_kind;
/* Weight storage. Q8_0 is what Linear::from_weight builds (nn/mod.rs:76-88); Q4_1 (32
 * 4-bit values with an f16 scale and min) has no reference counterpart. */
typedef enum { SVL_DT_F32 = 0, SVL_DT_BF16 = 1, SVL_DT_Q8_0 = 2, SVL_DT_Q4_1 = 3 } svl_dtype;

/* TransformerConfig (nn/transformer.rs:27-41). `quantize` becomes weight_dtype; context 0
 * means None (unlimited). kv_dtype is F32 (the reference CPU path) or BF16 (its CUDA path,
 * stt/mod.rs:193). */
typedef struct svl_transformer_config {
  int32_t d_model, num_layers, num_heads, num_kv_heads, head_dim;
  int32_t ffn_kind;
  int32_t ffn_hidden;
  int32_t norm_kind;
  float norm_eps;
  int32_t layer_scale;
  int32_t context;
  int32_t weight_dtype;
  int32_t kv_dtype;
  int32_t _pad;
  double max_period;
} svl_transformer_config;

/* The fields of SttConfig (stt/model.rs:17-43) that the language model uses. */
typedef struct svl_stt_config {
  int32_t card, n_q, text_card, extra_heads_num, extra_heads_dim, _pad;
} svl_stt_config;

/* The fields of FlowLmConfig / FlowHeadConfig (tts/config.rs:177-219) the step uses.
 * flow_kind: 0 lsd, 1 flow_matching, 2 drifting, 3 pointwise (FlowKind, tts/config.rs:177). */
typedef struct svl_tts_config {
  int32_t latent_dim, flow_dim, flow_depth, flow_kind, text_bins, _pad;
} svl_tts_config;

/* One named f32 tensor in host memory, row-major. The names are the reference's safetensors
 * names (stt/model.rs:224-231, nn/transformer.rs:206-218, :305-312, :429-432,
 * tts/flow_lm.rs:78-124). */
typedef struct svl_tensor_view {
  const char* name;
  const float* data;
  int64_t numel;
} svl_tensor_view;

typedef struct svl_model svl_model;
typedef struct svl_state svl_state;

/* LanguageModel::new (stt/model.rs:196-233) on `device`: uploads, converts and (for Q8_0 /
 * Q4_1) quantises the weights like Linear::from_weight (nn/mod.rs:76-88). */
SVL_API svl_status svl_stt_model_create(const svl_transformer_config* cfg,
                                        const svl_stt_config* stt,
                                        const svl_tensor_view* tensors, int32_t n_tensors,
                                        int32_t device, svl_model** out);

/* FlowLm::new (tts/flow_lm.rs:45-126). */
SVL_API svl_status svl_tts_model_create(const svl_transformer_config* cfg,
                                        const svl_tts_config* tts,
                                        const svl_tensor_view* tensors, int32_t n_tensors,
                                        int32_t device, svl_model** out);

SVL_API void svl_model_destroy(svl_model* model);

/* Bytes of weights the model streams per step (the roofline numerator without KV). */
SVL_API int64_t svl_model_weight_bytes(const svl_model* model);

/* Transformer::init_state (nn/transformer.rs:127-136) for up to max_batch independent
 * streams. Each stream holds a KV ring of `context` slots per layer (or max_positions slots
 * without a window) and its own position. */
SVL_API svl_status svl_state_create(svl_model* model, int32_t max_batch, int32_t max_positions,
                                    svl_state** out);
/* svl_state_create with options; flags is a combination of:
 *   SVL_STATE_REFERENCE_ORDER: every reduction whose order the reference's CPU path fixes
 *     runs in that order -- the norm sums element by element (candle rms_norm / layer_norm),
 *     the attention key by key (nn/kernels/attention.rs:142-169), RoPE from a table of the C
 *     library's cosf / sinf evaluated at state creation (nn/transformer.rs:159-166) -- and
 *     the f32 / bf16 weight products in kernels::dot's lane order (nn/kernels/mod.rs:68-91),
 *     so that a step reproduces the reference CPU arithmetic bit for bit on identical
 *     inputs. Quantised products use the reference order in every state. Slower (norm and
 *     softmax sums become serial chains; many-stream products stay off the tensor cores);
 *     positions are limited to max(max_positions, 8192) and rings to 51,200 keys.
 * No counterpart in the reference (whose CPU path is this order). */
#define SVL_STATE_REFERENCE_ORDER 1u
/* Testing only, quantised models: a failure drill for the device-side bounded waits. In every
 * step the first weight product withholds one of its staged weight copies and waits for it
 * only briefly, so that wait runs out: the kernel records the timeout, lets its other copies
 * land and returns, and the step reports SVL_ERR_TIMEOUT (svl_state_error for the _device
 * calls). Nothing faults or hangs; the state's contents after such a step are undefined. */
#define SVL_STATE_TEST_WITHHELD_COPY 2u
SVL_API svl_status svl_state_create_ex(svl_model* model, int32_t max_batch, int32_t max_positions,
                                       uint32_t flags, svl_state** out);
SVL_API void svl_state_destroy(svl_state* state);
/* Back to position 0 (a fresh init_state) for one stream, or all when stream < 0. */
SVL_API svl_status svl_state_reset(svl_state* state, int32_t stream);
/* TransformerState position of a stream (nn/transformer.rs:53-56). */
SVL_API svl_status svl_state_position(svl_state* state, int32_t stream, int32_t* position);
/* TransformerState::duplicate (nn/transformer.rs:64-73): copy stream src of `from` into
 * stream dst of `to` (same model). */
SVL_API svl_status svl_state_copy(svl_state* to, int32_t dst, const svl_state* from, int32_t src);
/* TransformerState::layer_caches (nn/transformer.rs:76-78): the keys and values a stream can
 * still attend to, as [kv_heads][len][head_dim] f32 per layer, oldest first. k and v hold
 * kv_heads * capacity * head_dim floats; *len receives the entry count. */
SVL_API svl_status svl_state_export(svl_state* state, int32_t stream, int32_t layer, float* k,
                                    float* v, int32_t* len, int32_t* position);
/* TransformerState::from_layer_caches (nn/transformer.rs:81-103) for one layer: k and v
 * [kv_heads][len][head_dim] are the entries of positions position-len .. position-1. Call for
 * every layer with the same position; from_layer_caches is position == len. Slots of the
 * window older than the imported entries keep their contents; len == 0 only moves the
 * stream to `position`. */
SVL_API svl_status svl_state_import(svl_state* state, int32_t stream, int32_t layer,
                                    const float* k, const float* v, int32_t len,
                                    int32_t position);

/* Voice::save (tts/voice.rs:78-99): stream `stream` of the state as a voice file, in the
 * safetensors layout of upstream Pocket TTS: per layer i, "transformer.layers.{i}.self_attn/cache"
 * f32 [2, 1, len, kv_heads, head_dim] (keys then values, oldest first),
 * ".../offset" i64 [1] = len and ".../pad" i64 [1] = 0. */
SVL_API svl_status svl_voice_save(svl_state* state, int32_t stream, const char* path);

/* Voice::load (tts/voice.rs:101-149) into streams[0..n_streams) of the state at once: reads a
 * voice file of that layout (cache f32, bf16 or f16; the length from ".../offset", else the
 * shape of ".../current_end", else the time axis), refuses padded (batched) states with
 * SVL_ERR_INVALID_INPUT, uploads the keys and values once and writes them into every listed
 * stream's ring with one kernel; each stream then continues at position len
 * (TransformerState::from_layer_caches). */
SVL_API svl_status svl_voice_load(svl_state* state, const int32_t* streams, int32_t n_streams,
                                  const char* path);

/* LanguageModel::step (stt/model.rs:239-277) for streams 0..batch-1, host buffers:
 * text_tokens [batch], audio_tokens [batch][n_q] in, out_tokens [batch] (greedy argmax,
 * lowest index on ties) out. out_logits [batch][text_card] and out_extra
 * [batch][extra_heads_num] (softmax p[0] of each extra head) may be NULL. */
SVL_API svl_status svl_stt_step(svl_model* model, svl_state* state, int32_t batch,
                                const uint32_t* text_tokens, const uint32_t* audio_tokens,
                                uint32_t* out_tokens, float* out_logits, float* out_extra);

/* The same step on device buffers, enqueued on `cuda_stream` (a cudaStream_t, NULL = the
 * model's stream) without host synchronisation. The step is one CUDA graph per batch size. */
SVL_API svl_status svl_stt_step_device(svl_model* model, svl_state* state, int32_t batch,
                                       const uint32_t* d_text_tokens,
                                       const uint32_t* d_audio_tokens, uint32_t* d_out_tokens,
                                       float* d_out_logits, void* cuda_stream);

/* Recognizer::step's token loop (stt/mod.rs:551-565) for n_frames frames: each stream's
 * first step (position 0) sees the initial tokens (audio = card, text = text_card), later
 * steps feed back the previous argmax on the device. audio_tokens [n_frames][batch][n_q],
 * out_tokens [n_frames][batch], host memory. */
SVL_API svl_status svl_stt_run_frames(svl_model* model, svl_state* state, int32_t batch,
                                      int32_t n_frames, const uint32_t* audio_tokens,
                                      uint32_t* out_tokens);

/* svl_stt_run_frames that also returns, per frame and stream, the extra (voice activity) heads'
 * softmax p[0] (Prediction::extra_head_probabilities, stt/model.rs:259-271), the input of
 * SttEvent::VoiceActivity (stt/mod.rs:566-572): out_extra [n_frames][batch][extra_heads_num]
 * host memory, or NULL. */
SVL_API svl_status svl_stt_run_frames_ex(svl_model* model, svl_state* state, int32_t batch,
                                         int32_t n_frames, const uint32_t* audio_tokens,
                                         uint32_t* out_tokens, float* out_extra);

/* Transformer::forward (nn/transformer.rs:139-154) of one stream over xs [t][d_model] (host,
 * in place), t >= 1: the prefill path. */
SVL_API svl_status svl_transformer_forward(svl_model* model, svl_state* state, int32_t stream,
                                           float* xs, int32_t t);

/* FlowLm::prompt_text (tts/flow_lm.rs:150-158) for one stream. */
SVL_API svl_status svl_tts_prompt_text(svl_model* model, svl_state* state, int32_t stream,
                                       const uint32_t* tokens, int32_t n);

/* FlowLm::prompt_text (tts/flow_lm.rs:150-158) for streams 0..batch-1 at once, n tokens
 * each: tokens [batch][n]. */
SVL_API svl_status svl_tts_prompt_text_batch(svl_model* model, svl_state* state, int32_t batch,
                                             const uint32_t* tokens, int32_t n);

/* FlowLm::step (tts/flow_lm.rs:162-185) for streams 0..batch-1: latent_in [batch][latent]
 * (NULL = BOS for every stream), noise [batch][latent] (the reference samples it on the host,
 * flow_lm.rs:187-203), latent_out [batch][latent], eos_logit [batch]. */
SVL_API svl_status svl_tts_step(svl_model* model, svl_state* state, int32_t batch,
                                const float* latent_in, const float* noise, int32_t decode_steps,
                                float* latent_out, float* eos_logit);

/* The same step on device buffers, enqueued on `cuda_stream` (NULL = the model's stream)
 * without host synchronisation; d_latent_in NULL = BOS. d_latent_in may be the previous
 * call's d_latent_out (the latent feedback of LatentGenerator::advance, tts/mod.rs:494). */
SVL_API svl_status svl_tts_step_device(svl_model* model, svl_state* state, int32_t batch,
                                       const float* d_latent_in, const float* d_noise,
                                       int32_t decode_steps, float* d_latent_out, float* d_eos,
                                       void* cuda_stream);

/* Profiling hook (no counterpart in the reference): enqueues `iters` repetitions of one
 * kernel family of the step for streams 0..batch-1 on `cuda_stream` so a caller can time
 * it with CUDA events on that stream. which = 0: every weight product of the transformer
 * (the layer linears, and the head of an STT model); which = 1: every layer's attention;
 * which = 2 (TTS models): the flow head with one decode step. The repetitions overwrite the
 * state's activations and KV slots at the current positions, so the state must be reset
 * before it is used again. *bytes_per_iter receives the algorithmic HBM bytes of one
 * repetition (weights, or the KV rows read at the current positions). */
SVL_API svl_status svl_profile_kernels(svl_model* model, svl_state* state, int32_t batch,
                                       int32_t which, int32_t iters, void* cuda_stream,
                                       int64_t* bytes_per_iter);

/* The device-side error flag of a state, for callers of the *_device entry points (the
 * host-buffer calls check it themselves): waits for the device, then returns
 * SVL_ERR_INVALID_INPUT if a token id out of range reached the device, SVL_ERR_TIMEOUT if a
 * bounded device-side wait ran out, SVL_OK otherwise; the flag is cleared. */
SVL_API svl_status svl_state_error(svl_state* state);

/* Kernels one step call (svl_stt_step[_device], or svl_tts_step[_device] with one decode
 * step) launches at this batch size: the kernel nodes of the step's CUDA graph, which this
 * call captures if no step of that batch size ran yet. Diagnostics only; no counterpart in
 * the reference. */
SVL_API svl_status svl_step_kernel_count(svl_model* model, svl_state* state, int32_t batch,
                                         int32_t* kernels);

/* The greedy head alone -- out_norm, text_linear and argmax, the end of LanguageModel::step
 * -- for callers that cannot allocate device memory. It has no counterpart in the
 * reference: it exists for hosts that own every device allocation of the process (a plugin
 * host's memory pool, a real-time audio thread that must never enter the allocator, code
 * where a cudaMalloc would synchronise the device mid-stream) and so cannot create a state,
 * whose scratch svl_stt_step uses.
 * d_hidden [batch][d_model] f32 (the transformer output), d_tokens [batch] out, d_logits
 * [batch][text_card] out or NULL; device pointers, enqueued on cuda_stream (NULL = the
 * model's stream). The argmax scratch is a fixed 19,200-byte __device__ array inside the
 * library (every GPU that loads the library holds it until the process exits): batch is
 * limited to 8 streams per call, larger batches are rejected with SVL_ERR_INVALID_INPUT.
 * Nothing is allocated: the first call on a device looks up the array's device address
 * (make that first call before any stream capture), every call clears the array's counter
 * on the stream and launches the head. All calls share the array, so calls that overlap on
 * the GPU (on different streams, or on different models of one device) race: serialise
 * them. */
SVL_API svl_status svl_stt_head_noalloc(svl_model* model, int32_t batch, const float* d_hidden,
                                        uint32_t* d_tokens, float* d_logits, void* cuda_stream);

/* ---- Mimi, the codec around the language models (nn/mimi.rs, nn/seanet.rs, nn/conv.rs) ---- */

/* SeanetConfig (nn/seanet.rs:14-30); pad_mode 0 = PadMode::Constant, 1 = Replicate. ratios[0 ..
 * n_ratios) are the up-sampling ratios from latent to waveform (the encoder uses them reversed). */
typedef struct svl_seanet_config {
  int32_t dimension, channels, n_filters, n_residual_layers;
  int32_t kernel_size, residual_kernel_size, last_kernel_size, dilation_base;
  int32_t pad_mode, compress, n_ratios;
  int32_t ratios[8];
  int32_t _pad;
} svl_seanet_config;
/* ProjectedTransformerConfig (nn/mimi.rs:18-29); layer scale is always on (mimi.rs:97). */
typedef struct svl_projected_transformer_config {
  int32_t d_model, input_dimension, output_dimension, num_heads, num_layers, context;
  int32_t dim_feedforward, _pad;
  double max_period;
} svl_projected_transformer_config;
/* MimiConfig (nn/mimi.rs:36-51). parts: SVL_MIMI_ENCODER | SVL_MIMI_DECODER, the halves to
 * load (the STT path needs only the encoder, the TTS path the decoder). */
#define SVL_MIMI_ENCODER 1
#define SVL_MIMI_DECODER 2
typedef struct svl_mimi_config {
  int32_t sample_rate, inner_dim, outer_dim, exact_gelu, parts, _pad;
  double frame_rate;
  svl_seanet_config encoder, decoder;
  svl_projected_transformer_config encoder_transformer, decoder_transformer;
} svl_mimi_config;
typedef struct svl_mimi svl_mimi;
typedef struct svl_mimi_state svl_mimi_state;
typedef struct svl_rvq svl_rvq;

/* MimiEncoder::new / MimiDecoder::new (nn/mimi.rs:140-166, :229-251) on `device`, from f32
 * tensors named as the reference's load_mimi_weights leaves them (nn/mod.rs:26-52):
 * "encoder.model.{i}.conv.weight", "encoder_transformer.transformer.layers.{l}...",
 * "downsample.conv.conv.weight", "upsample.convtr.convtr.weight", "decoder.model.{i}...". */
SVL_API svl_status svl_mimi_create(const svl_mimi_config* cfg, const svl_tensor_view* tensors,
                                   int32_t n_tensors, int32_t device, svl_mimi** out);
SVL_API void svl_mimi_destroy(svl_mimi* mimi);
/* Audio samples per codec frame (MimiConfig::frame_size, nn/mimi.rs:55-57). */
SVL_API int32_t svl_mimi_frame_size(const svl_mimi* mimi);
/* MimiEncoder::init_state and MimiDecoder::init_state (nn/mimi.rs:172-178, :253-259) for
 * max_batch streams, each call moving at most max_frames codec frames per stream. */
SVL_API svl_status svl_mimi_state_create(svl_mimi* mimi, int32_t max_batch, int32_t max_frames,
                                         svl_mimi_state** out);
SVL_API void svl_mimi_state_destroy(svl_mimi_state* state);
/* A fresh state for one stream, or every stream when stream < 0. */
SVL_API svl_status svl_mimi_state_reset(svl_mimi_state* state, int32_t stream);
/* MimiEncoder::encode_step (nn/mimi.rs:184-191) for streams 0..batch-1, device buffers:
 * d_pcm [batch][channels][frames * frame_size] in, d_latent [batch][inner_dim][frames] out
 * (unquantised latents at the codec frame rate), enqueued on cuda_stream (NULL = the codec's
 * stream). */
SVL_API svl_status svl_mimi_encode_step_device(svl_mimi* mimi, svl_mimi_state* state,
                                               int32_t batch, int32_t frames, const float* d_pcm,
                                               float* d_latent, void* cuda_stream);
/* MimiDecoder::decode_step (nn/mimi.rs:262-271) for streams 0..batch-1, device buffers:
 * d_latent [batch][outer_dim][frames] in, d_pcm [batch][channels][frames * frame_size] out. */
SVL_API svl_status svl_mimi_decode_step_device(svl_mimi* mimi, svl_mimi_state* state,
                                               int32_t batch, int32_t frames,
                                               const float* d_latent, float* d_pcm,
                                               void* cuda_stream);
/* Tts::decode_latent (tts/mod.rs:441-447) for streams 0..batch-1: d_latent
 * [batch][frames][latent_dim] (FlowLm::step's output layout), times d_emb_std plus d_emb_mean
 * ([latent_dim] each, the flow LM's "emb_std" / "emb_mean"; both NULL to skip), through the
 * latent projection "quantizer.output_proj.weight" [outer_dim][latent_dim][1] (loaded by
 * svl_mimi_create when present), then MimiDecoder::decode_step into d_pcm
 * [batch][channels][frames * frame_size]. Device buffers on cuda_stream. */
SVL_API svl_status svl_mimi_decode_latent_device(svl_mimi* mimi, svl_mimi_state* state,
                                                 int32_t batch, int32_t frames,
                                                 const float* d_latent, const float* d_emb_std,
                                                 const float* d_emb_mean, float* d_pcm,
                                                 void* cuda_stream);
/* The latent width of the loaded latent projection (0 without one). */
SVL_API int32_t svl_mimi_latent_dim(const svl_mimi* mimi);
/* Quantizer::new (stt/model.rs:92-98): n_q codebooks of `bins` entries from the tensors
 * "quantizer.rvq_first.input_proj.weight" [256][512][1],
 * "quantizer.rvq_first.vq.layers.0._codebook.{embedding_sum,cluster_usage}" and the same under
 * "quantizer.rvq_rest" (layers 0..n_q-2); entries are embedding_sum / max(cluster_usage, 1e-5). */
SVL_API svl_status svl_rvq_create(int32_t n_q, int32_t bins, const svl_tensor_view* tensors,
                                  int32_t n_tensors, int32_t device, svl_rvq** out);
SVL_API void svl_rvq_destroy(svl_rvq* rvq);
/* Quantizer::encode (stt/model.rs:100-103): d_latent [batch][512][frames] in, d_codes
 * [batch][frames][n_q] out (nearest entry per codebook, lowest index on ties), device buffers
 * on cuda_stream (NULL = the quantizer's stream). */
SVL_API svl_status svl_rvq_encode_device(svl_rvq* rvq, int32_t batch, int32_t frames,
                                         const float* d_latent, uint32_t* d_codes,
                                         void* cuda_stream);

/* Message of the last failure on this thread ("" when none). */
SVL_API const char* svl_last_error(void);
SVL_API const char* svl_version(void);

#ifdef __cplusplus
}
#endif
#endif
