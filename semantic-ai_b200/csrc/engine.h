// engine.h — host side of the B200 streaming LM step: weights on the device, per-stream KV
// rings, and the step as a sequence of kernels captured once per batch size in a CUDA
// graph. Mirrors the reference's types: Transformer / TransformerState
// (nn/transformer.rs:43-104), LanguageModel (stt/model.rs:176-186) and FlowLm
// (tts/flow_lm.rs:24-42).
#pragma once

#include <cuda_runtime.h>

#include <map>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/svl_cuda.h"
#include "common.cuh"
#include "kernels.cuh"

namespace svl {

// An error carrying the C-ABI status it maps to.
struct Error : std::runtime_error {
  svl_status code;
  Error(svl_status c, const std::string& m) : std::runtime_error(m), code(c) {}
};

void check_cuda(cudaError_t e, const char* what);

// Owning device allocation.
struct DevBuf {
  void* p = nullptr;
  size_t bytes = 0;
  DevBuf() = default;
  DevBuf(const DevBuf&) = delete;
  DevBuf& operator=(const DevBuf&) = delete;
  DevBuf(DevBuf&& o) noexcept : p(o.p), bytes(o.bytes) { o.p = nullptr; o.bytes = 0; }
  DevBuf& operator=(DevBuf&& o) noexcept;
  ~DevBuf();
  void alloc(size_t n);
  template <class T> T* as() const { return static_cast<T*>(p); }
};

// Owning pinned host allocation (staging for the host-buffer entry points).
struct HostBuf {
  void* p = nullptr;
  size_t bytes = 0;
  HostBuf() = default;
  HostBuf(const HostBuf&) = delete;
  HostBuf& operator=(const HostBuf&) = delete;
  ~HostBuf();
  void alloc(size_t n);
  template <class T> T* as() const { return static_cast<T*>(p); }
};

struct Linear {
  int n = 0, k = 0, wtype = W_F32;
  int64_t row_stride = 0;
  int interleave = 0;
  DevBuf w;
  DevBuf bias;  // f32 [n] or empty
  GemmOperand tc;  // TMA map of the bf16 weights for the tensor-core path
  DevBuf shadow;   // Q8_0 / Q4_1: the bf16 image of the dequantised weights (tensor cores)
  int64_t bytes() const { return row_stride * n + (bias.p ? 4LL * n : 0); }
};

struct Norm {
  int kind = NORM_NONE;
  float eps = 0.f;
  DevBuf w, b;
};

struct Layer {
  Norm norm1, norm2;
  Linear in_proj, out_proj, ff1, ff2;
  DevBuf ls1, ls2;
};

struct TimeEmbed {
  DevBuf freqs;  // [128]
  Linear l1, l2;
  DevBuf alpha;
};

struct ResBlock {
  Norm ln;
  Linear mlp1, mlp2, mod;
};

struct Model {
  int kind = 0;  // 0 STT LanguageModel, 1 Pocket-TTS FlowLm, 2 bare transformer
  int device = 0;
  svl_transformer_config cfg{};
  svl_stt_config stt{};
  svl_tts_config tts{};
  std::vector<Layer> layers;
  DevBuf inv_freq;
  // STT
  DevBuf text_emb, audio_emb;
  int tables_bf16 = 0;
  Norm out_norm;
  Linear text_linear;
  std::vector<Linear> extra;
  // TTS
  DevBuf cond_table;             // conditioner rows [text_bins + 1][d]
  Linear input_linear;
  DevBuf eos_w, eos_b;           // out_eos [d] and its bias [1]
  DevBuf bos;                    // bos_emb [latent]
  std::vector<TimeEmbed> time_emb;
  Linear cond_embed, input_proj, final_mod, final_linear;
  std::vector<ResBlock> res;
  // Every ResBlock's adaLN_modulation rows, then the final layer's, stacked into one product
  // (they all read the same conditioning): rows [3 dim i, 3 dim (i + 1)) are block i's,
  // the last 2 dim the final layer's.
  Linear mods;
  int64_t weight_bytes = 0;
  bool shadows = false;  // quantised linears have bf16 images for the tensor-core path
  std::mutex shadow_mu;
  cudaStream_t stream = nullptr;
  ~Model();
};

struct State {
  Model* m = nullptr;
  int max_batch = 0, cap = 0, windowed = 0;
  int kv_elt = 4;
  int64_t ring_stream_stride = 0;  // elements per stream per layer
  int64_t ring_layer_stride = 0;   // elements per layer
  DevBuf k_ring, v_ring;
  DevBuf pos;
  std::vector<int> hpos;
  // work buffers
  DevBuf x, q, attn, act, logits, extra_logits, extra_p;
  DevBuf tok_in, audio_in, tok_out;
  DevBuf am_val, am_idx, am_ticket, err;
  DevBuf frames_audio, frames_out, frames_extra;  // svl_stt_run_frames
  // TTS work buffers
  DevBuf latent_in, noise, latent_out, eos, z, y, sy, hbuf, h2buf, modbuf, xs2, tmp;
  DevBuf temb_in, temb_h, temb_o, prompt_tok;
  // TTS: the flow head's summed timestep embeddings, [decode step][flow_dim] per number of
  // decode steps (they depend on nothing else, so they are computed once).
  std::map<int, DevBuf> time_tables;
  std::map<int64_t, GemmOperand> xa_by_k;  // bf16 operand maps over xa, keyed by k * 512 + bn
  HostBuf h_tok_in, h_audio_in, h_tok_out, h_err;
  int splits = 1;
  // Many-stream attention (splits == 1): keys per piece, pieces per unit at most, and the
  // partials of the units of several pieces.
  int piece = 0, npieces = 0;
  DevBuf attn_part;
  // Few streams with short windows: flat chunks merged by the last CTA of each unit (the
  // tickets, [max_batch][heads], zero between launches; partials in attn_part).
  bool attn_flat = false;
  DevBuf attn_ticket;
  alignas(64) unsigned char kmap[128], vmap[128];  // bf16 rings as TMA tensors
  bool ring_maps = false;
  // Tensor-core path (bf16 weights, many streams): bf16 operand rows and their TMA maps, per
  // stream-tile width (64, 128, 256). xa holds normalised inputs / attention outputs, xh the
  // feed-forward hidden rows.
  DevBuf xa, xh, gemm_ws;
  DevBuf rope_cs;  // [max_batch][head_dim / 2] float2, refreshed at the start of every forward
  GemmOperand xa_d[3], xa_q[3], xh_f[3];
  std::map<int, cudaGraphExec_t> graphs;
  std::map<int, int> graph_kernels;  // kernel nodes of each captured step graph
  // Reference order (SVL_STATE_REFERENCE_ORDER at creation): every reduction whose
  // order the reference's CPU path fixes runs in that order -- norm sums element by element,
  // attention key by key, RoPE from a host table of the C library's cosf / sinf -- so the
  // step reproduces the reference CPU arithmetic bit for bit; the weight products always
  // do. The matrix-vector kernels serve every batch size in this mode.
  bool ref_order = false;
  DevBuf rope_tab;         // [rope_positions][head_dim / 2] (cos, sin)
  int rope_positions = 0;
  bool test_withheld_copy = false;  // SVL_STATE_TEST_WITHHELD_COPY: the bounded-wait drill
  ~State();
};

// Parameter blocks of one layer's kernels (see layer_params).
struct LayerParams {
  GemvParams in_proj, out_proj, ff1, ff2;
  AttnParams attn;
};

// Streams from which a step's weight products run on the tensor cores (bf16 weights).
constexpr int kGemmMinBatch = 16;
bool use_tensor_cores(const Model& m, const State& s, int nb);

// The state's device error flag: queue its read (before the stream synchronises), then raise
// it as an Error after the synchronisation (1: an id out of range on the device, 2 / 3: a
// bounded device wait ran out). The flag is cleared when raised.
void queue_error_read(State& s, cudaStream_t st);
void raise_device_error(State& s, cudaStream_t st);

// Weight loading (LanguageModel::new / FlowLm::new).
// kind 0 STT LanguageModel, 1 Pocket-TTS FlowLm, 2 a bare transformer whose tensors are
// named under `prefix` (Mimi's transformers).
Model* create_model(int kind, const svl_transformer_config& cfg, const svl_stt_config* stt,
                    const svl_tts_config* tts, const svl_tensor_view* t, int n, int device,
                    const char* prefix = nullptr);
State* create_state(Model* m, int max_batch, int max_positions, uint32_t flags = 0);

// The step kernels for streams [b0, b0 + nb) (no embedding / head).
void enqueue_layers(Model& m, State& s, int b0, int nb, cudaStream_t st);
// The whole STT step for streams [0, nb): embed tok_in/audio_in, layers, head into tok_out.
void enqueue_stt_step(Model& m, State& s, int nb, cudaStream_t st);
// Runs the captured graph of the STT step for nb streams (captures it on first use).
void launch_stt_graph(Model& m, State& s, int nb, cudaStream_t st);
// Captures the step graph of batch size nb if it is not captured yet; returns its kernels.
int capture_stt_graph(Model& m, State& s, int nb, cudaStream_t st);
// FlowLm::step (tts/flow_lm.rs:162-185) for streams [0, nb) from the state's latent_in /
// noise buffers into latent_out / eos, as one graph per (nb, decode_steps).
void launch_tts_graph(Model& m, State& s, int nb, int decode_steps, cudaStream_t st);
int capture_tts_graph(Model& m, State& s, int nb, int decode_steps, cudaStream_t st);
// FlowLm::prompt_text (tts/flow_lm.rs:150-158) for streams [b0, b0 + nb): n tokens each,
// device tokens [nb][n].
void enqueue_tts_prompt(Model& m, State& s, int b0, int nb, const uint32_t* d_tokens, int n,
                        cudaStream_t st);
// Profiling: one repetition of the step's weight products (which 0) or attention (which 1).
int64_t enqueue_profile(Model& m, State& s, int nb, int which, cudaStream_t st);
void enqueue_tts_step(Model& m, State& s, int nb, int decode_steps, bool bos, cudaStream_t st);

void state_reset(State& s, int stream);
// Message of the last failure on this thread (svl_last_error).
void set_last_error(const std::string& msg);
void state_export(State& s, int stream, int layer, float* k, float* v, int* len);
void state_import(State& s, int stream, int layer, const float* k, const float* v, int len,
                  int position);
// Voice::save / Voice::load (tts/voice.rs:78-149), voice.cu.
void voice_save(State& s, int stream, const char* path);
void voice_load(State& s, const int* streams, int n, const char* path);

}  // namespace svl

// The C ABI's opaque handles.
struct svl_model {
  svl::Model* m;
};
struct svl_state {
  svl::State* s;
  svl_model* model;
};
