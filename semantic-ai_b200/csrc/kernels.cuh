// kernels.cuh — parameter blocks and launchers of the step kernels (host/device shared).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace svl {

// CTAs of a logits product: the argmax scratch holds one (value, index) pair per CTA.
constexpr int kLogitsGrid = 296;
// Streams one product launch covers at most (the argmax scratch is [kMaxNbChunk][kLogitsGrid]).
constexpr int kMaxNbChunk = 8;
// Audio codebooks the embedding kernel stages per stream.
constexpr int kMaxCodebooks = 127;

// An L2 prefetch of a later kernel's data: every CTA of the kernel that carries it pulls its
// share of [p, p + bytes) into L2 (cp.async.bulk.prefetch.L2), so the later kernel's reads
// hit L2 instead of waiting on HBM.
struct PrefetchRange {
  const uint8_t* p;
  int64_t bytes;
};
constexpr int kMaxPrefetch = 3;

enum GemvEpilogue {
  EPI_STORE = 0,     // out = acc (+ bias)
  EPI_RESIDUAL = 1,  // out += (acc (+ bias)) * layer_scale
  EPI_QKV_ROPE = 2,  // RoPE on q,k; q to a buffer, k and v into the KV ring
  EPI_SWIGLU = 3,    // rows interleaved gate/value: out[i] = silu(gate) * value
  EPI_GELU_TANH = 4, // out = gelu_tanh(acc (+ bias))
  EPI_GELU_ERF = 5,
  EPI_LOGITS = 6,    // out = acc (+ bias), plus greedy argmax into tokens
  EPI_SILU = 7       // out = silu(acc (+ bias))
};

// One matrix-vector product over `nb` streams: out[b] = epilogue(W · norm(x[b])). Every CTA
// normalises and converts the input rows itself (see gemv.cu), while its first weight loads
// are in flight.
struct GemvParams {
  const uint8_t* w;      // device weights in the packed layout of `wtype`
  int64_t row_stride;    // bytes between rows
  int n, k;              // rows (outputs) and columns (inputs)
  int wtype;             // WeightType
  const float* x;        // [nb][x_stride] f32 inputs
  int64_t x_stride;
  int nb;
  int norm;              // NormKind applied to x first
  const float* norm_w;
  const float* norm_b;
  float eps;
  const float* bias;     // [n] or null
  int epi;
  float* out;            // [nb][out_stride]
  int64_t out_stride;
  const float* ls;       // layer scale [n] or null (EPI_RESIDUAL)
  // EPI_QKV_ROPE
  const float* inv_freq; // [head_dim / 2]
  const float2* rope_cs; // [nb][head_dim / 2] (cos, sin) of pos * inv_freq (tensor-core path)
  const int* pos;        // [nb] absolute positions of the new token
  int q_dim, kv_dim, head_dim;
  int ring_cap;          // KV slots per stream and head
  int windowed;          // slot = pos % ring_cap when set, else pos
  void* k_ring;          // [nb][kv_heads][ring_cap][head_dim], f32 or bf16
  void* v_ring;
  int64_t ring_stream_stride;  // elements between streams
  int kv_bf16;
  // EPI_LOGITS
  float* am_val;         // [nb][grid] scratch
  int* am_idx;           // [nb][grid] scratch
  unsigned* am_ticket;   // one counter, zero between launches
  uint32_t* tokens;      // [nb] argmax out
  int* pos_advance;      // [nb] positions to advance once the argmax is final, or null
  PrefetchRange pf[kMaxPrefetch];  // L2 prefetches of later kernels' data
  // Reference order (a state option): the norm sums run element by element on one thread,
  // as on the reference CPU path, instead of as a parallel reduction.
  int ref_order;
  // EPI_QKV_ROPE with a cos / sin table: rope_by_pos[pos][i] = (cos, sin)(pos * inv_freq[i])
  // for pos < rope_positions, evaluated on the host with the C library's cosf / sinf (the
  // functions the reference's CPU path calls); null = sincosf on the device.
  const float2* rope_by_pos;
  int rope_positions;
  // Set to 2 when a bounded device-side wait runs out (null: not reported).
  int* err;
  // Failure drill (quantised products): CTA 0 withholds its first staged copy and waits at
  // most wait_limit rounds for it (0: the default limit).
  int test_withhold;
  uint32_t wait_limit;
};

void launch_gemv(const GemvParams& p, cudaStream_t s);
// Kernel launches one launch_gemv(p) issues (streams are split into chunks that fit).
int gemv_launches(const GemvParams& p);
// Per device, once: raises the dynamic shared-memory limit of every product kernel.
void gemv_init_device();

// A bf16 GEMM operand in global memory: rows of k elements, row_bytes apart, described by a
// TMA tensor map whose box is 64 elements (128 bytes, 128-byte swizzle) by box_rows rows.
struct GemmOperand {
  alignas(64) unsigned char map[128];  // CUtensorMap
  int rows = 0, k = 0, box_rows = 0;
  int f16 = 0;  // element type: 0 bf16, 1 f16 (both operands of a product share it)
  bool valid = false;
};
bool make_gemm_operand(GemmOperand& op, const void* base, int rows, int k, int64_t row_bytes,
                       int box_rows, int f16 = 0);
// A bf16 KV ring as a 3-D tensor [layers][rows][head_dim] (rows = streams x kv_heads x slots,
// layer_stride elements apart) for TMA boxes of 64 dims x box_rows rows, 128-byte swizzle.
bool make_ring_map(unsigned char* map128, const void* base, int64_t rows, int head_dim, int layers,
                   int64_t layer_stride, int box_rows);
// Keys per chunk of the many-stream attention (the box height of its ring maps).
int attention_chunk_keys(int head_dim, int kv_bf16);
// Streams per GEMM tile (the MMA's N, and the box height of the X operand) for nb streams.
int gemm_stream_tile(int nb);
// Cluster split of K for an n x k product over nb streams with stream tiles of bn.
int gemm_split(int n, int k, int nb, int bn);
// out[b] = epilogue(W . X[x_row0 + b]) for b < p.nb on the tensor cores; p gives the sizes
// and the epilogue (p.x / p.norm are not read: X is the bf16 operand). out_bf16 writes the
// STORE / SWIGLU / GELU / SILU outputs as bf16. err is set to 2 if a bounded wait ran out.
// ws: the split-K exchange, gemm_workspace_bytes() of device memory.
void launch_gemm(const GemvParams& p, const GemmOperand& w, const GemmOperand& x, int x_row0,
                 int out_bf16, int* err, float* ws, cudaStream_t s);
size_t gemm_workspace_bytes();
// The norm of each of nb rows of x (NormKind), as bf16 (or f16) rows of the GEMM operand.
// quant: the rows first go through the Q8 activation blocks of the quantised products
// (quantised models, whose operands are f16).
void launch_prep_bf16(const float* x, int64_t x_stride, int nb, int norm, const float* norm_w,
                      const float* norm_b, float eps, int k, void* out, int64_t out_stride,
                      cudaStream_t s, int quant = 0, int f16 = 0);
// bf16 / f16 images of dequantised weights (launch_dequant_bf16 with f16 = 1 writes f16).
void gemm_init_device();

struct AttnParams {
  const float* q;        // [nb][heads][head_dim] (after RoPE)
  const void* k_ring;    // [nb][kv_heads][ring_cap][head_dim]
  const void* v_ring;
  int64_t ring_stream_stride;
  int kv_bf16;
  const int* pos;        // [nb] position of the newest key (already written)
  int nb, heads, kv_heads, head_dim, ring_cap, window;  // window 0 = unlimited
  float scale;
  int splits;            // key chunks per (stream, head): one thread-block cluster
  float* out;            // [nb][heads * head_dim]
  int* err;              // set to 4 when a bounded wait runs out
  // Many streams (splits == 1): keys per piece, pieces per unit at most, and the partials
  // [nb][heads][npieces][head_dim + 4] of the units of several pieces.
  int piece, npieces;
  float* part;
  // Few streams (attn_flat_kernel, when set): one ticket per (stream, head) unit, zero between
  // launches, and the chunks' partials [nb][heads][splits][head_dim + 4] in `part`.
  unsigned* ticket;
  // Tensor-map view of bf16 rings (make_ring_map): host copies of the maps of k_ring's and
  // v_ring's whole allocations, this layer's index in them, and the map row of stream 0's slot 0.
  const unsigned char* kmap;
  const unsigned char* vmap;
  int layer, ring_row0;
  PrefetchRange pf[kMaxPrefetch];  // L2 prefetches of later kernels' data
};

void launch_attention_decode(const AttnParams& p, cudaStream_t s);
int attention_max_splits();
// Keys per chunk at most of the flat few-stream attention (attn_flat_kernel).
int attention_flat_max_keys();
// Keys per piece of the many-stream attention for a ring of `ring_cap` keys; *npieces = the
// most pieces a (stream, head) can have.
int attention_piece(int head_dim, int kv_bf16, int ring_cap, int* npieces);
// Per device, once: raises the dynamic shared-memory limit of the attention kernels.
void attention_init_device();
// Decode attention in the reference CPU path's order (attention_ref.cu), for reference-order
// states: the same inputs and output as launch_attention_decode (splits, pieces and maps are
// not used). Supported for head_dim 64 / 128 and rings of up to 51,200 keys.
void launch_attention_ref(const AttnParams& p, cudaStream_t s);
bool attention_ref_supported(int head_dim, int ring_cap);
void attention_ref_init_device();

struct EmbedParams {
  const void* text_table;   // [text_card + 1][d]
  const void* audio_tables; // [n_q][card + 1][d]
  int tables_bf16;
  const uint32_t* text_tok; // [nb]
  const uint32_t* audio_tok;// [nb][n_q]
  int nb, d, n_q, card, text_card;
  float* x;                 // [nb][d]
  int* error_flag;          // set to 1 on an out-of-range id
};

void launch_embed(const EmbedParams& p, cudaStream_t s);
void launch_advance_positions(int* pos, int nb, cudaStream_t s);
// cs[b][i] = (cos, sin)(pos[b] * inv_freq[i]) for the streams' new tokens: one evaluation per
// (stream, frequency) per step, shared by every layer's RoPE epilogue.
void launch_rope_table(const int* pos, int nb, const float* inv_freq, int half, float2* cs,
                       cudaStream_t s);

// Weight packing: f32 [n][k] (device) into the layout of wtype. interleave_half = F swaps
// rows so that packed row 2i is source row i and 2i+1 is source row F + i (SwiGLU).
void launch_pack_linear(const float* src, uint8_t* dst, int64_t row_stride, int n, int k,
                        int wtype, int interleave_half, cudaStream_t s);
void launch_f32_to_bf16(const float* src, void* dst, int64_t n, cudaStream_t s);
// bf16 rows (dst_stride bytes apart) holding the dequantised values of a packed Q8_0 / Q4_1
// matrix.
void launch_dequant_bf16(const uint8_t* src, int64_t row_stride, int n, int k, int wtype, void* dst,
                         int64_t dst_stride, cudaStream_t s, int f16 = 0);
void launch_round_bf16_inplace(float* p, int64_t n, cudaStream_t s);

int64_t packed_row_stride(int wtype, int k);

// Pocket-TTS step pieces (tts.cu).
void launch_tts_head(const float* x, int nb, int d, const float* lnw, const float* lnb, float eps,
                     const float* w_eos, const float* b_eos, float* z, float* eos, cudaStream_t s);
void launch_time_input(const float* freqs, float t, float* emb, cudaStream_t s);
void launch_time_norm(const float* te, int dim, const float* alpha, float* tsum, int first,
                      cudaStream_t s);
void launch_cond_silu(const float* y, const float* tsum, float inv_n, int dim, int nb, float* sy,
                      cudaStream_t s);
void launch_adaln(const float* xs, int nb, int dim, const float* lnw, const float* lnb, int affine,
                  float eps, const float* mod, int64_t mod_stride, float* hh, cudaStream_t s);
void launch_gate_add(float* xs, const float* mod, int64_t mod_stride, int gate_off, const float* h,
                     int nb, int dim, cudaStream_t s);
void launch_flow_update(float* x, const float* flow, int64_t n, int mode, float scale,
                        cudaStream_t s);
void launch_prompt_embed(const float* table, const uint32_t* tokens, int nb, int n, int t, int d,
                         int bins, float* x, int* err, cudaStream_t s);

}  // namespace svl
