// codec.cu — Mimi, the codec on both sides of the language models, on the GPU.
//
// Replaces, for many streams at once, the reference's CPU codec path:
//  - StreamingConv1d / StreamingConvTranspose1d (nn/conv.rs:22-335) with the im2col and
//    overlap-add kernels (nn/kernels/conv.rs:8-166) and ELU (nn/kernels/activation.rs:60-67);
//  - SEANet encoder / decoder (nn/seanet.rs:126-245) and its resnet blocks (:36-73);
//  - MimiEncoder::encode_step / MimiDecoder::decode_step (nn/mimi.rs:140-272): SEANet, the
//    ProjectedTransformer (:66-123, run by the step engine as a bare transformer) and the learnt
//    down/up-sampling;
//  - Quantizer::encode (stt/model.rs:84-170): the split residual vector quantizer that turns
//    encoder latents into the STT model's audio tokens.
//
// Layout: activations are channel-first [stream][channel][time] like the reference's
// tensors; each convolution keeps, per stream, the input samples it still needs
// ([channel][context], the reference's Conv1dState) and a transposed convolution the
// overlapping outputs of the previous chunk ([channel][overlap], ConvTranspose1dState).
//
// Arithmetic: f32 on the CUDA cores, as the reference's f32 CPU path. Each convolution output
// is one sequential FMA chain over (input channel, tap) in the order of the reference's im2col
// columns, then + bias, then the resnet skip; a transposed convolution's output is bias +
// previous partial + its taps in tap order, as overlap_add adds them. The RVQ distances are
// sequential FMA chains over the 256 dimensions. The matrix products inside candle (gemm
// crate) have their own blocking, so these orders are a restatement, not a bit-for-bit pin.
#include <algorithm>
#include <climits>
#include <cmath>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "engine.h"
#include "sm100.cuh"

namespace svl {
namespace {

constexpr int ACT_NONE = 0, ACT_ELU = 1, ACT_AFFINE = 2;  // ACT_AFFINE: x * scale[c] + shift[c]
constexpr int kConvThreads = 256;
constexpr int kConvSmem = 46 * 1024;  // under the 48 KB default: no opt-in needed

// exp_parts of the reference's exp (nn/kernels/mod.rs:96-131): x = k ln2 + r (Cody-Waite, two-
// part ln2), expm1(r) by its degree-8 Taylor polynomial, 2^k from the exponent field.
__device__ __forceinline__ void exp_parts_dev(float x, float& two_k, float& expm1_r) {
  const float LN2_HI = 0.69314575f;
  const float LN2_LO = 1.4286068e-6f;
  const float ROUND = 12582912.0f;
  const float LOG2E = 1.44269504088896340736f;
  const float shifted = fmaf(x, LOG2E, ROUND);
  const float k = __fsub_rn(shifted, ROUND);
  const int k_int = (int)(__float_as_uint(shifted) - __float_as_uint(ROUND));
  const float r = fmaf(-k, LN2_LO, fmaf(-k, LN2_HI, x));
  float p = 1.0f / 40320.0f;
  p = fmaf(p, r, 1.0f / 5040.0f);
  p = fmaf(p, r, 1.0f / 720.0f);
  p = fmaf(p, r, 1.0f / 120.0f);
  p = fmaf(p, r, 1.0f / 24.0f);
  p = fmaf(p, r, 1.0f / 6.0f);
  p = fmaf(p, r, 0.5f);
  p = fmaf(p, r, 1.0f);
  two_k = __uint_as_float((uint32_t)(k_int + 127) << 23);
  expm1_r = __fmul_rn(p, r);
}

// Activation::Elu (nn/kernels/activation.rs:60-67): x above 0, else 2^k expm1(r) + (2^k - 1)
// of x clamped to [-20, 0] (NaN stays NaN, as f32::clamp keeps it).
__device__ __forceinline__ float elu_ref(float x) {
  if (x != x) return x;
  if (x > 0.f) return x;
  float two_k, e;
  exp_parts_dev(fminf(fmaxf(x, -20.0f), 0.0f), two_k, e);
  return fmaf(two_k, e, __fsub_rn(two_k, 1.0f));
}

// One StreamingConv1d::forward over `nb` streams (streams b0 .. b0 + nb - 1 of the state).
struct ConvArgs {
  const float* x;  // input chunk [b][cin][t]: stream stride x_bs, channel stride x_cs, time stride x_ts
  int64_t x_bs;
  int x_cs, x_ts, t;
  const float* in_scale;  // ACT_AFFINE: per input channel
  const float* in_shift;
  float* prev;  // state [stream][cin][ctx]
  const int* started;  // [stream]: 0 before the stream's first chunk
  int b0, ctx;
  int cin, cout, k, stride, dil, act, replicate;
  const float* w;     // transposed: [cin * k][cout]
  const float* bias;  // [cout] or null
  const float* skip;  // resnet skip [b][cout][len] with the output's strides, or null
  float* out;         // [b][cout][len]
  int64_t o_bs;
  int o_cs, len;
};

// Value i of the convolution's input [previous context | act(chunk)] for stream b, channel c.
__device__ __forceinline__ float conv_act(const ConvArgs& a, int c, float v) {
  if (a.act == ACT_ELU) return elu_ref(v);
  if (a.act == ACT_AFFINE) return __fadd_rn(__fmul_rn(v, a.in_scale[c]), a.in_shift[c]);
  return v;
}
__device__ __forceinline__ float conv_in(const ConvArgs& a, int b, int c, int i, bool started) {
  if (i >= a.ctx) return conv_act(a, c, a.x[b * a.x_bs + (int64_t)c * a.x_cs + (int64_t)(i - a.ctx) * a.x_ts]);
  if (started) return a.prev[((int64_t)(a.b0 + b) * a.cin + c) * a.ctx + i];
  if (!a.replicate) return 0.f;  // PadMode::Constant: zeros before the first chunk
  return conv_act(a, c, a.x[b * a.x_bs + (int64_t)c * a.x_cs]);  // PadMode::Replicate: the first sample
}

// CTA tile: 64 output channels x 64 columns, a column being one output time of one stream
// (column q = stream q / len, time q % len: short chunks of many streams share one tile, so a
// staged weight serves every stream of it). 256 threads in a 16 x 16 grid, each computing a
// 4 x 4 register block (channels o..o+3, columns q..q+3). Chunks of input channels are staged
// in shared memory as im2col rows, both operands [channel * k + tap][64]: the weights from the
// layer's transposed copy [cin * k][cout] and the inputs gathered per column from
// [carried context | act(chunk)]; the inner loop reads one float4 of each for 16 FMAs. Every
// output is one FMA chain over (channel, tap) in order.
constexpr int kConvTile = 64;

__global__ void __launch_bounds__(kConvThreads) conv1d_kernel(const ConvArgs a, int cc_max, int nb, int cpc,
                                                             float* partial) {
  constexpr int T = kConvTile, G = T / 4;
  extern __shared__ __align__(16) float sm[];
  float* ws = sm;                      // [cc_max * k][T]
  float* xsm = sm + cc_max * a.k * T;  // [cc_max * k][T]
  const int o0 = blockIdx.y * T, q0 = blockIdx.x * T, ncol = nb * a.len;
  const int tid = threadIdx.x, og = tid % G, cg = tid / G;
  const int total = a.ctx + a.t;
  // The reduction in chunks of cpc input channels (kConvChunkTerms / k): this CTA sums every
  // chunk in order (partial null), or only chunk blockIdx.z into `partial`.
  const int nchunks = (a.cin + cpc - 1) / cpc;
  const int z0 = partial ? blockIdx.z : 0, z1 = partial ? blockIdx.z + 1 : nchunks;
  float acc[4][4], sum[4][4];
  for (int z = z0; z < z1; z++) {
#pragma unroll
  for (int u = 0; u < 4; u++)
#pragma unroll
    for (int i = 0; i < 4; i++) acc[u][i] = 0.f;
  const int cz1 = min(a.cin, (z + 1) * cpc);
  for (int c0 = z * cpc; c0 < cz1; c0 += cc_max) {
    const int cc = min(cc_max, cz1 - c0), ck = cc * a.k;
    __syncthreads();
    for (int i = tid; i < ck * T; i += kConvThreads) {
      const int r = i / T, o = i - r * T;
      ws[i] = o0 + o < a.cout ? a.w[((int64_t)c0 * a.k + r) * a.cout + o0 + o] : 0.f;
    }
    // The gather: column-fastest walks one stream's time axis when a tile holds a single
    // stream's outputs (long chunks); tap-fastest keeps a warp on contiguous samples of one
    // stream's window when the tile's columns jump between streams (short chunks).
    const bool tap_fast = a.len < T;
    for (int i = tid; i < ck * T; i += kConvThreads) {
      int r, col;
      if (tap_fast) {
        const int j = i % a.k, rest = i / a.k;
        col = rest % T;
        r = (rest / T) * a.k + j;
      } else {
        r = i / T;
        col = i - r * T;
      }
      const int q = q0 + col;
      float v = 0.f;
      if (q < ncol) {
        const int b = q / a.len, l = q - b * a.len, c = r / a.k, j = r - c * a.k;
        const int pos = l * a.stride + j * a.dil;
        if (pos < total) v = conv_in(a, b, c0 + c, pos, a.started[a.b0 + b] != 0);
      }
      xsm[r * T + col] = v;
    }
    __syncthreads();
    const float* wb = ws + 4 * og;
    const float* xb = xsm + 4 * cg;
    for (int r = 0; r < ck; r++) {
      const float4 w4 = *reinterpret_cast<const float4*>(wb + r * T);
      const float4 x4 = *reinterpret_cast<const float4*>(xb + r * T);
      const float wv[4] = {w4.x, w4.y, w4.z, w4.w}, xv[4] = {x4.x, x4.y, x4.z, x4.w};
#pragma unroll
      for (int u = 0; u < 4; u++)
#pragma unroll
        for (int i = 0; i < 4; i++) acc[u][i] = fmaf(wv[u], xv[i], acc[u][i]);
    }
  }
#pragma unroll
  for (int u = 0; u < 4; u++)
#pragma unroll
    for (int i = 0; i < 4; i++) sum[u][i] = z == z0 ? acc[u][i] : __fadd_rn(sum[u][i], acc[u][i]);
  }  // chunks
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int q = q0 + 4 * cg + i;
    if (q >= ncol) continue;
    const int b = q / a.len, l = q - b * a.len;
#pragma unroll
    for (int u = 0; u < 4; u++) {
      const int o = o0 + 4 * og + u;
      if (o >= a.cout) continue;
      if (partial) {  // this chunk's sum, combined in chunk order by conv_combine_kernel
        partial[((int64_t)blockIdx.z * nb * a.cout + (int64_t)b * a.cout + o) * a.len + l] = sum[u][i];
        continue;
      }
      float v = sum[u][i];
      if (a.bias) v = __fadd_rn(v, a.bias[o]);  // matmul, then broadcast_add of the bias
      const int64_t off = b * a.o_bs + (int64_t)o * a.o_cs + l;
      if (a.skip) v = __fadd_rn(a.skip[off], v);  // ResnetBlock: xs + ys
      a.out[off] = v;
    }
  }
}

// The convolution's state after the chunk: the last ctx samples of [previous | act(chunk)]
// (nn/conv.rs:168-177). One thread per (stream, channel) walks its row upward, so reading
// position t + u (>= u) before writing u is safe in place.
__global__ void conv_state_kernel(const ConvArgs a, int nb) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nb * a.cin) return;
  const int b = i / a.cin, c = i - b * a.cin;
  const bool started = a.started[a.b0 + b] != 0;
  float* row = a.prev + ((int64_t)(a.b0 + b) * a.cin + c) * a.ctx;
  for (int u = 0; u < a.ctx; u++) row[u] = conv_in(a, b, c, a.t + u, started);
}

// The chunks' sums of a split convolution added in chunk order, then the bias and the skip.
__global__ void conv_combine_kernel(const ConvArgs a, const float* partial, int nchunks, int nb) {
  const int64_t n = (int64_t)nb * a.cout * a.len;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int l = (int)(i % a.len), o = (int)((i / a.len) % a.cout), b = (int)(i / ((int64_t)a.len * a.cout));
  float v = partial[i];
  for (int z = 1; z < nchunks; z++) v = __fadd_rn(v, partial[(int64_t)z * n + i]);
  if (a.bias) v = __fadd_rn(v, a.bias[o]);
  const int64_t off = b * a.o_bs + (int64_t)o * a.o_cs + l;
  if (a.skip) v = __fadd_rn(a.skip[off], v);
  a.out[off] = v;
}

// One StreamingConvTranspose1d::forward (nn/conv.rs:265-335) over nb streams: outputs
// [0, t * stride) are complete, [t * stride, t * stride + overlap) the new partial tail (written
// after the complete ones in the output rows, then moved into the state).
struct ConvTrArgs {
  const float* x;  // [b][cin][t]
  int64_t x_bs;
  int x_cs, t, act;
  float* partial;  // state [stream][cout][overlap]
  int b0, overlap;
  int cin, cout, k, stride, depthwise;
  const float* w;     // [cin][cout / groups][k]
  const float* bias;  // [cout] or null
  float* out;         // [b][cout][t * stride + overlap]
  int64_t o_bs;
  int o_cs;
};
constexpr int kTrMaxHits = 4;  // kernel <= 4 strides: taps landing on one output

// Output s of channel o (s < t * stride + overlap): (bias for complete outputs, else 0) +
// previous partial[s] (s < overlap) + the taps tap = s % stride + h stride from step
// s / stride - h, in tap order (the overlap_add of nn/kernels/conv.rs:117-166). A tap's value
// is prod[o * k + tap][step]: for an ungrouped layer the products were computed beforehand as
// one 1x1 convolution (each a single FMA chain over the input channels); for a depthwise one
// it is w[o][tap] x[o][step].
__global__ void convtr_add_kernel(const ConvTrArgs a, const float* prod, int nb) {
  const int complete = a.t * a.stride, total = complete + a.overlap;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)nb * a.cout * total) return;
  const int s = (int)(i % total), o = (int)((i / total) % a.cout), b = (int)(i / ((int64_t)total * a.cout));
  float v = s < complete && a.bias ? a.bias[o] : 0.f;
  if (s < a.overlap) v = __fadd_rn(v, a.partial[((int64_t)(a.b0 + b) * a.cout + o) * a.overlap + s]);
#pragma unroll
  for (int h = 0; h < kTrMaxHits; h++) {
    const int tap = s % a.stride + h * a.stride, step = s / a.stride - h;
    if (tap >= a.k || step < 0 || step >= a.t) continue;
    float p;
    if (a.depthwise) {
      float xv = a.x[b * a.x_bs + (int64_t)o * a.x_cs + step];
      if (a.act == ACT_ELU) xv = elu_ref(xv);
      p = __fmul_rn(a.w[(int64_t)o * a.k + tap], xv);
    } else {
      p = prod[(((int64_t)b * a.cout + o) * a.k + tap) * a.t + step];
    }
    v = __fadd_rn(v, p);
  }
  a.out[b * a.o_bs + (int64_t)o * a.o_cs + s] = v;
}

// The new partial: the tail outputs [t * stride, t * stride + overlap) of the chunk.
__global__ void convtr_state_kernel(const ConvTrArgs a, int nb) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nb * a.cout * a.overlap) return;
  const int u = i % a.overlap, bo = i / a.overlap, o = bo % a.cout, b = bo / a.cout;
  a.partial[((int64_t)(a.b0 + b) * a.cout + o) * a.overlap + u] =
      a.out[b * a.o_bs + (int64_t)o * a.o_cs + a.t * a.stride + u];
}

// ---- split residual vector quantizer (Quantizer::encode, stt/model.rs:100-170) -------------
//
// A row is one latent frame of one stream. A cluster of kRvqRanks CTAs takes R rows (8, or 4 / 2
// for small batches);
// CTA `rank` owns entries [rank * per, (rank + 1) * per) of every codebook. Each CTA keeps the
// rows' latents and residuals in shared memory, so per codebook a thread scores its entries
// against the residuals (dist = half_norm - entry . residual, Codebook::encode), the CTA finds
// its best (distance, index) per row, every CTA pushes its candidates into every CTA of the
// cluster through distributed shared memory, one cluster barrier publishes them, and every CTA
// reduces them identically (lowest index on ties, like candle's argmin) and subtracts the
// chosen entry from its residuals (codebook.decode). Candidates alternate between two slots,
// so one barrier per codebook suffices. Codebooks are stored transposed, [dim][entry], so the
// threads of a warp read consecutive entries.
constexpr int kRvqDim = 256;   // ResidualQuantizer::DIM
constexpr int kRvqIn = 512;    // the latent width Quantizer::new expects
constexpr int kRvqMaxRows = 8;  // rows per cluster: 8, or 4 / 2 for small batches (more CTAs)
constexpr int kRvqRanks = 8;
constexpr int kRvqThreads = 256;

struct RvqArgs {
  const float* x;  // latents [b][512][frames]
  int64_t x_bs;
  int x_cs, frames, rows;
  const float* proj_t[2];  // input projections transposed [512][256]: rvq_first, rvq_rest
  const float* et;         // codebooks [n_q][256][bins]
  const float* hn;         // half squared norms [n_q][bins]
  int n_q, bins;
  uint32_t* codes;         // [row][n_q], row = b * frames + f
};

__device__ __forceinline__ void dsmem_st_i32(uint32_t addr, int v) {
  asm volatile("st.shared::cluster.s32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ bool rvq_better(float v, int i, float bv, int bi) {
  return v < bv || (v == bv && i < bi);
}

template <int R>
__global__ void __launch_bounds__(kRvqThreads) rvq_kernel(const RvqArgs a) {
  constexpr int NW = kRvqThreads / 32;
  __shared__ float xs[R][kRvqIn];
  __shared__ float res[R][kRvqDim];
  __shared__ float cand_v[2][kRvqRanks][R];
  __shared__ int cand_i[2][kRvqRanks][R];
  __shared__ float warp_v[NW][R];
  __shared__ int warp_i[NW][R];
  __shared__ int chosen[R];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int rank = (int)cluster_rank(), row0 = blockIdx.y * R;
  const int per = (a.bins + kRvqRanks - 1) / kRvqRanks;
  const int e0 = rank * per, e1 = min(a.bins, e0 + per);

  for (int i = tid; i < R * kRvqIn; i += kRvqThreads) {
    const int r = i / kRvqIn, c = i - r * kRvqIn, row = row0 + r;
    float v = 0.f;
    if (row < a.rows) {
      const int b = row / a.frames, f = row - b * a.frames;
      v = a.x[b * a.x_bs + (int64_t)c * a.x_cs + f];
    }
    xs[r][c] = v;
  }
  __syncthreads();

  for (int q = 0; q < a.n_q; q++) {
    if (q <= 1) {
      // ResidualQuantizer::encode: the residual starts as input_proj(x), a 1x1 convolution
      // (rvq_first for codebook 0, rvq_rest for the others): sequential FMA over the 512 inputs.
      const float* pt = a.proj_t[q];
      float acc[R];
#pragma unroll
      for (int r = 0; r < R; r++) acc[r] = 0.f;
      // 16 weights in flight per thread, then their FMAs in order.
      for (int c0 = 0; c0 < kRvqIn; c0 += 16) {
        float wv[16];
#pragma unroll
        for (int u = 0; u < 16; u++) wv[u] = pt[(int64_t)(c0 + u) * kRvqDim + tid];
#pragma unroll
        for (int u = 0; u < 16; u++)
#pragma unroll
          for (int r = 0; r < R; r++) acc[r] = fmaf(wv[u], xs[r][c0 + u], acc[r]);
      }
#pragma unroll
      for (int r = 0; r < R; r++) res[r][tid] = acc[r];
      __syncthreads();
    }
    // This CTA's best entry per row.
    const float* et = a.et + (int64_t)q * kRvqDim * a.bins;
    float bv[R];
    int bi[R];
#pragma unroll
    for (int r = 0; r < R; r++) {
      bv[r] = __int_as_float(0x7f800000);
      bi[r] = INT_MAX;
    }
    for (int j = e0 + tid; j < e1; j += kRvqThreads) {
      float acc[R];
#pragma unroll
      for (int r = 0; r < R; r++) acc[r] = 0.f;
      for (int d0 = 0; d0 < kRvqDim; d0 += 16) {
        float e[16];
#pragma unroll
        for (int u = 0; u < 16; u++) e[u] = et[(int64_t)(d0 + u) * a.bins + j];
#pragma unroll
        for (int u = 0; u < 16; u++)
#pragma unroll
          for (int r = 0; r < R; r++) acc[r] = fmaf(e[u], res[r][d0 + u], acc[r]);
      }
      const float h = a.hn[(int64_t)q * a.bins + j];
#pragma unroll
      for (int r = 0; r < R; r++) {
        const float dist = __fsub_rn(h, acc[r]);  // half_norms.broadcast_sub(dot)
        if (rvq_better(dist, j, bv[r], bi[r])) {
          bv[r] = dist;
          bi[r] = j;
        }
      }
    }
#pragma unroll
    for (int r = 0; r < R; r++) {
#pragma unroll
      for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv[r], o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi[r], o);
        if (rvq_better(ov, oi, bv[r], bi[r])) {
          bv[r] = ov;
          bi[r] = oi;
        }
      }
      if (lane == 0) {
        warp_v[warp][r] = bv[r];
        warp_i[warp][r] = bi[r];
      }
    }
    __syncthreads();
    const int slot = q & 1;
    if (tid < R) {
      float v = warp_v[0][tid];
      int i = warp_i[0][tid];
      for (int w = 1; w < NW; w++)
        if (rvq_better(warp_v[w][tid], warp_i[w][tid], v, i)) {
          v = warp_v[w][tid];
          i = warp_i[w][tid];
        }
      for (int dst = 0; dst < kRvqRanks; dst++) {
        dsmem_st(dsmem_addr(&cand_v[slot][rank][tid], dst), v);
        dsmem_st_i32(dsmem_addr(&cand_i[slot][rank][tid], dst), i);
      }
    }
    cluster_sync();
    if (tid < R) {
      float v = cand_v[slot][0][tid];
      int i = cand_i[slot][0][tid];
      for (int k = 1; k < kRvqRanks; k++)
        if (rvq_better(cand_v[slot][k][tid], cand_i[slot][k][tid], v, i)) {
          v = cand_v[slot][k][tid];
          i = cand_i[slot][k][tid];
        }
      // Every distance NaN: no entry wins; entry 0 keeps the code in range.
      if (i == INT_MAX) i = 0;
      chosen[tid] = i;
      if (rank == 0 && row0 + tid < a.rows) a.codes[(int64_t)(row0 + tid) * a.n_q + q] = (uint32_t)i;
    }
    __syncthreads();
    // residual = residual - codebook.decode(indices)
#pragma unroll
    for (int r = 0; r < R; r++) res[r][tid] = __fsub_rn(res[r][tid], et[(int64_t)tid * a.bins + chosen[r]]);
    __syncthreads();
  }
}

// Frame t of channel-first activations [b][C][T] to the transformer's rows [b][C], and back.
__global__ void frame_gather_kernel(const float* src, int64_t s_bs, int s_cs, int t, float* dst, int C, int nb) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nb * C) return;
  const int b = i / C, c = i - b * C;
  dst[i] = src[b * s_bs + (int64_t)c * s_cs + t];
}
__global__ void frame_scatter_kernel(const float* src, int C, int nb, float* dst, int64_t d_bs, int d_cs, int t) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nb * C) return;
  const int b = i / C, c = i - b * C;
  dst[b * d_bs + (int64_t)c * d_cs + t] = src[i];
}
__global__ void mark_started_kernel(int* started, int nb) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < nb) started[i] = 1;
}

}  // namespace

// ---- host side ------------------------------------------------------------------------------

// One convolution layer of the codec, with its place in the per-stream state.
struct ConvLayer {
  bool tr = false, depthwise = false;
  int cin = 0, cout = 0, k = 1, stride = 1, dil = 1, replicate = 0;
  int ctx = 0;      // StreamingConv1d: input samples carried over
  int overlap = 0;  // StreamingConvTranspose1d: outputs carried over
  DevBuf w, bias;
  int64_t state_off = 0;  // first float of this layer's block in the state ([stream][...])
  int64_t state_per_stream() const { return tr ? (int64_t)cout * overlap : (int64_t)cin * ctx; }
};

// A step of a SEANet / codec pipeline: layer `layer` reads buffer `in` and writes `out` (both
// channel-first; buffer ids below), with ELU on its input and an optional resnet skip.
enum Buf { BUF_IN = 0, BUF_A = 1, BUF_B = 2, BUF_H = 3, BUF_OUT = 4, BUF_T = 5, BUF_P = 6, BUF_L = 7, BUF_S = 8 };
struct ConvStep {
  int layer, in, out, act, skip;  // skip: a buffer id or -1
};

struct Codec {
  int device = 0;
  svl_mimi_config cfg{};
  int frame_size = 0;
  int enc_hop = 1, dec_hop = 1, enc_stride = 1, dec_stride = 1;
  std::vector<ConvLayer> layers;
  std::vector<ConvStep> enc_seanet, dec_seanet;
  int down = -1, up = -1;
  int enc_in_proj = -1, enc_out_proj = -1, dec_in_proj = -1, dec_out_proj = -1;
  int latent_proj = -1, latent_dim = 0;  // Pocket TTS's quantizer.output_proj (tts/mod.rs:218-224)
  Model* enc_tr = nullptr;
  Model* dec_tr = nullptr;
  int64_t state_floats = 0;  // per stream
  cudaStream_t stream = nullptr;
  ~Codec() {
    delete enc_tr;
    delete dec_tr;
    if (stream) cudaStreamDestroy(stream);
  }
};

struct CodecState {
  Codec* c = nullptr;
  int max_batch = 0, max_frames = 0;
  DevBuf conv_state;           // [layer block][stream][...]
  DevBuf enc_started, dec_started;
  DevBuf buf[7];  // blocks A, B, H, T, transposed-convolution products P, projected latents L,
                  // split-convolution partial sums S
  int64_t buf_floats[7] = {0, 0, 0, 0, 0, 0, 0};
  State* enc_ts = nullptr;
  State* dec_ts = nullptr;
  ~CodecState() {
    delete enc_ts;
    delete dec_ts;
  }
};

struct Rvq {
  int device = 0, n_q = 0, bins = 0;
  DevBuf proj_t[2], et, hn;
  cudaStream_t stream = nullptr;
  ~Rvq() {
    if (stream) cudaStreamDestroy(stream);
  }
};

const svl_tensor_view& need_tensor(const svl_tensor_view* t, int n, const std::string& name, int64_t numel) {
  for (int i = 0; i < n; i++)
    if (t[i].name && name == t[i].name) {
      if (t[i].numel != numel)
        throw Error(SVL_ERR_CONFIG, "tensor " + name + ": " + std::to_string(t[i].numel) +
                                        " elements, expected " + std::to_string(numel));
      if (!t[i].data) throw Error(SVL_ERR_CONFIG, "tensor " + name + " has no data");
      return t[i];
    }
  throw Error(SVL_ERR_CONFIG, "missing tensor " + name);
}
bool has_tensor(const svl_tensor_view* t, int n, const std::string& name) {
  for (int i = 0; i < n; i++)
    if (t[i].name && name == t[i].name) return true;
  return false;
}
void upload(DevBuf& dst, const float* src, int64_t numel, cudaStream_t st) {
  dst.alloc(numel * 4);
  check_cuda(cudaMemcpyAsync(dst.p, src, numel * 4, cudaMemcpyHostToDevice, st), "upload");
  check_cuda(cudaStreamSynchronize(st), "upload");
}

struct CodecLoader {
  Codec& c;
  const svl_tensor_view* t;
  int n;
  // StreamingConv1d::new (nn/conv.rs:81-106): "<prefix>.weight" [cout][cin][k], "<prefix>.bias".
  int conv(const std::string& prefix, int cin, int cout, int k, int stride, int dil, int replicate, bool bias) {
    if (cin <= 0 || cout <= 0 || k <= 0 || stride <= 0 || dil <= 0)
      throw Error(SVL_ERR_CONFIG, "invalid convolution " + prefix);
    ConvLayer L;
    L.cin = cin;
    L.cout = cout;
    L.k = k;
    L.stride = stride;
    L.dil = dil;
    L.replicate = replicate;
    L.ctx = std::max(0, (k - 1) * dil + 1 - stride);  // StreamingConv1d::context
    // Stored transposed, [cin * k][cout] (row c * k + j), for the kernel's coalesced staging.
    const float* src = need_tensor(t, n, prefix + ".weight", (int64_t)cout * cin * k).data;
    std::vector<float> tr((size_t)cout * cin * k);
    for (int o = 0; o < cout; o++)
      for (int r = 0; r < cin * k; r++) tr[(size_t)r * cout + o] = src[(size_t)o * cin * k + r];
    upload(L.w, tr.data(), (int64_t)tr.size(), c.stream);
    if (bias) upload(L.bias, need_tensor(t, n, prefix + ".bias", cout).data, cout, c.stream);
    c.layers.push_back(std::move(L));
    return (int)c.layers.size() - 1;
  }
  // StreamingConvTranspose1d::new (nn/conv.rs:227-262): "<prefix>.weight" [cin][cout / groups][k].
  int convtr(const std::string& prefix, int cin, int cout, int k, int stride, int groups, bool bias) {
    if (cin <= 0 || cout <= 0 || k <= 0 || stride <= 0) throw Error(SVL_ERR_CONFIG, "invalid convolution " + prefix);
    if (k < stride || k > kTrMaxHits * stride)
      throw Error(SVL_ERR_UNSUPPORTED, prefix + ": a transposed convolution's kernel must span 1 to 4 strides");
    if (groups != 1 && !(groups == cin && cout == cin))
      throw Error(SVL_ERR_UNSUPPORTED, prefix + ": only ungrouped and depthwise transposed convolutions");
    ConvLayer L;
    L.tr = true;
    L.depthwise = groups != 1;
    L.cin = cin;
    L.cout = cout;
    L.k = k;
    L.stride = stride;
    L.overlap = k - stride;
    const int64_t numel = (int64_t)cin * (cout / groups) * k;
    upload(L.w, need_tensor(t, n, prefix + ".weight", numel).data, numel, c.stream);
    if (bias) upload(L.bias, need_tensor(t, n, prefix + ".bias", cout).data, cout, c.stream);
    c.layers.push_back(std::move(L));
    return (int)c.layers.size() - 1;
  }
  // ResnetBlock::new (nn/seanet.rs:44-66) at "<prefix>.block.{1,3}.conv": ELU, conv (k, dilation),
  // ELU, 1x1 conv, then the skip. Runs in place on buffer `buf` with BUF_H for the hidden rows.
  void resnet(std::vector<ConvStep>& steps, const svl_seanet_config& s, const std::string& prefix, int dim,
              int dilation, int buf) {
    const int hidden = dim / s.compress;
    const int a = conv(prefix + ".block.1.conv", dim, hidden, s.residual_kernel_size, 1, dilation, s.pad_mode, true);
    const int b = conv(prefix + ".block.3.conv", hidden, dim, 1, 1, 1, s.pad_mode, true);
    steps.push_back({a, buf, BUF_H, ACT_ELU, -1});
    steps.push_back({b, BUF_H, buf, ACT_ELU, buf});
  }
};

void validate_seanet(const svl_seanet_config& s) {
  if (s.dimension <= 0 || s.channels <= 0 || s.n_filters <= 0 || s.n_residual_layers < 0 || s.kernel_size <= 0 ||
      s.residual_kernel_size <= 0 || s.last_kernel_size <= 0 || s.dilation_base <= 0 || s.compress <= 0 ||
      s.n_ratios < 0 || s.n_ratios > 8 || (s.pad_mode != 0 && s.pad_mode != 1))
    throw Error(SVL_ERR_CONFIG, "invalid SEANet config");
  for (int i = 0; i < s.n_ratios; i++)
    if (s.ratios[i] <= 0) throw Error(SVL_ERR_CONFIG, "invalid SEANet ratio");
}
int hop_of(const svl_seanet_config& s) {
  int h = 1;
  for (int i = 0; i < s.n_ratios; i++) h *= s.ratios[i];
  return h;
}

// The bare transformer of a ProjectedTransformer (nn/mimi.rs:74-112): LayerNorm 1e-5, plain
// GELU feed-forward (erf or tanh), layer scale, f32 weights and caches.
svl_transformer_config projected_cfg(const svl_projected_transformer_config& p, int exact_gelu) {
  svl_transformer_config t{};
  if (p.num_heads <= 0 || p.d_model <= 0 || p.d_model % p.num_heads)
    throw Error(SVL_ERR_CONFIG, "invalid Mimi transformer config");
  t.d_model = p.d_model;
  t.num_layers = p.num_layers;
  t.num_heads = p.num_heads;
  t.num_kv_heads = p.num_heads;
  t.head_dim = p.d_model / p.num_heads;
  t.ffn_kind = exact_gelu ? SVL_FFN_PLAIN_GELU_ERF : SVL_FFN_PLAIN_GELU_TANH;
  t.ffn_hidden = p.dim_feedforward;
  t.norm_kind = SVL_NORM_LAYER;
  t.norm_eps = 1e-5f;
  t.layer_scale = 1;
  t.context = p.context;
  t.weight_dtype = SVL_DT_F32;
  t.kv_dtype = SVL_DT_F32;
  t.max_period = p.max_period;
  return t;
}

Codec* create_codec(const svl_mimi_config& cfg, const svl_tensor_view* t, int n, int device) {
  if (!(cfg.parts & (SVL_MIMI_ENCODER | SVL_MIMI_DECODER))) throw Error(SVL_ERR_CONFIG, "no codec part requested");
  if (cfg.sample_rate <= 0 || !(cfg.frame_rate > 0) || cfg.inner_dim <= 0 || cfg.outer_dim <= 0)
    throw Error(SVL_ERR_CONFIG, "invalid Mimi config");
  int count = 0;
  check_cuda(cudaGetDeviceCount(&count), "cudaGetDeviceCount");
  if (device < 0 || device >= count) throw Error(SVL_ERR_CUDA, "no such CUDA device");
  check_cuda(cudaSetDevice(device), "cudaSetDevice");
  Codec* c = new Codec();
  try {
    c->device = device;
    c->cfg = cfg;
    check_cuda(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking), "stream");
    CodecLoader ld{*c, t, n};
    // MimiConfig::frame_size / resample_stride (nn/mimi.rs:53-64).
    c->frame_size = (int)std::lround((double)cfg.sample_rate / cfg.frame_rate);
    auto stride_of = [&](const svl_seanet_config& s) {
      const double rate = (double)cfg.sample_rate / hop_of(s);
      return (int)std::lround(rate / cfg.frame_rate);
    };
    if (cfg.parts & SVL_MIMI_ENCODER) {
      const svl_seanet_config& s = cfg.encoder;
      validate_seanet(s);
      c->enc_hop = hop_of(s);
      c->enc_stride = stride_of(s);
      if (c->enc_stride < 1 || c->enc_hop * c->enc_stride != c->frame_size)
        throw Error(SVL_ERR_CONFIG, "the encoder's hop and resampling do not make a codec frame");
      // SeanetEncoder::new (nn/seanet.rs:133-181); Elu layers count in the module indices.
      auto name = [](int i) { return "encoder.model." + std::to_string(i); };
      int li = 0, cur = BUF_A, mult = 1;
      const int c0 = ld.conv(name(li) + ".conv", s.channels, s.n_filters, s.kernel_size, 1, 1, s.pad_mode, true);
      c->enc_seanet.push_back({c0, BUF_IN, BUF_A, ACT_NONE, -1});
      li++;
      for (int r = s.n_ratios - 1; r >= 0; r--) {
        const int dim = mult * s.n_filters;
        int dil = 1;
        for (int j = 0; j < s.n_residual_layers; j++, dil *= s.dilation_base) ld.resnet(c->enc_seanet, s, name(li++), dim, dil, cur);
        li++;  // Elu
        const int nxt = cur == BUF_A ? BUF_B : BUF_A;
        const int dc = ld.conv(name(li++) + ".conv", dim, 2 * dim, 2 * s.ratios[r], s.ratios[r], 1, s.pad_mode, true);
        c->enc_seanet.push_back({dc, cur, nxt, ACT_ELU, -1});
        cur = nxt;
        mult *= 2;
      }
      li++;  // Elu
      const int last = ld.conv(name(li) + ".conv", mult * s.n_filters, s.dimension, s.last_kernel_size, 1, 1, s.pad_mode, true);
      c->enc_seanet.push_back({last, cur, BUF_OUT, ACT_ELU, -1});
      // ProjectedTransformer (nn/mimi.rs:74-122).
      const auto& p = cfg.encoder_transformer;
      if (p.input_dimension != s.dimension) throw Error(SVL_ERR_CONFIG, "encoder transformer input width != SEANet dimension");
      if (p.input_dimension != p.d_model)
        c->enc_in_proj = ld.conv("encoder_transformer.input_proj", p.input_dimension, p.d_model, 1, 1, 1, 0, false);
      if (p.output_dimension != p.d_model)
        c->enc_out_proj = ld.conv("encoder_transformer.output_projs.0", p.d_model, p.output_dimension, 1, 1, 1, 0, false);
      const svl_transformer_config tc = projected_cfg(p, cfg.exact_gelu);
      c->enc_tr = create_model(2, tc, nullptr, nullptr, t, n, device, "encoder_transformer.transformer.");
      // The learnt down-sampling (nn/mimi.rs:143-158): kernel 2 stride, no bias, replicate pad.
      if (c->enc_stride > 1)
        c->down = ld.conv("downsample.conv.conv", p.output_dimension, cfg.inner_dim, 2 * c->enc_stride, c->enc_stride, 1, 1, false);
      else if (p.output_dimension != cfg.inner_dim)
        throw Error(SVL_ERR_CONFIG, "without down-sampling the encoder width must be inner_dim");
    }
    if (cfg.parts & SVL_MIMI_DECODER) {
      const svl_seanet_config& s = cfg.decoder;
      validate_seanet(s);
      c->dec_hop = hop_of(s);
      c->dec_stride = stride_of(s);
      if (c->dec_stride < 1 || c->dec_hop * c->dec_stride != c->frame_size)
        throw Error(SVL_ERR_CONFIG, "the decoder's hop and resampling do not make a codec frame");
      const auto& p = cfg.decoder_transformer;
      // The learnt up-sampling (nn/mimi.rs:232-245): depthwise, kernel 2 stride, no bias.
      if (c->dec_stride > 1)
        c->up = ld.convtr("upsample.convtr.convtr", cfg.outer_dim, s.dimension, 2 * c->dec_stride, c->dec_stride,
                          s.dimension, false);
      else if (cfg.outer_dim != s.dimension)
        throw Error(SVL_ERR_CONFIG, "without up-sampling outer_dim must be the SEANet dimension");
      if (p.input_dimension != s.dimension) throw Error(SVL_ERR_CONFIG, "decoder transformer input width != SEANet dimension");
      if (p.input_dimension != p.d_model)
        c->dec_in_proj = ld.conv("decoder_transformer.input_proj", p.input_dimension, p.d_model, 1, 1, 1, 0, false);
      if (p.output_dimension != p.d_model)
        c->dec_out_proj = ld.conv("decoder_transformer.output_projs.0", p.d_model, p.output_dimension, 1, 1, 1, 0, false);
      if (p.output_dimension != s.dimension) throw Error(SVL_ERR_CONFIG, "decoder transformer output width != SEANet dimension");
      const svl_transformer_config tc = projected_cfg(p, cfg.exact_gelu);
      c->dec_tr = create_model(2, tc, nullptr, nullptr, t, n, device, "decoder_transformer.transformer.");
      // The latent projection of Tts::decode_latent (tts/mod.rs:218-224, :441-447), when the
      // tensors carry it: "quantizer.output_proj.weight" [outer_dim][latent_dim][1].
      for (int i = 0; i < n; i++)
        if (t[i].name && std::string(t[i].name) == "quantizer.output_proj.weight") {
          if (t[i].numel <= 0 || t[i].numel % cfg.outer_dim)
            throw Error(SVL_ERR_CONFIG, "quantizer.output_proj.weight is not [outer_dim][latent][1]");
          c->latent_dim = (int)(t[i].numel / cfg.outer_dim);
          c->latent_proj = ld.conv("quantizer.output_proj", c->latent_dim, cfg.outer_dim, 1, 1, 1, 0, false);
        }
      // SeanetDecoder::new (nn/seanet.rs:197-235).
      auto name = [](int i) { return "decoder.model." + std::to_string(i); };
      int mult = 1 << s.n_ratios, li = 0, cur = BUF_A;
      const int c0 = ld.conv(name(li++) + ".conv", s.dimension, mult * s.n_filters, s.kernel_size, 1, 1, s.pad_mode, true);
      c->dec_seanet.push_back({c0, BUF_IN, BUF_A, ACT_NONE, -1});
      for (int r = 0; r < s.n_ratios; r++) {
        const int dim = mult * s.n_filters;
        li++;  // Elu
        const int nxt = cur == BUF_A ? BUF_B : BUF_A;
        const int up = ld.convtr(name(li++) + ".convtr", dim, dim / 2, 2 * s.ratios[r], s.ratios[r], 1, true);
        c->dec_seanet.push_back({up, cur, nxt, ACT_ELU, -1});
        cur = nxt;
        int dil = 1;
        for (int j = 0; j < s.n_residual_layers; j++, dil *= s.dilation_base) ld.resnet(c->dec_seanet, s, name(li++), dim / 2, dil, cur);
        mult /= 2;
      }
      li++;  // Elu
      const int last = ld.conv(name(li) + ".conv", s.n_filters, s.channels, s.last_kernel_size, 1, 1, s.pad_mode, true);
      c->dec_seanet.push_back({last, cur, BUF_OUT, ACT_ELU, -1});
    }
    for (ConvLayer& L : c->layers) {
      L.state_off = c->state_floats;
      c->state_floats += L.state_per_stream();
    }
  } catch (...) {
    delete c;
    throw;
  }
  return c;
}

// A channel-first activation block: C rows of `rowlen` floats per stream, t of them valid.
struct View {
  float* p = nullptr;
  int C = 0, t = 0, rowlen = 0;
  int64_t bs() const { return (int64_t)C * rowlen; }
};

// Input channels per chunk of a convolution's reduction: the (channel, tap) terms are summed
// in chunks of at most kConvChunkTerms (one FMA chain each), the chunks' sums in order. The
// blocking depends on the layer's shape only, so results do not depend on the batch or the
// launch; the CPU oracle sums the same way.
constexpr int kConvChunkTerms = 1024;
int conv_chunk_channels(int k) { return std::max(1, kConvChunkTerms / k); }
int conv_chunks(int cin, int k) { return (cin + conv_chunk_channels(k) - 1) / conv_chunk_channels(k); }

// scratch: nchunks * nb * cout * len floats when the layer has more than one chunk.
void launch_conv(const ConvArgs& a, int nb, cudaStream_t st, float* scratch = nullptr) {
  // Input channels per stage: both operands' rows, 2 x 64 floats per (channel, tap).
  const int per_channel = 2 * kConvTile * a.k * 4;
  const int cpc = conv_chunk_channels(a.k);
  const int cc = std::max(1, std::min({a.cin, cpc, kConvSmem / per_channel}));
  const size_t smem = (size_t)cc * per_channel;
  if (smem > (size_t)kConvSmem) throw Error(SVL_ERR_UNSUPPORTED, "convolution kernel too wide for one tile");
  const int64_t ncol = (int64_t)nb * a.len;
  const int nchunks = conv_chunks(a.cin, a.k);
  const int tiles = (int)(((ncol + kConvTile - 1) / kConvTile) * ((a.cout + kConvTile - 1) / kConvTile));
  // Few tiles (short chunks of a batch): one CTA per (tile, chunk), then the combine.
  const bool split = nchunks > 1 && scratch && tiles < 148;
  const dim3 grid((unsigned)((ncol + kConvTile - 1) / kConvTile), (a.cout + kConvTile - 1) / kConvTile,
                  split ? nchunks : 1);
  conv1d_kernel<<<grid, kConvThreads, smem, st>>>(a, cc, nb, cpc, split ? scratch : nullptr);
  if (split) {
    const int64_t n = (int64_t)nb * a.cout * a.len;
    conv_combine_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(a, scratch, nchunks, nb);
  }
  if (a.ctx > 0) conv_state_kernel<<<(nb * a.cin + 255) / 256, 256, 0, st>>>(a, nb);
}

// prod: for an ungrouped layer, the products [b][cout * k][t] (computed by the caller).
void launch_convtr(const ConvTrArgs& a, const float* prod, int nb, cudaStream_t st) {
  const int64_t n = (int64_t)nb * a.cout * (a.t * a.stride + a.overlap);
  convtr_add_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(a, prod, nb);
  if (a.overlap > 0) convtr_state_kernel<<<(nb * a.cout * a.overlap + 255) / 256, 256, 0, st>>>(a, nb);
}

// Runs (or, with dry set, only sizes) one encode / decode call. Buffers A, B, H and the
// transformer block T come from the state; `need` records the floats each one must hold.
struct Exec {
  CodecState& S;
  int nb;
  bool dry;
  int64_t need[7] = {0, 0, 0, 0, 0, 0, 0};
  cudaStream_t st;
  const int* started;

  float* buf(int id, int64_t floats) {
    const int i = id == BUF_A ? 0 : id == BUF_B ? 1 : id == BUF_H ? 2 : id == BUF_P ? 4 : id == BUF_L ? 5 : id == BUF_S ? 6 : 3;  // BUF_T: 3
    need[i] = std::max(need[i], floats);
    if (dry) return nullptr;
    if (floats > S.buf_floats[i]) throw Error(SVL_ERR_INVALID_INPUT, "codec call larger than the state's max_frames");
    return S.buf[i].as<float>();
  }
  float* layer_state(const ConvLayer& L) {
    return S.conv_state.as<float>() + L.state_off * S.max_batch;
  }

  View conv(const ConvLayer& L, const View& in, float* outp, int out_id, int act, const View* skip) {
    if (in.C != L.cin) throw Error(SVL_ERR_CONFIG, "codec layer widths do not chain");
    View out;
    if (L.tr) {
      out.C = L.cout;
      out.t = in.t * L.stride;
      out.rowlen = out.t + L.overlap;
    } else {
      if (in.t % L.stride) throw Error(SVL_ERR_INVALID_INPUT, "a convolution's input is not a multiple of its stride");
      out.C = L.cout;
      out.t = in.t / L.stride;
      out.rowlen = out.t;
    }
    if (skip) {
      // ResnetBlock: xs + ys, written in place over xs with its layout.
      if (skip->C != out.C || skip->t != out.t) throw Error(SVL_ERR_CONFIG, "resnet skip does not match its block");
      out.rowlen = skip->rowlen;
      out.p = skip->p;
    } else {
      out.p = outp ? outp : buf(out_id, out.bs() * nb);
    }
    // A transposed convolution's taps: products [b][cout * k][t] in block P.
    float* prod = L.tr && !L.depthwise ? buf(BUF_P, (int64_t)L.cout * L.k * in.t * nb) : nullptr;
    // A convolution of several reduction chunks: room for the chunks' sums (block S).
    const int nchunks = L.tr ? 1 : conv_chunks(L.cin, L.k);
    float* scratch = nchunks > 1 ? buf(BUF_S, (int64_t)nchunks * nb * L.cout * out.t) : nullptr;
    if (dry) return out;
    if (L.tr) {
      if (!L.depthwise) {
        // The taps' products as a 1x1 convolution with cout * k output channels: the layer's
        // weight [cin][cout][k] is that convolution's transposed weight [cin][cout * k].
        ConvArgs p{};
        p.x = in.p;
        p.x_bs = in.bs();
        p.x_cs = in.rowlen;
        p.x_ts = 1;
        p.t = in.t;
        p.started = started;
        p.cin = L.cin;
        p.cout = L.cout * L.k;
        p.k = p.stride = p.dil = 1;
        p.act = act;
        p.w = L.w.as<float>();
        p.out = prod;
        p.o_bs = (int64_t)p.cout * in.t;
        p.o_cs = in.t;
        p.len = in.t;
        launch_conv(p, nb, st);
      }
      ConvTrArgs a{};
      a.x = in.p;
      a.x_bs = in.bs();
      a.x_cs = in.rowlen;
      a.t = in.t;
      a.act = act;
      a.partial = layer_state(L);
      a.b0 = 0;
      a.overlap = L.overlap;
      a.cin = L.cin;
      a.cout = L.cout;
      a.k = L.k;
      a.stride = L.stride;
      a.depthwise = L.depthwise;
      a.w = L.w.as<float>();
      a.bias = L.bias.as<float>();
      a.out = out.p;
      a.o_bs = out.bs();
      a.o_cs = out.rowlen;
      launch_convtr(a, prod, nb, st);
    } else {
      ConvArgs a{};
      a.x = in.p;
      a.x_bs = in.bs();
      a.x_cs = in.rowlen;
      a.x_ts = 1;
      a.t = in.t;
      a.prev = layer_state(L);
      a.started = started;
      a.b0 = 0;
      a.ctx = L.ctx;
      a.cin = L.cin;
      a.cout = L.cout;
      a.k = L.k;
      a.stride = L.stride;
      a.dil = L.dil;
      a.act = act;
      a.replicate = L.replicate;
      a.w = L.w.as<float>();
      a.bias = L.bias.as<float>();
      a.skip = skip ? skip->p : nullptr;
      a.out = out.p;
      a.o_bs = out.bs();
      a.o_cs = out.rowlen;
      a.len = out.t;
      launch_conv(a, nb, st, scratch);
    }
    check_cuda(cudaGetLastError(), "codec convolution launch");
    return out;
  }

  // A SEANet pipeline from `in`; the last step writes into `outp`, or into block T when null.
  View seanet(const std::vector<ConvStep>& steps, const View& in, float* outp) {
    View v[6];
    v[BUF_IN] = in;
    View o;
    for (const ConvStep& s : steps) {
      const ConvLayer& L = S.c->layers[s.layer];
      const View* skip = s.skip >= 0 ? &v[s.skip] : nullptr;
      const bool final = s.out == BUF_OUT;
      o = conv(L, v[s.in], final ? outp : nullptr, final ? BUF_T : s.out, s.act, skip);
      v[s.out] = o;
    }
    return o;
  }
};

// The transformer of a ProjectedTransformer over the t frames of `x` (in place), one step per
// frame: causal attention makes a block of t queries equal to t single steps
// (nn/transformer.rs:598-628).
void run_transformer(Exec& E, Model& m, State& ts, const View& x) {
  if (x.C != m.cfg.d_model) throw Error(SVL_ERR_CONFIG, "Mimi transformer width mismatch");
  if (E.dry) return;
  const int nb = E.nb, d = x.C;
  float* rows = ts.x.as<float>();
  const int blocks = (nb * d + 255) / 256;
  for (int i = 0; i < x.t; i++) {
    frame_gather_kernel<<<blocks, 256, 0, E.st>>>(x.p, x.bs(), x.rowlen, i, rows, d, nb);
    enqueue_layers(m, ts, 0, nb, E.st);
    launch_advance_positions(ts.pos.as<int>(), nb, E.st);
    frame_scatter_kernel<<<blocks, 256, 0, E.st>>>(rows, d, nb, x.p, x.bs(), x.rowlen, i);
  }
  for (int b = 0; b < nb; b++) ts.hpos[b] += x.t;
  check_cuda(cudaGetLastError(), "Mimi transformer launch");
}

// MimiEncoder::encode_step (nn/mimi.rs:184-191).
void encode(Exec& E, int frames, const float* pcm, float* latent) {
  Codec& c = *E.S.c;
  View in;
  in.p = const_cast<float*>(pcm);
  in.C = c.cfg.encoder.channels;
  in.t = in.rowlen = frames * c.frame_size;
  View x = E.seanet(c.enc_seanet, in, nullptr);
  if (c.enc_in_proj >= 0) x = E.conv(c.layers[c.enc_in_proj], x, nullptr, BUF_A, ACT_NONE, nullptr);
  run_transformer(E, *c.enc_tr, *E.S.enc_ts, x);
  if (c.enc_out_proj >= 0) x = E.conv(c.layers[c.enc_out_proj], x, nullptr, BUF_B, ACT_NONE, nullptr);
  if (c.down >= 0) {
    E.conv(c.layers[c.down], x, latent ? latent : nullptr, BUF_B, ACT_NONE, nullptr);
  } else if (!E.dry) {
    check_cuda(cudaMemcpy2DAsync(latent, (size_t)x.t * 4, x.p, (size_t)x.rowlen * 4, (size_t)x.t * 4,
                                 (size_t)x.C * E.nb, cudaMemcpyDeviceToDevice, E.st),
               "latent copy");
  }
}

// MimiDecoder::decode_step (nn/mimi.rs:262-271).
void decode(Exec& E, int frames, const float* latent, float* pcm) {
  Codec& c = *E.S.c;
  View in;
  in.p = const_cast<float*>(latent);
  in.C = c.cfg.outer_dim;
  in.t = in.rowlen = frames;
  View x;
  if (c.up >= 0) {
    x = E.conv(c.layers[c.up], in, nullptr, BUF_T, ACT_NONE, nullptr);
  } else {
    x = in;
    x.p = E.buf(BUF_T, in.bs() * E.nb);
    if (!E.dry)
      check_cuda(cudaMemcpyAsync(x.p, latent, in.bs() * E.nb * 4, cudaMemcpyDeviceToDevice, E.st), "latent copy");
  }
  if (c.dec_in_proj >= 0) x = E.conv(c.layers[c.dec_in_proj], x, nullptr, BUF_A, ACT_NONE, nullptr);
  run_transformer(E, *c.dec_tr, *E.S.dec_ts, x);
  if (c.dec_out_proj >= 0) x = E.conv(c.layers[c.dec_out_proj], x, nullptr, BUF_B, ACT_NONE, nullptr);
  E.seanet(c.dec_seanet, x, pcm);
}

// Tts::decode_latent (tts/mod.rs:441-447): latents [b][frames][latent_dim] (the flow LM's
// layout), times emb_std plus emb_mean (null: left as they are), through the latent projection
// into [b][outer_dim][frames], then MimiDecoder::decode_step.
void decode_latent(Exec& E, int frames, const float* latent, const float* std_, const float* mean,
                   float* pcm) {
  Codec& c = *E.S.c;
  const ConvLayer& L = c.layers[c.latent_proj];
  float* proj = E.buf(BUF_L, (int64_t)L.cout * frames * E.nb);
  if (!E.dry) {
    ConvArgs a{};
    a.x = latent;
    a.x_bs = (int64_t)frames * L.cin;
    a.x_cs = 1;
    a.x_ts = L.cin;
    a.t = frames;
    a.act = std_ ? ACT_AFFINE : ACT_NONE;
    a.in_scale = std_;
    a.in_shift = mean;
    a.started = E.started;
    a.cin = L.cin;
    a.cout = L.cout;
    a.k = a.stride = a.dil = 1;
    a.w = L.w.as<float>();
    a.out = proj;
    a.o_bs = (int64_t)L.cout * frames;
    a.o_cs = frames;
    a.len = frames;
    launch_conv(a, E.nb, E.st);
    check_cuda(cudaGetLastError(), "latent projection launch");
  }
  decode(E, frames, proj, pcm);
}

CodecState* create_codec_state(Codec* c, int max_batch, int max_frames) {
  if (max_batch <= 0 || max_frames <= 0) throw Error(SVL_ERR_INVALID_INPUT, "max_batch and max_frames must be positive");
  check_cuda(cudaSetDevice(c->device), "cudaSetDevice");
  CodecState* S = new CodecState();
  try {
    S->c = c;
    S->max_batch = max_batch;
    S->max_frames = max_frames;
    // Size the work blocks by a dry run of the largest call of each half.
    int64_t need[7] = {0, 0, 0, 0, 0, 0, 0};
    for (int half = 0; half < 2; half++) {
      if (half == 0 && !c->enc_tr) continue;
      if (half == 1 && !c->dec_tr) continue;
      Exec E{*S, max_batch, true, {0, 0, 0, 0, 0, 0, 0}, c->stream, nullptr};
      if (half == 0) encode(E, max_frames, nullptr, nullptr);
      else if (c->latent_proj >= 0) decode_latent(E, max_frames, nullptr, nullptr, nullptr, nullptr);
      else decode(E, max_frames, nullptr, nullptr);
      for (int i = 0; i < 7; i++) need[i] = std::max(need[i], E.need[i]);
    }
    for (int i = 0; i < 7; i++) {
      S->buf_floats[i] = need[i];
      if (need[i] > 0) S->buf[i].alloc(need[i] * 4);
    }
    if (c->state_floats > 0) {
      S->conv_state.alloc(c->state_floats * max_batch * 4);
      check_cuda(cudaMemsetAsync(S->conv_state.p, 0, c->state_floats * max_batch * 4, c->stream), "memset");
    }
    S->enc_started.alloc(max_batch * 4);
    S->dec_started.alloc(max_batch * 4);
    check_cuda(cudaMemsetAsync(S->enc_started.p, 0, max_batch * 4, c->stream), "memset");
    check_cuda(cudaMemsetAsync(S->dec_started.p, 0, max_batch * 4, c->stream), "memset");
    if (c->enc_tr) S->enc_ts = create_state(c->enc_tr, max_batch, 0);
    if (c->dec_tr) S->dec_ts = create_state(c->dec_tr, max_batch, 0);
    check_cuda(cudaStreamSynchronize(c->stream), "codec state init");
  } catch (...) {
    delete S;
    throw;
  }
  return S;
}

void reset_codec_state(CodecState& S, int stream) {
  Codec& c = *S.c;
  check_cuda(cudaSetDevice(c.device), "cudaSetDevice");
  const int b0 = stream < 0 ? 0 : stream, nb = stream < 0 ? S.max_batch : 1;
  for (const ConvLayer& L : c.layers) {
    const int64_t per = L.state_per_stream();
    if (per == 0) continue;
    float* base = S.conv_state.as<float>() + L.state_off * S.max_batch + (int64_t)b0 * per;
    check_cuda(cudaMemsetAsync(base, 0, per * nb * 4, c.stream), "memset");
  }
  check_cuda(cudaMemsetAsync(S.enc_started.as<int>() + b0, 0, nb * 4, c.stream), "memset");
  check_cuda(cudaMemsetAsync(S.dec_started.as<int>() + b0, 0, nb * 4, c.stream), "memset");
  check_cuda(cudaStreamSynchronize(c.stream), "reset");
  if (S.enc_ts) state_reset(*S.enc_ts, stream);
  if (S.dec_ts) state_reset(*S.dec_ts, stream);
}

// Quantizer::new (stt/model.rs:92-98) and Codebook::new (:146-157).
Rvq* create_rvq(int n_q, int bins, const svl_tensor_view* t, int n, int device) {
  if (n_q < 1 || bins < 1) throw Error(SVL_ERR_CONFIG, "n_q and bins must be positive");
  int count = 0;
  check_cuda(cudaGetDeviceCount(&count), "cudaGetDeviceCount");
  if (device < 0 || device >= count) throw Error(SVL_ERR_CUDA, "no such CUDA device");
  check_cuda(cudaSetDevice(device), "cudaSetDevice");
  Rvq* q = new Rvq();
  try {
    q->device = device;
    q->n_q = n_q;
    q->bins = bins;
    check_cuda(cudaStreamCreateWithFlags(&q->stream, cudaStreamNonBlocking), "stream");
    const char* parts[2] = {"quantizer.rvq_first", "quantizer.rvq_rest"};
    for (int p = 0; p < 2; p++) {
      if (p == 1 && n_q == 1) continue;
      const svl_tensor_view& w = need_tensor(t, n, std::string(parts[p]) + ".input_proj.weight", (int64_t)kRvqDim * kRvqIn);
      std::vector<float> tr((size_t)kRvqIn * kRvqDim);
      for (int d = 0; d < kRvqDim; d++)
        for (int c = 0; c < kRvqIn; c++) tr[(size_t)c * kRvqDim + d] = w.data[(size_t)d * kRvqIn + c];
      upload(q->proj_t[p], tr.data(), (int64_t)tr.size(), q->stream);
    }
    std::vector<float> et((size_t)n_q * kRvqDim * bins), hn((size_t)n_q * bins), emb((size_t)kRvqDim);
    for (int k = 0; k < n_q; k++) {
      const std::string pre = k == 0 ? std::string(parts[0]) + ".vq.layers.0._codebook."
                                     : std::string(parts[1]) + ".vq.layers." + std::to_string(k - 1) + "._codebook.";
      const svl_tensor_view& sum = need_tensor(t, n, pre + "embedding_sum", (int64_t)bins * kRvqDim);
      const svl_tensor_view& use = need_tensor(t, n, pre + "cluster_usage", bins);
      for (int j = 0; j < bins; j++) {
        const float u = std::max(use.data[j], 1e-5f);  // cluster_usage.maximum(1e-5)
        float h = 0.f;
        for (int d = 0; d < kRvqDim; d++) {
          const float e = sum.data[(size_t)j * kRvqDim + d] / u;  // embedding_sum / usage
          et[((size_t)k * kRvqDim + d) * bins + j] = e;
          h = h + e * e;  // embedding.sqr().sum(D::Minus1), in order
        }
        hn[(size_t)k * bins + j] = h * 0.5f;  // / 2
      }
    }
    upload(q->et, et.data(), (int64_t)et.size(), q->stream);
    upload(q->hn, hn.data(), (int64_t)hn.size(), q->stream);
  } catch (...) {
    delete q;
    throw;
  }
  return q;
}

void rvq_encode(Rvq& q, int nb, int frames, const float* latent, uint32_t* codes, cudaStream_t st) {
  RvqArgs a{};
  a.x = latent;
  a.x_bs = (int64_t)kRvqIn * frames;
  a.x_cs = frames;
  a.frames = frames;
  a.rows = nb * frames;
  a.proj_t[0] = q.proj_t[0].as<float>();
  a.proj_t[1] = q.n_q > 1 ? q.proj_t[1].as<float>() : q.proj_t[0].as<float>();
  a.et = q.et.as<float>();
  a.hn = q.hn.as<float>();
  a.n_q = q.n_q;
  a.bins = q.bins;
  a.codes = codes;
  // Rows per cluster: enough clusters to cover the SMs (each CTA scores its entries for its
  // cluster's rows; fewer rows per cluster means more CTAs reading the same codebook slices).
  const int R = a.rows <= 32 ? 2 : a.rows <= 96 ? 4 : kRvqMaxRows;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kRvqRanks, (a.rows + R - 1) / R, 1);
  cfg.blockDim = dim3(kRvqThreads);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kRvqRanks;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (R == 2)
    check_cuda(cudaLaunchKernelEx(&cfg, rvq_kernel<2>, a), "RVQ launch");
  else if (R == 4)
    check_cuda(cudaLaunchKernelEx(&cfg, rvq_kernel<4>, a), "RVQ launch");
  else
    check_cuda(cudaLaunchKernelEx(&cfg, rvq_kernel<kRvqMaxRows>, a), "RVQ launch");
}

template <class F>
svl_status codec_guarded(F&& f) {
  try {
    f();
    return SVL_OK;
  } catch (const Error& e) {
    set_last_error(e.what());
    return e.code;
  } catch (const std::bad_alloc&) {
    set_last_error("host allocation failed");
    return SVL_ERR_OOM;
  } catch (const std::exception& e) {
    set_last_error(e.what());
    return SVL_ERR_CUDA;
  }
}

}  // namespace svl

struct svl_mimi {
  svl::Codec* c;
};
struct svl_mimi_state {
  svl::CodecState* s;
  svl_mimi* mimi;
};
struct svl_rvq {
  svl::Rvq* q;
};

using svl::Error;

extern "C" {

SVL_API svl_status svl_mimi_create(const svl_mimi_config* cfg, const svl_tensor_view* tensors, int32_t n_tensors,
                                   int32_t device, svl_mimi** out) {
  return svl::codec_guarded([&] {
    if (!cfg || !out || (!tensors && n_tensors)) throw Error(SVL_ERR_INVALID_INPUT, "null argument");
    *out = nullptr;
    svl::Codec* c = svl::create_codec(*cfg, tensors, n_tensors, device);
    *out = new svl_mimi{c};
  });
}

SVL_API void svl_mimi_destroy(svl_mimi* mimi) {
  if (!mimi) return;
  cudaSetDevice(mimi->c->device);
  cudaDeviceSynchronize();
  delete mimi->c;
  delete mimi;
}

SVL_API int32_t svl_mimi_frame_size(const svl_mimi* mimi) { return mimi ? mimi->c->frame_size : 0; }

SVL_API svl_status svl_mimi_state_create(svl_mimi* mimi, int32_t max_batch, int32_t max_frames,
                                         svl_mimi_state** out) {
  return svl::codec_guarded([&] {
    if (!mimi || !out) throw Error(SVL_ERR_INVALID_INPUT, "null argument");
    *out = nullptr;
    svl::CodecState* s = svl::create_codec_state(mimi->c, max_batch, max_frames);
    *out = new svl_mimi_state{s, mimi};
  });
}

SVL_API void svl_mimi_state_destroy(svl_mimi_state* state) {
  if (!state) return;
  cudaSetDevice(state->s->c->device);
  cudaDeviceSynchronize();
  delete state->s;
  delete state;
}

SVL_API svl_status svl_mimi_state_reset(svl_mimi_state* state, int32_t stream) {
  return svl::codec_guarded([&] {
    if (!state) throw Error(SVL_ERR_INVALID_INPUT, "null argument");
    if (stream >= state->s->max_batch) throw Error(SVL_ERR_INVALID_INPUT, "stream index out of range");
    cudaSetDevice(state->s->c->device);
    svl::check_cuda(cudaDeviceSynchronize(), "reset");
    svl::reset_codec_state(*state->s, stream);
  });
}

SVL_API svl_status svl_mimi_encode_step_device(svl_mimi* mimi, svl_mimi_state* state, int32_t batch, int32_t frames,
                                               const float* d_pcm, float* d_latent, void* cuda_stream) {
  return svl::codec_guarded([&] {
    if (!mimi || !state || !d_pcm || !d_latent) throw Error(SVL_ERR_INVALID_INPUT, "null argument");
    svl::CodecState& S = *state->s;
    if (S.c != mimi->c) throw Error(SVL_ERR_INVALID_INPUT, "state of another codec");
    if (!mimi->c->enc_tr) throw Error(SVL_ERR_INVALID_INPUT, "the codec was created without its encoder");
    if (batch < 1 || batch > S.max_batch) throw Error(SVL_ERR_INVALID_INPUT, "batch out of range");
    if (frames < 1 || frames > S.max_frames) throw Error(SVL_ERR_INVALID_INPUT, "frames must be 1..max_frames");
    svl::check_cuda(cudaSetDevice(mimi->c->device), "cudaSetDevice");
    cudaStream_t st = cuda_stream ? static_cast<cudaStream_t>(cuda_stream) : mimi->c->stream;
    svl::Exec E{S, batch, false, {0, 0, 0, 0, 0, 0, 0}, st, S.enc_started.as<int>()};
    svl::encode(E, frames, d_pcm, d_latent);
    svl::mark_started_kernel<<<(batch + 255) / 256, 256, 0, st>>>(S.enc_started.as<int>(), batch);
    svl::check_cuda(cudaGetLastError(), "encode");
  });
}

SVL_API svl_status svl_mimi_decode_step_device(svl_mimi* mimi, svl_mimi_state* state, int32_t batch, int32_t frames,
                                               const float* d_latent, float* d_pcm, void* cuda_stream) {
  return svl::codec_guarded([&] {
    if (!mimi || !state || !d_pcm || !d_latent) throw Error(SVL_ERR_INVALID_INPUT, "null argument");
    svl::CodecState& S = *state->s;
    if (S.c != mimi->c) throw Error(SVL_ERR_INVALID_INPUT, "state of another codec");
    if (!mimi->c->dec_tr) throw Error(SVL_ERR_INVALID_INPUT, "the codec was created without its decoder");
    if (batch < 1 || batch > S.max_batch) throw Error(SVL_ERR_INVALID_INPUT, "batch out of range");
    if (frames < 1 || frames > S.max_frames) throw Error(SVL_ERR_INVALID_INPUT, "frames must be 1..max_frames");
    svl::check_cuda(cudaSetDevice(mimi->c->device), "cudaSetDevice");
    cudaStream_t st = cuda_stream ? static_cast<cudaStream_t>(cuda_stream) : mimi->c->stream;
    svl::Exec E{S, batch, false, {0, 0, 0, 0, 0, 0, 0}, st, S.dec_started.as<int>()};
    svl::decode(E, frames, d_latent, d_pcm);
    svl::mark_started_kernel<<<(batch + 255) / 256, 256, 0, st>>>(S.dec_started.as<int>(), batch);
    svl::check_cuda(cudaGetLastError(), "decode");
  });
}

SVL_API svl_status svl_mimi_decode_latent_device(svl_mimi* mimi, svl_mimi_state* state, int32_t batch,
                                                 int32_t frames, const float* d_latent, const float* d_emb_std,
                                                 const float* d_emb_mean, float* d_pcm, void* cuda_stream) {
  return svl::codec_guarded([&] {
    if (!mimi || !state || !d_pcm || !d_latent) throw Error(SVL_ERR_INVALID_INPUT, "null argument");
    if (!d_emb_std != !d_emb_mean) throw Error(SVL_ERR_INVALID_INPUT, "emb_std and emb_mean go together");
    svl::CodecState& S = *state->s;
    if (S.c != mimi->c) throw Error(SVL_ERR_INVALID_INPUT, "state of another codec");
    if (!mimi->c->dec_tr) throw Error(SVL_ERR_INVALID_INPUT, "the codec was created without its decoder");
    if (mimi->c->latent_proj < 0)
      throw Error(SVL_ERR_INVALID_INPUT, "the codec was created without quantizer.output_proj.weight");
    if (batch < 1 || batch > S.max_batch) throw Error(SVL_ERR_INVALID_INPUT, "batch out of range");
    if (frames < 1 || frames > S.max_frames) throw Error(SVL_ERR_INVALID_INPUT, "frames must be 1..max_frames");
    svl::check_cuda(cudaSetDevice(mimi->c->device), "cudaSetDevice");
    cudaStream_t st = cuda_stream ? static_cast<cudaStream_t>(cuda_stream) : mimi->c->stream;
    svl::Exec E{S, batch, false, {0, 0, 0, 0, 0, 0, 0}, st, S.dec_started.as<int>()};
    svl::decode_latent(E, frames, d_latent, d_emb_std, d_emb_mean, d_pcm);
    svl::mark_started_kernel<<<(batch + 255) / 256, 256, 0, st>>>(S.dec_started.as<int>(), batch);
    svl::check_cuda(cudaGetLastError(), "decode");
  });
}

SVL_API int32_t svl_mimi_latent_dim(const svl_mimi* mimi) { return mimi ? mimi->c->latent_dim : 0; }

SVL_API svl_status svl_rvq_create(int32_t n_q, int32_t bins, const svl_tensor_view* tensors, int32_t n_tensors,
                                  int32_t device, svl_rvq** out) {
  return svl::codec_guarded([&] {
    if (!out || (!tensors && n_tensors)) throw Error(SVL_ERR_INVALID_INPUT, "null argument");
    *out = nullptr;
    svl::Rvq* q = svl::create_rvq(n_q, bins, tensors, n_tensors, device);
    *out = new svl_rvq{q};
  });
}

SVL_API void svl_rvq_destroy(svl_rvq* rvq) {
  if (!rvq) return;
  cudaSetDevice(rvq->q->device);
  cudaDeviceSynchronize();
  delete rvq->q;
  delete rvq;
}

SVL_API svl_status svl_rvq_encode_device(svl_rvq* rvq, int32_t batch, int32_t frames, const float* d_latent,
                                         uint32_t* d_codes, void* cuda_stream) {
  return svl::codec_guarded([&] {
    if (!rvq || !d_latent || !d_codes) throw Error(SVL_ERR_INVALID_INPUT, "null argument");
    if (batch < 1 || frames < 1) throw Error(SVL_ERR_INVALID_INPUT, "batch and frames must be positive");
    if ((int64_t)batch * frames > (int64_t)INT_MAX / 2) throw Error(SVL_ERR_INVALID_INPUT, "too many rows");
    svl::check_cuda(cudaSetDevice(rvq->q->device), "cudaSetDevice");
    cudaStream_t st = cuda_stream ? static_cast<cudaStream_t>(cuda_stream) : rvq->q->stream;
    svl::rvq_encode(*rvq->q, batch, frames, d_latent, d_codes, st);
  });
}

}  // extern "C"
