// gemv_common.cuh — device code of the matrix-vector kernels (gemv.cu): the argmax order,
// the fused epilogue, the norm statistics and the input records (norm + the weight format's
// activation conversion) in shared memory.
#pragma once

#include <climits>

#include "common.cuh"
#include "kernels.cuh"

namespace svl {

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
  if (v != v) return false;
  if (bi == INT_MAX) return true;
  return v > bv || (v == bv && i < bi);
}

// The fused epilogue for row `row` of stream b (value v; v_lo / v_hi are the values of the
// aligned row pair (2i, 2i+1) that holds `row`, for RoPE and SwiGLU).
__device__ __forceinline__ void epilogue(const GemvParams& p, int b, int row, float v, float v_lo,
                                         float v_hi) {
  switch (p.epi) {
    case EPI_STORE:
    case EPI_LOGITS:
      if (p.out) p.out[b * p.out_stride + row] = v + (p.bias ? p.bias[row] : 0.f);
      break;
    case EPI_RESIDUAL: {
      float u = p.bias ? v + p.bias[row] : v;
      if (p.ls) u = u * p.ls[row];
      float* o = p.out + b * p.out_stride + row;
      *o = *o + u;
      break;
    }
    case EPI_GELU_TANH:
      p.out[b * p.out_stride + row] = gelu_tanh_ref(p.bias ? v + p.bias[row] : v);
      break;
    case EPI_GELU_ERF:
      p.out[b * p.out_stride + row] = gelu_erf_ref(p.bias ? v + p.bias[row] : v);
      break;
    case EPI_SILU:
      p.out[b * p.out_stride + row] = silu_ref(p.bias ? v + p.bias[row] : v);
      break;
    case EPI_SWIGLU:
      // Packed row 2i is gate row i, 2i+1 value row i (FeedForwardLayer::Gated,
      // nn/transformer.rs:457-461).
      if (!(row & 1)) p.out[b * p.out_stride + row / 2] = silu_ref(v_lo) * v_hi;
      break;
    case EPI_QKV_ROPE: {
      const int hd = p.head_dim;
      const int pos = p.pos[b];
      const int slot = p.windowed ? pos % p.ring_cap : pos;
      if (row < p.q_dim + p.kv_dim) {
        // rope_i (candle; nn/transformer.rs:339-340): pairs (2i, 2i+1) rotate by pos * f_i,
        // out[2i] = a cos - b sin, out[2i+1] = a sin + b cos, each product rounded (the
        // library is built without implicit FMA contraction).
        const int dim = row % hd, i = dim >> 1;
        float sn, cs;
        if (p.rope_by_pos) {
          const float2 t = p.rope_by_pos[(int64_t)min(pos, p.rope_positions - 1) * (hd >> 1) + i];
          cs = t.x;
          sn = t.y;
        } else {
          sincosf((float)pos * p.inv_freq[i], &sn, &cs);
        }
        const float val = (dim & 1) ? v_lo * sn + v_hi * cs : v_lo * cs - v_hi * sn;
        if (row < p.q_dim) {
          p.out[b * p.out_stride + row] = val;
        } else {
          const int kh = (row - p.q_dim) / hd;
          const int64_t off = b * p.ring_stream_stride + ((int64_t)kh * p.ring_cap + slot) * hd + dim;
          if (p.kv_bf16)
            reinterpret_cast<__nv_bfloat16*>(p.k_ring)[off] = __float2bfloat16_rn(val);
          else
            reinterpret_cast<float*>(p.k_ring)[off] = val;
        }
      } else {
        const int vr = row - p.q_dim - p.kv_dim;
        const int kh = vr / hd, dim = vr % hd;
        const int64_t off = b * p.ring_stream_stride + ((int64_t)kh * p.ring_cap + slot) * hd + dim;
        if (p.kv_bf16)
          reinterpret_cast<__nv_bfloat16*>(p.v_ring)[off] = __float2bfloat16_rn(v);
        else
          reinterpret_cast<float*>(p.v_ring)[off] = v;
      }
      break;
    }
  }
}

// ---- Norm statistics -------------------------------------------------------------------
//
// stat[b] = {sqrt(mean(x^2) + eps)} (RMS, candle rms_norm) or {mean, 1 / sqrt(var + eps)}
// with var = E[x^2] - mean^2 (LayerNorm, candle layer_norm) of row b of p.x.

// Reference order: thread b sums row b's elements one after another, as the reference's CPU
// norm does (oracle: orc_rms_norm / orc_layer_norm). A 2048-element row is a ~4 us chain.
template <int NB>
__device__ __forceinline__ void norm_stats_sequential(const GemvParams& p, float (*stat)[2]) {
  const int b = threadIdx.x;
  if (b < NB && b < p.nb) {
    const float4* x = reinterpret_cast<const float4*>(p.x + b * p.x_stride);
    float s = 0.f, s2 = 0.f;
    const int n4 = p.k / 4;
    for (int i0 = 0; i0 < n4; i0 += 8) {
      float4 v[8];
#pragma unroll
      for (int u = 0; u < 8; u++) v[u] = i0 + u < n4 ? __ldcg(x + i0 + u) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int u = 0; u < 8; u++) {
        if (i0 + u >= n4) break;
        const float e[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
        for (int c = 0; c < 4; c++) {
          s = s + e[c];
          s2 = s2 + e[c] * e[c];
        }
      }
    }
    const float kf = (float)p.k;
    if (p.norm == NORM_RMS) {
      stat[b][0] = sqrtf(s2 / kf + p.eps);
    } else {
      const float mean = s / kf;
      stat[b][0] = mean;
      stat[b][1] = 1.0f / sqrtf(s2 / kf - mean * mean + p.eps);
    }
  }
}

// Finishes stat[b] from the CTA's partial sums (a, c) = (sum, sum of squares).
__device__ __forceinline__ void norm_finish(const GemvParams& p, float a, float c, float* st) {
  const float kf = (float)p.k;
  if (p.norm == NORM_RMS) {
    st[0] = sqrtf(c / kf + p.eps);
  } else {
    const float mean = a / kf;
    st[0] = mean;
    st[1] = 1.0f / sqrtf(c / kf - mean * mean + p.eps);
  }
}

// The normalised value of element i with value v of stream b (norm weights w, bias bb).
__device__ __forceinline__ float norm_apply(const GemvParams& p, const float* st, float v, float w,
                                            float bb) {
  if (p.norm == NORM_RMS) return v / st[0] * w;
  return (v - st[0]) * st[1] * w + bb;
}

constexpr int kMaxGroupsPerThread = 5;  // 8-element groups per thread: k <= 256 * 8 * 5

// Loads thread t's 8-element groups g = t + j * NT of row x (zeros past k / 8 groups).
template <int NT>
__device__ __forceinline__ void load_groups(const float* x, int ngr, float (&v)[kMaxGroupsPerThread][8]) {
  const int t = threadIdx.x;
#pragma unroll
  for (int j = 0; j < kMaxGroupsPerThread; j++) {
    const int g = t + j * NT;
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f), c = a;
    if (g < ngr) {
      a = __ldcg(reinterpret_cast<const float4*>(x + g * 8));
      c = __ldcg(reinterpret_cast<const float4*>(x + g * 8) + 1);
    }
    v[j][0] = a.x; v[j][1] = a.y; v[j][2] = a.z; v[j][3] = a.w;
    v[j][4] = c.x; v[j][5] = c.y; v[j][6] = c.z; v[j][7] = c.w;
  }
}

// Parallel norm statistics of one row whose groups thread t holds in v: warp sums into the
// row's slots of red, one barrier, then every thread adds the warps' sums (in the same order)
// into its own copy of the statistics, st.
template <int NT>
__device__ __forceinline__ void norm_stats_parallel(const GemvParams& p, const float (&v)[kMaxGroupsPerThread][8],
                                                    float (*red)[NT / 32], float* st) {
  constexpr int kWarps = NT / 32;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  float s = 0.f, s2 = 0.f;
#pragma unroll
  for (int j = 0; j < kMaxGroupsPerThread; j++)
#pragma unroll
    for (int e = 0; e < 8; e++) {
      s += v[j][e];
      s2 += v[j][e] * v[j][e];
    }
  s = warp_sum(s);
  s2 = warp_sum(s2);
  if (lane == 0) {
    red[0][warp] = s;
    red[1][warp] = s2;
  }
  __syncthreads();
  float a = 0.f, c = 0.f;
#pragma unroll
  for (int w = 0; w < kWarps; w++) {
    a += red[0][w];
    c += red[1][w];
  }
  norm_finish(p, a, c, st);
}

// The norm weights (and LayerNorm bias) of thread t's first kPreGroups groups, loaded before
// the kernel waits on its predecessor (they are constants), so the record build does not
// wait on them.
constexpr int kPreGroups = 2;
struct NormPre {
  float w[kPreGroups][8], b[kPreGroups][8];
};

template <int NT>
__device__ __forceinline__ void norm_preload(const GemvParams& p, NormPre& n) {
  const int t = threadIdx.x, ngr = p.k / 8;
#pragma unroll
  for (int j = 0; j < kPreGroups; j++) {
    const int g = t + j * NT;
#pragma unroll
    for (int e = 0; e < 8; e++) {
      n.w[j][e] = 0.f;
      n.b[j][e] = 0.f;
    }
    if (p.norm == NORM_NONE || g >= ngr) continue;
    const float4 wa = __ldg(reinterpret_cast<const float4*>(p.norm_w + g * 8));
    const float4 wc = __ldg(reinterpret_cast<const float4*>(p.norm_w + g * 8) + 1);
    n.w[j][0] = wa.x; n.w[j][1] = wa.y; n.w[j][2] = wa.z; n.w[j][3] = wa.w;
    n.w[j][4] = wc.x; n.w[j][5] = wc.y; n.w[j][6] = wc.z; n.w[j][7] = wc.w;
    if (p.norm == NORM_LAYER) {
      const float4 ba = __ldg(reinterpret_cast<const float4*>(p.norm_b + g * 8));
      const float4 bc = __ldg(reinterpret_cast<const float4*>(p.norm_b + g * 8) + 1);
      n.b[j][0] = ba.x; n.b[j][1] = ba.y; n.b[j][2] = ba.z; n.b[j][3] = ba.w;
      n.b[j][4] = bc.x; n.b[j][5] = bc.y; n.b[j][6] = bc.z; n.b[j][7] = bc.w;
    }
  }
}

// Normalises thread t's group j (values vv, element offset i0) in place.
template <int NT>
__device__ __forceinline__ void norm_group(const GemvParams& p, const NormPre& pre, int j, int i0,
                                           const float* st, float* vv) {
  float w8[8], b8[8];
  if (j < kPreGroups) {
#pragma unroll
    for (int e = 0; e < 8; e++) {
      w8[e] = pre.w[j < kPreGroups ? j : 0][e];
      b8[e] = pre.b[j < kPreGroups ? j : 0][e];
    }
  } else {
    const float4 wa = reinterpret_cast<const float4*>(p.norm_w + i0)[0];
    const float4 wc = reinterpret_cast<const float4*>(p.norm_w + i0)[1];
    w8[0] = wa.x; w8[1] = wa.y; w8[2] = wa.z; w8[3] = wa.w;
    w8[4] = wc.x; w8[5] = wc.y; w8[6] = wc.z; w8[7] = wc.w;
#pragma unroll
    for (int e = 0; e < 8; e++) b8[e] = 0.f;
    if (p.norm == NORM_LAYER) {
      const float4 ba = reinterpret_cast<const float4*>(p.norm_b + i0)[0];
      const float4 bc = reinterpret_cast<const float4*>(p.norm_b + i0)[1];
      b8[0] = ba.x; b8[1] = ba.y; b8[2] = ba.z; b8[3] = ba.w;
      b8[4] = bc.x; b8[5] = bc.y; b8[6] = bc.z; b8[7] = bc.w;
    }
  }
#pragma unroll
  for (int e = 0; e < 8; e++) vv[e] = norm_apply(p, st, vv[e], w8[e], b8[e]);
}

// ---- Dense input records (f32 / bf16 weights) --------------------------------------------
//
// Record of one stream: k f32 values (bf16-rounded for bf16 weights), padded to 16 bytes.
__host__ __device__ inline int dense_rec_bytes(int k) { return (k * 4 + 15) / 16 * 16; }

template <int WT, int NB, int NT = 256>
__device__ __forceinline__ void build_dense_records(const GemvParams& p, const NormPre& pre, uint8_t* xsm,
                                                    int rec, float (*red)[2][NT / 32], float (*stat)[2]) {
  const int t = threadIdx.x, k = p.k, ngr = k / 8;
  if (p.norm != NORM_NONE && p.ref_order) {
    norm_stats_sequential<NB>(p, stat);
    __syncthreads();
  }
  for (int b = 0; b < NB; b++) {
    if (b >= p.nb) break;
    float v[kMaxGroupsPerThread][8];
    load_groups<NT>(p.x + b * p.x_stride, ngr, v);
    float st[2] = {0.f, 0.f};
    if (p.norm != NORM_NONE) {
      if (p.ref_order) {
        st[0] = stat[b][0];
        st[1] = stat[b][1];
      } else {
        norm_stats_parallel<NT>(p, v, red[b], st);
      }
    }
    uint8_t* r = xsm + (size_t)b * rec;
#pragma unroll
    for (int j = 0; j < kMaxGroupsPerThread; j++) {
      const int g = t + j * NT;
      if (g >= ngr) break;
      const int i0 = g * 8;
      float* vv = v[j];
      if (p.norm != NORM_NONE) norm_group<NT>(p, pre, j, i0, st, vv);
      if (WT == W_BF16)
#pragma unroll
        for (int e = 0; e < 8; e++) vv[e] = round_bf16(vv[e]);
      float4* dst = reinterpret_cast<float4*>(r + (size_t)i0 * 4);
      dst[0] = make_float4(vv[0], vv[1], vv[2], vv[3]);
      dst[1] = make_float4(vv[4], vv[5], vv[6], vv[7]);
    }
  }
  __syncthreads();
}

// ---- Quantised weights: super-blocks -----------------------------------------------------
//
// Q8_0 and Q4_1 rows are stored in super-blocks of 8 quantisation blocks (256 values), laid
// out so that the 8 lanes of a row each stream one "slot" -- values 4l..4l+3 of every block --
// with 16-byte loads, which is the order in which the reference's CPU dot accumulates
// (candle's AVX2 vec_dot_q8_0_q8_0 / ggml's vec_dot_q4_1_q8_1: lane l of an 8-wide register
// accumulates d_w*d_x times the integer sum of slot l, block after block).
//
//  Q8_0 super-block s (272 bytes): [0,128) blocks 8s..8s+3 and [128,256) blocks 8s+4..8s+7,
//    each as 8 slots x (4 blocks x 4 bytes): byte (16 l + 4 j + e) of a half is element
//    4l + e of its block j; then [256,272) the 8 blocks' f16 scales d.
//  Q4_1 super-block s (160 bytes): [0,128) 4 byte groups m x (8 blocks x 4 bytes): byte
//    (32 m + 4 j + e) is byte 4m + e of block 8s+j (ggml nibble order: byte i holds values
//    i (low) and i + 16 (high)); then [128,160) the blocks' (f16 d, f16 m) pairs.
// Blocks past k / 32 in the last super-block are zero.
constexpr int kSbBlocks = 8;
constexpr int kQ8SbBytes = 272;
constexpr int kQ4SbBytes = 160;
__host__ __device__ inline int super_blocks(int k) { return (k / QBLK + kSbBlocks - 1) / kSbBlocks; }

// Quantised input record of one stream: the activation blocks (ggml Q8_0, or Q8_1 for Q4_1
// weights: candle's QMatMul quantises the input row the same way) in the weights' slot order,
// [super-block][half][slot][4 blocks x 4 bytes] int8 (256 bytes per super-block), then the
// blocks' scales d as f32 (8 per super-block), then for Q8_1 the blocks' f16-rounded
// s = d * sum(q) as f32.
__host__ __device__ inline int q_rec_bytes(int wtype, int k) {
  const int nsb = super_blocks(k);
  return nsb * 256 + nsb * kSbBlocks * 4 * (wtype == W_Q4 ? 2 : 1);
}

// Byte offset of slot l of block blk within the quants of a record (or a Q8_0 super-block row).
__host__ __device__ inline int q8_slot_offset(int blk, int l) {
  return (blk >> 3) * 256 + ((blk >> 2) & 1) * 128 + 16 * l + 4 * (blk & 3);
}

// Builds the NB quantised records: norm (optional), then per 32-value block d = amax / 127,
// q = round(x / d) with the reciprocal taken first (candle/ggml quantize_row_q8_0), d stored
// as its f16 value. Thread t owns the 8-element groups t, t + NT, ...; a block's four groups
// sit on four adjacent lanes.
template <int WT, int NB, int NT = 256>
__device__ __forceinline__ void build_q_records(const GemvParams& p, const NormPre& pre, uint8_t* xsm, int rec,
                                                float (*red)[2][NT / 32], float (*stat)[2]) {
  const int t = threadIdx.x, k = p.k, ngr = k / 8, nsb = super_blocks(k);
  if (p.norm != NORM_NONE && p.ref_order) {
    norm_stats_sequential<NB>(p, stat);
    __syncthreads();
  }
  for (int b = 0; b < NB; b++) {
    if (b >= p.nb) break;
    float v[kMaxGroupsPerThread][8];
    load_groups<NT>(p.x + b * p.x_stride, ngr, v);
    float st[2] = {0.f, 0.f};
    if (p.norm != NORM_NONE) {
      if (p.ref_order) {
        st[0] = stat[b][0];
        st[1] = stat[b][1];
      } else {
        norm_stats_parallel<NT>(p, v, red[b], st);
      }
    }
    uint8_t* r = xsm + (size_t)b * rec;
    float* dscale = reinterpret_cast<float*>(r + nsb * 256);
#pragma unroll
    for (int j = 0; j < kMaxGroupsPerThread; j++) {
      if (j * NT >= ngr) break;  // uniform: whole warps leave together
      const int g = t + j * NT;
      const bool on = g < ngr;
      const int i0 = (on ? g : 0) * 8;
      float* vv = v[j];
      if (p.norm != NORM_NONE) norm_group<NT>(p, pre, j, i0, st, vv);
      float amax = 0.f;
#pragma unroll
      for (int e = 0; e < 8; e++) amax = fmaxf(amax, fabsf(vv[e]));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
      const float d = amax / 127.0f;
      const float id = d != 0.0f ? 1.0f / d : 0.0f;
      int sum = 0;
      uint32_t w2[2];
#pragma unroll
      for (int h = 0; h < 2; h++) {
        uint32_t word = 0;
#pragma unroll
        for (int e = 0; e < 4; e++) {
          const int q = (int)roundf(vv[4 * h + e] * id);
          sum += q;
          word |= ((uint32_t)q & 0xffu) << (8 * e);
        }
        w2[h] = word;
      }
      sum += __shfl_xor_sync(0xffffffffu, sum, 1);
      sum += __shfl_xor_sync(0xffffffffu, sum, 2);
      if (on) {
        // Group g holds slots 2 (g & 3) and 2 (g & 3) + 1 of block g / 4.
        const int blk = g >> 2, l0 = 2 * (g & 3);
        *reinterpret_cast<uint32_t*>(r + q8_slot_offset(blk, l0)) = w2[0];
        *reinterpret_cast<uint32_t*>(r + q8_slot_offset(blk, l0 + 1)) = w2[1];
        if ((g & 3) == 0) {
          dscale[blk] = f16_round(d);
          if (WT == W_Q4) dscale[nsb * kSbBlocks + blk] = f16_round((float)sum * d);
        }
      }
    }
  }
  __syncthreads();
}

}  // namespace svl
