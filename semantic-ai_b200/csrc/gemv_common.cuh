// gemv_common.cuh — device code shared by the matrix-vector kernel (gemv.cu) and the
// persistent step kernel (stepk.cu): the argmax order, the fused epilogue, and the input
// records (norm + the weight format's activation conversion) in shared memory.
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

__host__ __device__ inline int chunks_per_row(int wt, int k) {
  switch (wt) {
    case W_F32: return k / 4;
    case W_BF16: return k / 8;
    case W_Q8: return k / 16;
    default: return k / 32;
  }
}

// The fused epilogue for row `row` of stream b (value v; v_pair is the other row of the
// aligned pair, for RoPE and SwiGLU).
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
        // rope_i (candle; nn/transformer.rs:339-340): pairs (2i, 2i+1) rotate by pos * f_i.
        const int dim = row % hd, i = dim >> 1;
        float sn, cs;
        sincosf((float)pos * p.inv_freq[i], &sn, &cs);
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

// Input record of one stream in shared memory. F32 / BF16: k f32 (bf16-rounded for BF16).
// Q8 / Q4: k int8 (Q8_0 / Q8_1 activation blocks), then k/32 f32 scales d, then (Q4) k/32
// f32 block sums s = d * sum(q). Padded to 16 bytes.
__host__ __device__ inline int rec_bytes_of(int wtype, int k) {
  const int b = (wtype == W_F32 || wtype == W_BF16) ? k * 4 : k + (k / QBLK) * 4 * (wtype == W_Q4 ? 2 : 1);
  return (b + 15) / 16 * 16;
}

constexpr int kMaxGroupsPerThread = 5;  // 8-element groups per thread: k <= 256 * 8 * 5

// Builds the NB input records from the raw rows p.x: thread t owns the 8-element groups
// t, t + 256, ... (so the four groups of a 32-element block sit on four adjacent lanes).
template <int WT, int NB, int NT = 256, class Sync>
__device__ __forceinline__ void build_records(const GemvParams& p, uint8_t* xsm, int rec,
                                              float (*red)[NT / 32], float* stat, Sync sync) {
  constexpr int kThreads = NT, kWarps = NT / 32;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5, k = p.k, ngr = k / 8, nblk = k / QBLK;
  for (int b = 0; b < NB; b++) {
    if (b >= p.nb) break;
    float v[kMaxGroupsPerThread][8];
    const float* x = p.x + b * p.x_stride;
#pragma unroll
    for (int j = 0; j < kMaxGroupsPerThread; j++) {
      const int g = t + j * kThreads;
      float4 a = make_float4(0.f, 0.f, 0.f, 0.f), c = a;
      if (g < ngr) {
        a = __ldcg(reinterpret_cast<const float4*>(x + g * 8));
        c = __ldcg(reinterpret_cast<const float4*>(x + g * 8) + 1);
      }
      v[j][0] = a.x; v[j][1] = a.y; v[j][2] = a.z; v[j][3] = a.w;
      v[j][4] = c.x; v[j][5] = c.y; v[j][6] = c.z; v[j][7] = c.w;
    }
    if (p.norm != NORM_NONE) {
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
      sync();
      if (t == 0) {
        float a = 0.f, c = 0.f;
        for (int w = 0; w < kWarps; w++) {
          a += red[0][w];
          c += red[1][w];
        }
        if (p.norm == NORM_RMS) {
          stat[0] = sqrtf(c / (float)k + p.eps);  // candle rms_norm: sqrt(mean(x^2) + eps)
        } else {
          const float mean = a / (float)k;        // candle layer_norm: E[x^2] - mean^2
          const float var = c / (float)k - mean * mean;
          stat[0] = mean;
          stat[1] = 1.0f / sqrtf(var + p.eps);
        }
      }
      sync();
    }
    uint8_t* r = xsm + (size_t)b * rec;
#pragma unroll
    for (int j = 0; j < kMaxGroupsPerThread; j++) {
      if (j * kThreads >= ngr) break;
      const int g = t + j * kThreads;
      const bool on = g < ngr;
      const int i0 = (on ? g : 0) * 8;
      float* vv = v[j];
      if (p.norm != NORM_NONE) {
        const float4 wa = reinterpret_cast<const float4*>(p.norm_w + i0)[0];
        const float4 wc = reinterpret_cast<const float4*>(p.norm_w + i0)[1];
        const float w8[8] = {wa.x, wa.y, wa.z, wa.w, wc.x, wc.y, wc.z, wc.w};
        if (p.norm == NORM_RMS) {
#pragma unroll
          for (int e = 0; e < 8; e++) vv[e] = vv[e] / stat[0] * w8[e];
        } else {
          const float4 ba = reinterpret_cast<const float4*>(p.norm_b + i0)[0];
          const float4 bc = reinterpret_cast<const float4*>(p.norm_b + i0)[1];
          const float b8[8] = {ba.x, ba.y, ba.z, ba.w, bc.x, bc.y, bc.z, bc.w};
#pragma unroll
          for (int e = 0; e < 8; e++) vv[e] = (vv[e] - stat[0]) * stat[1] * w8[e] + b8[e];
        }
      }
      if (WT == W_F32 || WT == W_BF16) {
        if (on) {
          if (WT == W_BF16)
#pragma unroll
            for (int e = 0; e < 8; e++) vv[e] = round_bf16(vv[e]);
          float4* dst = reinterpret_cast<float4*>(r + (size_t)i0 * 4);
          dst[0] = make_float4(vv[0], vv[1], vv[2], vv[3]);
          dst[1] = make_float4(vv[4], vv[5], vv[6], vv[7]);
        }
      } else {
        // ggml/candle activation block: d = amax / 127, q = round(x * (1 / d)).
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
          *reinterpret_cast<uint2*>(r + i0) = make_uint2(w2[0], w2[1]);
          if ((g & 3) == 0) {
            float* dd = reinterpret_cast<float*>(r + k);
            dd[g >> 2] = f16_round(d);
            if (WT == W_Q4) dd[nblk + (g >> 2)] = f16_round((float)sum * d);
          }
        }
      }
    }
  }
  sync();
}


}  // namespace svl
