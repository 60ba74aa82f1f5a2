// gemv.cu — weight-streaming matrix-vector products for small stream counts.
//
// At batch 1 the step is bound by reading every weight once (nn/mod.rs:91-99 runs the
// same product on the CPU through kernels::matvec, nn/kernels/matvec.rs:29-58). Each CTA
// first applies the layer's norm to the input row(s) and converts them for the weight
// format (bf16 rounding, or Q8_0 / Q8_1 blocks as candle's QMatMul quantises the
// activation), then its warps stream groups of R rows with 16-byte loads, U loads per row
// in flight, and finish each group with a fused epilogue (RoPE + KV-ring write, SwiGLU,
// GELU, residual add, logits + argmax).
#include "common.cuh"
#include "kernels.cuh"

#include <climits>

namespace svl {

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

template <int WT> struct Tile;
template <> struct Tile<W_F32> { static constexpr int R = 2, U = 8; };
template <> struct Tile<W_BF16> { static constexpr int R = 4, U = 4; };
template <> struct Tile<W_Q8> { static constexpr int R = 4, U = 4; };
template <> struct Tile<W_Q4> { static constexpr int R = 4, U = 4; };

// 16-byte chunks per row for each format.
__host__ __device__ inline int chunks_per_row(int wt, int k) {
  switch (wt) {
    case W_F32: return k / 4;
    case W_BF16: return k / 8;
    case W_Q8: return k / 16;
    default: return k / 32;
  }
}

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
  if (v != v) return false;
  if (bi == INT_MAX) return true;
  return v > bv || (v == bv && i < bi);
}

__device__ __forceinline__ int dp4a(int a, int b, int c) { return __dp4a(a, b, c); }

template <int WT, int NB>
__global__ void __launch_bounds__(kThreads) gemv_kernel(const GemvParams p) {
  constexpr int R = Tile<WT>::R;
  constexpr int U = Tile<WT>::U;
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ float red_a[kWarps][NB], red_b[kWarps][NB];
  __shared__ float stat_a[NB], stat_b[NB];
  __shared__ float am_v[kWarps][NB];
  __shared__ int am_i[kWarps][NB];
  __shared__ bool am_last;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int k = p.k;
  const int nb = p.nb;

  // ---- prologue 1: norm statistics of each input row.
  if (p.norm != NORM_NONE) {
    float s[NB], s2[NB];
#pragma unroll
    for (int b = 0; b < NB; b++) {
      s[b] = 0.f;
      s2[b] = 0.f;
      if (b < nb) {
        const float* x = p.x + b * p.x_stride;
        for (int i = tid; i < k; i += kThreads) {
          float v = x[i];
          s[b] += v;
          s2[b] += v * v;
        }
      }
      s[b] = warp_sum(s[b]);
      s2[b] = warp_sum(s2[b]);
      if (lane == 0) {
        red_a[warp][b] = s[b];
        red_b[warp][b] = s2[b];
      }
    }
    __syncthreads();
    if (tid < NB) {
      float a = 0.f, c = 0.f;
      for (int w = 0; w < kWarps; w++) {
        a += red_a[w][tid];
        c += red_b[w][tid];
      }
      if (p.norm == NORM_RMS) {
        // candle rms_norm: m = sqrt(sum(x^2) / d + eps)
        stat_a[tid] = sqrtf(c / (float)k + p.eps);
      } else {
        // candle layer_norm: var = E[x^2] - mean^2, inv_std = 1 / sqrt(var + eps)
        float mean = a / (float)k;
        float var = c / (float)k - mean * mean;
        stat_a[tid] = mean;
        stat_b[tid] = 1.0f / sqrtf(var + p.eps);
      }
    }
    __syncthreads();
  }

  auto normed = [&](int b, int i) -> float {
    float v = p.x[b * p.x_stride + i];
    if (p.norm == NORM_RMS) {
      v = v / stat_a[b] * p.norm_w[i];
    } else if (p.norm == NORM_LAYER) {
      v = (v - stat_a[b]) * stat_b[b] * p.norm_w[i] + p.norm_b[i];
    }
    return v;
  };

  // ---- prologue 2: the converted input rows in shared memory.
  float* xs = reinterpret_cast<float*>(smem);                     // F32 / BF16: [NB][k]
  int8_t* xq = reinterpret_cast<int8_t*>(smem);                   // Q8 / Q4: [NB][k]
  float* xd = reinterpret_cast<float*>(smem + (size_t)NB * k);    // [NB][k/32]
  float* xsum = xd + (size_t)NB * (k / QBLK);                     // [NB][k/32] (Q4 only)
  if (WT == W_F32 || WT == W_BF16) {
    for (int b = 0; b < NB; b++)
      for (int i = tid; i < k; i += kThreads) {
        float v = b < nb ? normed(b, i) : 0.f;
        xs[b * k + i] = WT == W_BF16 ? round_bf16(v) : v;
      }
  } else {
    const int nblk = k / QBLK;
    for (int b = 0; b < NB; b++)
      for (int blk = warp; blk < nblk; blk += kWarps) {
        float v = b < nb ? normed(b, blk * QBLK + lane) : 0.f;
        // ggml/candle Q8_0 (and Q8_1) block: d = amax / 127, q = round(x * (1 / d)).
        float amax = warp_max(fabsf(v));
        float d = amax / 127.0f;
        float id = d != 0.0f ? 1.0f / d : 0.0f;
        int q = (int)roundf(v * id);
        xq[b * k + blk * QBLK + lane] = (int8_t)q;
        if (WT == W_Q4) {
          int sum = warp_sum_int(q);
          if (lane == 0) xsum[b * nblk + blk] = f16_round((float)sum * d);
        }
        if (lane == 0) xd[b * nblk + blk] = f16_round(d);
      }
  }
  __syncthreads();

  // ---- main loop: groups of R rows per warp.
  const int nch = chunks_per_row(WT, k);
  const int groups = (p.n + R - 1) / R;
  float best_v = 0.f;
  int best_i = INT_MAX;

  for (int g = blockIdx.x * kWarps + warp; g < groups; g += gridDim.x * kWarps) {
    const int r0 = g * R;
    float acc[R][NB];
#pragma unroll
    for (int r = 0; r < R; r++)
#pragma unroll
      for (int b = 0; b < NB; b++) acc[r][b] = 0.f;

    for (int c0 = 0; c0 < nch; c0 += 32 * U) {
      uint4 wv[R][U];
#pragma unroll
      for (int r = 0; r < R; r++)
#pragma unroll
        for (int u = 0; u < U; u++) {
          int c = c0 + lane + 32 * u;
          if (c < nch && r0 + r < p.n)
            wv[r][u] = ldg_stream(p.w + (int64_t)(r0 + r) * p.row_stride + (int64_t)c * 16);
          else
            wv[r][u] = make_uint4(0, 0, 0, 0);
        }
#pragma unroll
      for (int u = 0; u < U; u++) {
        const int c = c0 + lane + 32 * u;
        const bool valid = c < nch;
        if (WT == W_F32) {
          if (valid) {
#pragma unroll
            for (int b = 0; b < NB; b++) {
              float4 xv = reinterpret_cast<const float4*>(xs + b * k)[c];
#pragma unroll
              for (int r = 0; r < R; r++) {
                float4 w = *reinterpret_cast<float4*>(&wv[r][u]);
                acc[r][b] = fmaf(w.x, xv.x, acc[r][b]);
                acc[r][b] = fmaf(w.y, xv.y, acc[r][b]);
                acc[r][b] = fmaf(w.z, xv.z, acc[r][b]);
                acc[r][b] = fmaf(w.w, xv.w, acc[r][b]);
              }
            }
          }
        } else if (WT == W_BF16) {
          if (valid) {
#pragma unroll
            for (int b = 0; b < NB; b++) {
              float4 x0 = reinterpret_cast<const float4*>(xs + b * k)[2 * c];
              float4 x1 = reinterpret_cast<const float4*>(xs + b * k)[2 * c + 1];
#pragma unroll
              for (int r = 0; r < R; r++) {
                uint4 w = wv[r][u];
                float a = acc[r][b];
                a = fmaf(bf16_lo(w.x), x0.x, a);
                a = fmaf(bf16_hi(w.x), x0.y, a);
                a = fmaf(bf16_lo(w.y), x0.z, a);
                a = fmaf(bf16_hi(w.y), x0.w, a);
                a = fmaf(bf16_lo(w.z), x1.x, a);
                a = fmaf(bf16_hi(w.z), x1.y, a);
                a = fmaf(bf16_lo(w.w), x1.z, a);
                a = fmaf(bf16_hi(w.w), x1.w, a);
                acc[r][b] = a;
              }
            }
          }
        } else if (WT == W_Q8) {
          // Chunk c holds half of block c/2; lanes 2j and 2j+1 share a block.
          const int blk = c >> 1;
          const int nblk = k / QBLK;
#pragma unroll
          for (int b = 0; b < NB; b++) {
            int4 xv = valid ? reinterpret_cast<const int4*>(xq + b * k)[c] : make_int4(0, 0, 0, 0);
            float dx = valid ? xd[b * nblk + blk] : 0.f;
#pragma unroll
            for (int r = 0; r < R; r++) {
              uint4 w = wv[r][u];
              int s = dp4a((int)w.x, xv.x, 0);
              s = dp4a((int)w.y, xv.y, s);
              s = dp4a((int)w.z, xv.z, s);
              s = dp4a((int)w.w, xv.w, s);
              s += __shfl_xor_sync(0xffffffffu, s, 1);
              if (valid && !(lane & 1) && r0 + r < p.n) {
                const __half* scales = reinterpret_cast<const __half*>(
                    p.w + (int64_t)(r0 + r) * p.row_stride + k);
                float dd = __half2float(scales[blk]) * dx;
                acc[r][b] = fmaf(dd, (float)s, acc[r][b]);
              }
            }
          }
        } else {  // W_Q4: chunk c is block c (16 bytes of nibbles, ggml Q4_1 order).
          const int nblk = k / QBLK;
          if (valid) {
#pragma unroll
            for (int b = 0; b < NB; b++) {
              const int4* xb = reinterpret_cast<const int4*>(xq + b * k + c * QBLK);
              int4 xlo = xb[0], xhi = xb[1];
              float dx = xd[b * nblk + c], sx = xsum[b * nblk + c];
#pragma unroll
              for (int r = 0; r < R; r++) {
                if (r0 + r >= p.n) continue;
                uint4 w = wv[r][u];
                int s = 0;
                s = dp4a((int)(w.x & 0x0f0f0f0fu), xlo.x, s);
                s = dp4a((int)(w.y & 0x0f0f0f0fu), xlo.y, s);
                s = dp4a((int)(w.z & 0x0f0f0f0fu), xlo.z, s);
                s = dp4a((int)(w.w & 0x0f0f0f0fu), xlo.w, s);
                s = dp4a((int)((w.x >> 4) & 0x0f0f0f0fu), xhi.x, s);
                s = dp4a((int)((w.y >> 4) & 0x0f0f0f0fu), xhi.y, s);
                s = dp4a((int)((w.z >> 4) & 0x0f0f0f0fu), xhi.z, s);
                s = dp4a((int)((w.w >> 4) & 0x0f0f0f0fu), xhi.w, s);
                const __half2* dm = reinterpret_cast<const __half2*>(
                    p.w + (int64_t)(r0 + r) * p.row_stride + k / 2);
                float2 f = __half22float2(dm[c]);
                acc[r][b] += (f.x * dx) * (float)s + f.y * sx;
              }
            }
          }
        }
      }
    }
#pragma unroll
    for (int r = 0; r < R; r++)
#pragma unroll
      for (int b = 0; b < NB; b++) acc[r][b] = warp_sum(acc[r][b]);

    // ---- epilogue: lane j owns (row r0 + j / NB, stream j % NB).
    if (p.epi == EPI_LOGITS && lane < NB && lane < nb) {
#pragma unroll
      for (int r = 0; r < R; r++) {
        int row = r0 + r;
        if (row < p.n) {
          float v = acc[r][lane] + (p.bias ? p.bias[row] : 0.f);
          if (better(v, row, best_v, best_i)) {
            best_v = v;
            best_i = row;
          }
        }
      }
    }
#pragma unroll
    for (int j = 0; j < R * NB; j++) {
      if (lane != j) continue;
      const int r = j / NB, b = j % NB, row = r0 + r;
      if (b >= nb || row >= p.n) continue;
      float v = acc[r][b];
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
          if (!(r & 1)) {
            float g = v, val = acc[r | 1][b];
            p.out[b * p.out_stride + row / 2] = silu_ref(g) * val;
          }
          break;
        case EPI_QKV_ROPE: {
          const int hd = p.head_dim;
          const int pos = p.pos[b];
          if (row < p.q_dim + p.kv_dim) {
            // rope_i (candle, used at nn/transformer.rs:339-340): pairs (2i, 2i+1).
            const int dim = row % hd, i = dim >> 1;
            const float a = acc[r & ~1][b], c2 = acc[r | 1][b];
            float sn, cs;
            sincosf((float)pos * p.inv_freq[i], &sn, &cs);
            float val = (dim & 1) ? a * sn + c2 * cs : a * cs - c2 * sn;
            if (row < p.q_dim) {
              p.out[b * p.out_stride + row] = val;
            } else {
              const int kh = (row - p.q_dim) / hd;
              const int slot = p.windowed ? pos % p.ring_cap : pos;
              int64_t off = b * p.ring_stream_stride + ((int64_t)kh * p.ring_cap + slot) * hd + dim;
              if (p.kv_bf16)
                reinterpret_cast<__nv_bfloat16*>(p.k_ring)[off] = __float2bfloat16_rn(val);
              else
                reinterpret_cast<float*>(p.k_ring)[off] = val;
            }
          } else {
            const int vr = row - p.q_dim - p.kv_dim;
            const int kh = vr / hd, dim = vr % hd;
            const int slot = p.windowed ? pos % p.ring_cap : pos;
            int64_t off = b * p.ring_stream_stride + ((int64_t)kh * p.ring_cap + slot) * hd + dim;
            if (p.kv_bf16)
              reinterpret_cast<__nv_bfloat16*>(p.v_ring)[off] = __float2bfloat16_rn(v);
            else
              reinterpret_cast<float*>(p.v_ring)[off] = v;
          }
          break;
        }
      }
    }
  }

  // ---- argmax: CTA best, then the last CTA reduces the CTA bests.
  if (p.epi == EPI_LOGITS) {
    if (lane < NB) {
      am_v[warp][lane] = best_v;
      am_i[warp][lane] = best_i;
    }
    __syncthreads();
    if (tid < nb && tid < NB) {
      float bv = 0.f;
      int bi = INT_MAX;
      for (int w = 0; w < kWarps; w++)
        if (am_i[w][tid] != INT_MAX && better(am_v[w][tid], am_i[w][tid], bv, bi)) {
          bv = am_v[w][tid];
          bi = am_i[w][tid];
        }
      p.am_val[tid * gridDim.x + blockIdx.x] = bv;
      p.am_idx[tid * gridDim.x + blockIdx.x] = bi;
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) am_last = atomicAdd(p.am_ticket, 1u) == gridDim.x - 1;
    __syncthreads();
    if (am_last) {
      __threadfence();
      if (tid < nb && tid < NB) {
        float bv = 0.f;
        int bi = INT_MAX;
        for (int g = 0; g < (int)gridDim.x; g++) {
          float v = __ldcg(p.am_val + tid * gridDim.x + g);
          int i = __ldcg(p.am_idx + tid * gridDim.x + g);
          if (i != INT_MAX && better(v, i, bv, bi)) {
            bv = v;
            bi = i;
          }
        }
        p.tokens[tid] = bi == INT_MAX ? 0u : (uint32_t)bi;
      }
      if (tid == 0) *p.am_ticket = 0u;
    }
  }
}

template <int WT, int NB>
size_t smem_bytes(int k) {
  if (WT == W_F32 || WT == W_BF16) return (size_t)NB * k * 4;
  return (size_t)NB * k + (size_t)NB * (k / QBLK) * 4 * (WT == W_Q4 ? 2 : 1);
}

constexpr size_t kMaxSmem = 200 * 1024;

template <int WT, int NB>
void launch_t(const GemvParams& p, cudaStream_t s) {
  constexpr int R = Tile<WT>::R;
  size_t sm = smem_bytes<WT, NB>(p.k);
  int groups = (p.n + R - 1) / R;
  int grid = (groups + kWarps - 1) / kWarps;
  int max_grid = p.epi == EPI_LOGITS ? kLogitsGrid : 2 * 148;
  if (grid > max_grid) grid = max_grid;
  gemv_kernel<WT, NB><<<grid, kThreads, sm, s>>>(p);
}

template <int WT>
void set_attrs() {
  cudaFuncSetAttribute(gemv_kernel<WT, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem);
  cudaFuncSetAttribute(gemv_kernel<WT, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem);
  cudaFuncSetAttribute(gemv_kernel<WT, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem);
  cudaFuncSetAttribute(gemv_kernel<WT, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem);
}

// Streams per launch: the largest template width whose input rows fit in shared memory.
template <int WT>
int max_nb(int k) {
  if (smem_bytes<WT, 8>(k) <= kMaxSmem) return 8;
  if (smem_bytes<WT, 4>(k) <= kMaxSmem) return 4;
  if (smem_bytes<WT, 2>(k) <= kMaxSmem) return 2;
  return 1;
}

template <int WT>
void launch_w(const GemvParams& p0, cudaStream_t s) {
  const int cap = max_nb<WT>(p0.k);
  for (int b0 = 0; b0 < p0.nb; b0 += cap) {
    GemvParams p = p0;
    p.nb = p0.nb - b0 < cap ? p0.nb - b0 : cap;
    p.x = p0.x + b0 * p0.x_stride;
    if (p0.out) p.out = p0.out + b0 * p0.out_stride;
    if (p0.pos) p.pos = p0.pos + b0;
    if (p0.tokens) p.tokens = p0.tokens + b0;
    if (p0.k_ring) {
      size_t el = p0.kv_bf16 ? 2 : 4;
      p.k_ring = static_cast<uint8_t*>(p0.k_ring) + b0 * p0.ring_stream_stride * el;
      p.v_ring = static_cast<uint8_t*>(p0.v_ring) + b0 * p0.ring_stream_stride * el;
    }
    switch (p.nb) {
      case 1: launch_t<WT, 1>(p, s); break;
      case 2: launch_t<WT, 2>(p, s); break;
      case 3:
      case 4: launch_t<WT, 4>(p, s); break;
      default: launch_t<WT, 8>(p, s); break;
    }
  }
}

}  // namespace

void gemv_init_device() {
  set_attrs<W_F32>();
  set_attrs<W_BF16>();
  set_attrs<W_Q8>();
  set_attrs<W_Q4>();
}

void launch_gemv(const GemvParams& p, cudaStream_t s) {
  switch (p.wtype) {
    case W_F32: launch_w<W_F32>(p, s); break;
    case W_BF16: launch_w<W_BF16>(p, s); break;
    case W_Q8: launch_w<W_Q8>(p, s); break;
    default: launch_w<W_Q4>(p, s); break;
  }
}

}  // namespace svl
