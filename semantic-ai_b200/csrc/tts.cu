// tts.cu — the per-stream pieces of the Pocket-TTS FlowLm step (tts/flow_lm.rs:162-387) that
// are not weight products: the LayerNorm + EOS head, the timestep embedding's input and
// normalisation, AdaLN modulation, gated residuals and the latent update. The weight products
// (input_linear, cond_embed, input_proj, the residual blocks' MLPs and modulations, the final
// layer) run on the matrix-vector kernel or, for many bf16 streams, on the tensor cores.
#include <cuda_bf16.h>

#include "common.cuh"
#include "kernels.cuh"
#include "sm100.cuh"

namespace svl {
namespace {

constexpr int kT = 256;

// Block-wide sum of one value per thread (kT threads).
__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
  for (int w = 0; w < (int)(blockDim.x >> 5); w++) t += red[w];
  return t;
}

// One CTA per stream: z = layer_norm(x; w, b, eps) (candle: E[x^2] - mean^2,
// transformer.rs:284 / flow_lm.rs:176), eos = out_eos . z + bias (flow_lm.rs:177).
__global__ void __launch_bounds__(kT) tts_head_kernel(const float* x, int d, const float* lnw,
                                                      const float* lnb, float eps,
                                                      const float* w_eos, const float* b_eos,
                                                      float* z, float* eos) {
  __shared__ float red[kT / 32];
  pdl_launch();
  pdl_wait();
  const int b = blockIdx.x;
  const float* xr = x + (int64_t)b * d;
  float s = 0.f, s2 = 0.f;
  for (int i = threadIdx.x; i < d; i += kT) {
    const float v = xr[i];
    s += v;
    s2 += v * v;
  }
  s = block_sum(s, red);
  s2 = block_sum(s2, red);
  const float mean = s / (float)d;
  const float inv = 1.0f / sqrtf(s2 / (float)d - mean * mean + eps);
  float dot = 0.f;
  for (int i = threadIdx.x; i < d; i += kT) {
    const float zi = (xr[i] - mean) * inv * lnw[i] + lnb[i];
    z[(int64_t)b * d + i] = zi;
    dot = fmaf(zi, w_eos[i], dot);
  }
  dot = block_sum(dot, red);
  if (threadIdx.x == 0) eos[b] = dot + b_eos[0];
}

// TimestepEmbedder input (flow_lm.rs:339-343): [cos(freqs * t), sin(freqs * t)], 128 each.
__global__ void time_input_kernel(const float* freqs, float t, float* emb) {
  pdl_launch();
  pdl_wait();
  const int i = threadIdx.x;
  if (i < 128) {
    const float a = freqs[i] * t;
    emb[i] = cosf(a);
    emb[128 + i] = sinf(a);
  }
}

// TimestepEmbedder output norm (flow_lm.rs:345-351): te * rsqrt(var + 1e-5) * alpha with the
// unbiased variance over dim; accumulated into tsum (first embedder sets it).
__global__ void __launch_bounds__(1024) time_norm_kernel(const float* te, int dim, const float* alpha,
                                                         float* tsum, int first) {
  __shared__ float red[32];
  pdl_launch();
  pdl_wait();
  const int i = threadIdx.x;
  const float v = i < dim ? te[i] : 0.f;
  const float mean = block_sum(v, red) * (float)(1.0 / (double)dim);
  const float c = i < dim ? v - mean : 0.f;
  const float var = block_sum(c * c, red) * (float)(1.0 / (double)(dim - 1));
  const float r = 1.0f / sqrtf(var + 1e-5f);
  if (i < dim) {
    const float o = v * r * alpha[i];
    tsum[i] = first ? o : tsum[i] + o;
  }
}

// FlowHead::forward (flow_lm.rs:266-275): sy = silu(y + tsum / n_time), n_time 0: silu(y).
__global__ void cond_silu_kernel(const float* y, const float* tsum, float inv_n, int dim, int64_t n,
                                 float* sy) {
  pdl_launch();
  pdl_wait();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float v = y[i];
  if (tsum) v = v + tsum[i % dim] * inv_n;
  sy[i] = silu_ref(v);
}

// AdaLN (ResBlock::forward, flow_lm.rs:373-386, and the final layer, :377-383): one CTA per
// stream, hh = norm(xs) * (1 + scale) + shift with (shift, scale) = mod[0:dim], mod[dim:2dim].
// affine: candle layer_norm with weight and bias (E[x^2] - mean^2); otherwise
// layer_norm_no_affine (flow_lm.rs:226-231): centred values, mean of their squares.
__global__ void __launch_bounds__(kT) adaln_kernel(const float* xs, int dim, const float* lnw,
                                                   const float* lnb, int affine, float eps,
                                                   const float* mod, int64_t mod_stride,
                                                   float* hh) {
  __shared__ float red[kT / 32];
  pdl_launch();
  pdl_wait();
  const int b = blockIdx.x;
  const float* xr = xs + (int64_t)b * dim;
  const float* mr = mod + (int64_t)b * mod_stride;
  float s = 0.f, s2 = 0.f;
  for (int i = threadIdx.x; i < dim; i += kT) {
    const float v = xr[i];
    s += v;
    s2 += v * v;
  }
  s = block_sum(s, red);
  float mean, inv;
  if (affine) {
    s2 = block_sum(s2, red);
    mean = s / (float)dim;
    inv = 1.0f / sqrtf(s2 / (float)dim - mean * mean + eps);
  } else {
    const float inv_n = (float)(1.0 / (double)dim);
    mean = s * inv_n;
    float c2 = 0.f;
    for (int i = threadIdx.x; i < dim; i += kT) {
      const float c = xr[i] - mean;
      c2 += c * c;
    }
    c2 = block_sum(c2, red);
    inv = 1.0f / sqrtf(c2 * inv_n + eps);
  }
  for (int i = threadIdx.x; i < dim; i += kT) {
    float h = affine ? (xr[i] - mean) * inv * lnw[i] + lnb[i] : (xr[i] - mean) * inv;
    hh[(int64_t)b * dim + i] = h * (mr[dim + i] + 1.0f) + mr[i];
  }
}

// Gated residual (flow_lm.rs:385): xs += gate * h, gate = mod[gate_off : gate_off + dim].
__global__ void gate_add_kernel(float* xs, const float* mod, int64_t mod_stride, int gate_off,
                                const float* h, int dim, int64_t n) {
  pdl_launch();
  pdl_wait();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int64_t b = i / dim, j = i % dim;
  xs[i] = xs[i] + mod[b * mod_stride + gate_off + j] * h[i];
}

// FlowHead::decode (flow_lm.rs:290-315): mode 0 x += flow * scale (lsd, flow matching),
// 1 x = flow (drifting), 2 x += flow (pointwise).
__global__ void flow_update_kernel(float* x, const float* flow, int64_t n, int mode, float scale) {
  pdl_launch();
  pdl_wait();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  x[i] = mode == 0 ? x[i] + flow[i] * scale : mode == 1 ? flow[i] : x[i] + flow[i];
}

// FlowLm::prompt_text (flow_lm.rs:150-158): x[b] = conditioner row tokens[b * n + t].
__global__ void prompt_embed_kernel(const float* table, const uint32_t* tokens, int n, int t, int d,
                                    int bins, float* x, int* err) {
  pdl_launch();
  pdl_wait();
  const int b = blockIdx.x;
  uint32_t tok = tokens[(int64_t)b * n + t];
  if (tok > (uint32_t)bins) {
    if (threadIdx.x == 0) atomicExch(err, 1);
    tok = 0;
  }
  for (int i = threadIdx.x; i < d; i += blockDim.x)
    x[(int64_t)b * d + i] = table[(int64_t)tok * d + i];
}

template <class K, class... Args>
void launch_pdl(K kernel, dim3 grid, dim3 block, cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, kernel, args...);
}

unsigned blocks_for(int64_t n) { return (unsigned)((n + 255) / 256); }

}  // namespace

void launch_tts_head(const float* x, int nb, int d, const float* lnw, const float* lnb, float eps,
                     const float* w_eos, const float* b_eos, float* z, float* eos, cudaStream_t s) {
  launch_pdl(tts_head_kernel, dim3(nb), dim3(kT), s, x, d, lnw, lnb, eps, w_eos, b_eos, z, eos);
}
void launch_time_input(const float* freqs, float t, float* emb, cudaStream_t s) {
  launch_pdl(time_input_kernel, dim3(1), dim3(128), s, freqs, t, emb);
}
void launch_time_norm(const float* te, int dim, const float* alpha, float* tsum, int first,
                      cudaStream_t s) {
  launch_pdl(time_norm_kernel, dim3(1), dim3((dim + 31) / 32 * 32), s, te, dim, alpha, tsum, first);
}
void launch_cond_silu(const float* y, const float* tsum, float inv_n, int dim, int nb, float* sy,
                      cudaStream_t s) {
  const int64_t n = (int64_t)nb * dim;
  launch_pdl(cond_silu_kernel, dim3(blocks_for(n)), dim3(256), s, y, tsum, inv_n, dim, n, sy);
}
void launch_adaln(const float* xs, int nb, int dim, const float* lnw, const float* lnb, int affine,
                  float eps, const float* mod, int64_t mod_stride, float* hh, cudaStream_t s) {
  launch_pdl(adaln_kernel, dim3(nb), dim3(kT), s, xs, dim, lnw, lnb, affine, eps, mod, mod_stride, hh);
}
void launch_gate_add(float* xs, const float* mod, int64_t mod_stride, int gate_off, const float* h,
                     int nb, int dim, cudaStream_t s) {
  const int64_t n = (int64_t)nb * dim;
  launch_pdl(gate_add_kernel, dim3(blocks_for(n)), dim3(256), s, xs, mod, mod_stride, gate_off, h,
             dim, n);
}
void launch_flow_update(float* x, const float* flow, int64_t n, int mode, float scale,
                        cudaStream_t s) {
  launch_pdl(flow_update_kernel, dim3(blocks_for(n)), dim3(256), s, x, flow, n, mode, scale);
}
void launch_prompt_embed(const float* table, const uint32_t* tokens, int nb, int n, int t, int d,
                         int bins, float* x, int* err, cudaStream_t s) {
  launch_pdl(prompt_embed_kernel, dim3(nb), dim3(256), s, table, tokens, n, t, d, bins, x, err);
}

}  // namespace svl
