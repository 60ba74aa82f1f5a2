// misc.cu — embedding sum, position advance and weight packing.
#include "common.cuh"
#include "gemv_common.cuh"
#include "kernels.cuh"
#include "sm100.cuh"

namespace svl {
namespace {

// LanguageModel::step's input (stt/model.rs:246-250): the text embedding row, then each of
// the n_q audio embedding rows added in codebook order, in f32 -- the reference's order and
// rounding, so the sum is bit-identical to it. One CTA per stream: the token ids are staged
// first (validated; an id past its table sets the error flag and reads row 0), then every
// thread sums its columns over the 1 + n_q rows.
template <bool BF16>
__global__ void __launch_bounds__(64) embed_kernel(const EmbedParams p) {
  __shared__ uint32_t toks[kMaxCodebooks + 1];
  const int b = blockIdx.x, t = threadIdx.x;
  // x is still read by the previous kernel (programmatic dependent launch).
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  for (int i = t; i <= p.n_q; i += 64) {
    uint32_t v = i == 0 ? p.text_tok[b] : p.audio_tok[b * p.n_q + i - 1];
    const uint32_t lim = i == 0 ? (uint32_t)p.text_card : (uint32_t)p.card;
    if (v > lim) {
      atomicExch(p.error_flag, 1);
      v = 0;
    }
    toks[i] = v;
  }
  __syncthreads();
  auto row = [&](const void* table, int64_t r, int c4) -> float4 {
    if (BF16) {
      const uint2 v = reinterpret_cast<const uint2*>(
          reinterpret_cast<const __nv_bfloat16*>(table) + r * p.d)[c4];
      return make_float4(bf16_lo(v.x), bf16_hi(v.x), bf16_lo(v.y), bf16_hi(v.y));
    }
    return reinterpret_cast<const float4*>(reinterpret_cast<const float*>(table) + r * p.d)[c4];
  };
  float* x = p.x + (int64_t)b * p.d;
  // Column block blockIdx.y of 64 float4; the rows' loads go out 16 at a time, the adds stay
  // in the reference's order.
  const int c4 = blockIdx.y * 64 + t;
  if (c4 >= p.d / 4) return;
  float4 acc = row(p.text_table, toks[0], c4);
  for (int c0 = 0; c0 < p.n_q; c0 += 16) {
    float4 e[16];
#pragma unroll
    for (int j = 0; j < 16; j++)
      e[j] = c0 + j < p.n_q ? row(p.audio_tables, (int64_t)(c0 + j) * (p.card + 1) + toks[c0 + j + 1], c4)
                            : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int j = 0; j < 16; j++) {
      if (c0 + j >= p.n_q) break;
      acc.x = acc.x + e[j].x;
      acc.y = acc.y + e[j].y;
      acc.z = acc.z + e[j].z;
      acc.w = acc.w + e[j].w;
    }
  }
  reinterpret_cast<float4*>(x)[c4] = acc;
}

__global__ void advance_kernel(int* pos, int nb) {
  int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < nb) pos[b] += 1;
}

// One warp per (packed row, 32-column block).
__global__ void pack_kernel(const float* src, uint8_t* dst, int64_t row_stride, int n, int k,
                            int wtype, int interleave_half) {
  const int lane = threadIdx.x & 31;
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int nblk = k / QBLK;
  if (gw >= (int64_t)n * nblk) return;
  const int r = (int)(gw / nblk), blk = (int)(gw % nblk);
  int sr = r;
  if (interleave_half > 0) sr = (r & 1) ? interleave_half + (r >> 1) : (r >> 1);
  const float x = src[(int64_t)sr * k + blk * QBLK + lane];
  uint8_t* row = dst + (int64_t)r * row_stride;
  if (wtype == W_F32) {
    reinterpret_cast<float*>(row)[blk * QBLK + lane] = x;
  } else if (wtype == W_BF16) {
    reinterpret_cast<__nv_bfloat16*>(row)[blk * QBLK + lane] = __float2bfloat16_rn(x);
  } else if (wtype == W_Q8) {
    // Q8_0 (ggml; candle QTensor::quantize, nn/mod.rs:81-83): d = amax / 127 stored f16,
    // q = round(x * (1 / d)).
    // Stored in super-blocks (gemv_common.cuh): element lane of block blk sits in slot lane / 4.
    float amax = warp_max(fabsf(x));
    float d = amax / 127.0f;
    float id = d != 0.0f ? 1.0f / d : 0.0f;
    uint8_t* sb = row + (int64_t)(blk / kSbBlocks) * kQ8SbBytes;
    const int bj = blk % kSbBlocks;
    reinterpret_cast<int8_t*>(sb)[(bj >> 2) * 128 + 16 * (lane >> 2) + 4 * (bj & 3) + (lane & 3)] =
        (int8_t)(int)roundf(x * id);
    if (lane == 0) reinterpret_cast<__half*>(sb + 256)[bj] = __float2half_rn(d);
  } else {
    // Q4_1 (ggml): d = (max - min) / 15, m = min, q = min(15, trunc((x - min) / d + 0.5)),
    // byte j holds q[j] (low nibble) and q[j + 16] (high nibble).
    float mn = x, mx = x;
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    float d = (mx - mn) / 15.0f;
    float id = d != 0.0f ? 1.0f / d : 0.0f;
    int q = (int)((x - mn) * id + 0.5f);
    q = q > 15 ? 15 : q;
    int hi = __shfl_down_sync(0xffffffffu, q, 16);
    // Super-block layout (gemv_common.cuh): byte i of block j sits in 4-byte group i / 4.
    uint8_t* sb = row + (int64_t)(blk / kSbBlocks) * kQ4SbBytes;
    const int bj = blk % kSbBlocks;
    if (lane < 16) sb[32 * (lane >> 2) + 4 * bj + (lane & 3)] = (uint8_t)(q | (hi << 4));
    if (lane == 0)
      reinterpret_cast<__half2*>(sb + 128)[bj] = __halves2half2(__float2half_rn(d), __float2half_rn(mn));
  }
}

// The bf16 image of a packed Q8_0 / Q4_1 matrix (the values the quantised dot products use:
// q * d, or d * q + m), one warp per (row, 32-element block); rows of k bf16, dst_stride
// bytes apart.
__global__ void dequant_bf16_kernel(const uint8_t* src, int64_t row_stride, int n, int k, int wtype,
                                    uint16_t* dst, int64_t dst_stride, int f16) {
  const int lane = threadIdx.x & 31;
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int nblk = k / QBLK;
  if (gw >= (int64_t)n * nblk) return;
  const int r = (int)(gw / nblk), blk = (int)(gw % nblk);
  const uint8_t* row = src + (int64_t)r * row_stride;
  float x;
  const int bj = blk % kSbBlocks;
  if (wtype == W_Q8) {
    const uint8_t* sb = row + (int64_t)(blk / kSbBlocks) * kQ8SbBytes;
    const float d = __half2float(reinterpret_cast<const __half*>(sb + 256)[bj]);
    x = (float)reinterpret_cast<const int8_t*>(sb)[(bj >> 2) * 128 + 16 * (lane >> 2) + 4 * (bj & 3) + (lane & 3)] * d;
  } else {
    const uint8_t* sb = row + (int64_t)(blk / kSbBlocks) * kQ4SbBytes;
    const int i = lane & 15;
    const uint8_t b = sb[32 * (i >> 2) + 4 * bj + (i & 3)];
    const int q = lane < 16 ? (b & 15) : (b >> 4);
    const float2 dm = __half22float2(reinterpret_cast<const __half2*>(sb + 128)[bj]);
    x = dm.x * (float)q + dm.y;
  }
  uint16_t* o = reinterpret_cast<uint16_t*>(reinterpret_cast<uint8_t*>(dst) + (int64_t)r * dst_stride);
  if (f16) {
    const __half h = __float2half_rn(x);
    o[blk * QBLK + lane] = *reinterpret_cast<const uint16_t*>(&h);
  } else {
    const __nv_bfloat16 h = __float2bfloat16_rn(x);
    o[blk * QBLK + lane] = *reinterpret_cast<const uint16_t*>(&h);
  }
}

__global__ void f32_to_bf16_kernel(const float* src, __nv_bfloat16* dst, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    dst[i] = __float2bfloat16_rn(src[i]);
}

__global__ void round_bf16_kernel(float* p, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    p[i] = round_bf16(p[i]);
}

}  // namespace

void launch_embed(const EmbedParams& p, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.nb, (p.d / 4 + 63) / 64);
  cfg.blockDim = dim3(64);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (p.tables_bf16)
    cudaLaunchKernelEx(&cfg, embed_kernel<true>, p);
  else
    cudaLaunchKernelEx(&cfg, embed_kernel<false>, p);
}

__global__ void rope_table_kernel(const int* pos, int nb, const float* inv_freq, int half, float2* cs) {
  pdl_launch();
  pdl_wait();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)nb * half) return;
  const int b = (int)(i / half), f = (int)(i % half);
  float sn, c;
  sincosf((float)pos[b] * inv_freq[f], &sn, &c);
  cs[i] = make_float2(c, sn);
}

void launch_rope_table(const int* pos, int nb, const float* inv_freq, int half, float2* cs,
                       cudaStream_t s) {
  const int64_t n = (int64_t)nb * half;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((n + 255) / 256));
  cfg.blockDim = dim3(256);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, rope_table_kernel, pos, nb, inv_freq, half, cs);
}

void launch_advance_positions(int* pos, int nb, cudaStream_t s) {
  advance_kernel<<<(nb + 255) / 256, 256, 0, s>>>(pos, nb);
}

void launch_dequant_bf16(const uint8_t* src, int64_t row_stride, int n, int k, int wtype, void* dst,
                         int64_t dst_stride, cudaStream_t s, int f16) {
  const int64_t warps = (int64_t)n * (k / QBLK);
  dequant_bf16_kernel<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, s>>>(
      src, row_stride, n, k, wtype, static_cast<uint16_t*>(dst), dst_stride, f16);
}

int64_t packed_row_stride(int wtype, int k) {
  auto pad16 = [](int64_t x) { return (x + 15) / 16 * 16; };
  switch (wtype) {
    case W_F32: return pad16((int64_t)k * 4);
    case W_BF16: return pad16((int64_t)k * 2);
    case W_Q8: return (int64_t)super_blocks(k) * kQ8SbBytes;
    default: return (int64_t)super_blocks(k) * kQ4SbBytes;
  }
}

void launch_pack_linear(const float* src, uint8_t* dst, int64_t row_stride, int n, int k,
                        int wtype, int interleave_half, cudaStream_t s) {
  int64_t warps = (int64_t)n * (k / QBLK);
  int64_t blocks = (warps * 32 + 255) / 256;
  pack_kernel<<<(unsigned)blocks, 256, 0, s>>>(src, dst, row_stride, n, k, wtype, interleave_half);
}

void launch_f32_to_bf16(const float* src, void* dst, int64_t n, cudaStream_t s) {
  f32_to_bf16_kernel<<<1184, 256, 0, s>>>(src, reinterpret_cast<__nv_bfloat16*>(dst), n);
}

void launch_round_bf16_inplace(float* p, int64_t n, cudaStream_t s) {
  round_bf16_kernel<<<1184, 256, 0, s>>>(p, n);
}

}  // namespace svl

namespace svl {
namespace {

// softmax_last_dim(head logits)[0] per (stream, extra head) (stt/model.rs:259-271).
__global__ void extra_p0_kernel(const float* logits, int nb, int heads, int dim, float* out) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nb * heads) return;
  const float* x = logits + (int64_t)i * dim;
  float mx = x[0];
  for (int j = 1; j < dim; j++) mx = fmaxf(mx, x[j]);
  float sum = 0.f, e0 = 0.f;
  for (int j = 0; j < dim; j++) {
    float e = expf(x[j] - mx);
    if (j == 0) e0 = e;
    sum = sum + e;
  }
  out[i] = e0 / sum;
}

}  // namespace

void launch_extra_heads(const float* logits, int nb, int heads, int dim, float* out,
                        cudaStream_t st) {
  int n = nb * heads;
  extra_p0_kernel<<<(n + 127) / 128, 128, 0, st>>>(logits, nb, heads, dim, out);
}

}  // namespace svl
