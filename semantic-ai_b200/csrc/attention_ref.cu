// attention_ref.cu — decode attention in the reference CPU path's order (reference-order
// states only; the fast kernels are in attention.cu).
//
// The reference's CPU attention (nn/kernels/attention.rs:142-169, `attend`) for one query:
//   w_j = scale * dot(q, k_j)                 dot: kernels::dot, 16 FMA lanes + pairwise tree
//   m   = max_j w_j
//   e_j = exp(w_j - m), sum = e_0 + e_1 + ...  in key order, the reference's own exp
//   out = 0; out[i] = fma(e_j / sum, v_j[i], out[i])   for j in key order
// with keys oldest first. One CTA per (head, stream) runs exactly those operations: the dots
// in parallel (half a warp per key, lane i = dot lane i, the tree as xor-shuffles), the key-
// order sum on one thread, and the output chain on thread i for dimension i. A full STT-1b
// window costs a few microseconds per layer; it exists so that a reference-order state is the
// reference's arithmetic bit for bit.
#include "common.cuh"
#include "kernels.cuh"

namespace svl {
namespace {

constexpr int kRefThreads = 256;

template <bool BF16>
__device__ __forceinline__ float kv_at(const void* ring, int64_t i) {
  if (BF16) return __uint_as_float((uint32_t)__ldcg(reinterpret_cast<const unsigned short*>(ring) + i) << 16);
  return __ldcg(reinterpret_cast<const float*>(ring) + i);
}

template <int HD, bool BF16>
__global__ void __launch_bounds__(kRefThreads) attn_ref_kernel(const AttnParams p) {
  extern __shared__ float wj[];  // [count] scores, then exp values
  __shared__ float qs[HD];
  __shared__ float red[kRefThreads / 32];
  __shared__ float sum_sh, max_sh;
  const int h = blockIdx.x, b = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int pos = p.pos[b];
  const int count = p.window > 0 ? min(pos + 1, p.window) : pos + 1;
  const int first_pos = pos - count + 1;
  const int kvh = h / (p.heads / p.kv_heads);
  const int64_t head_base = b * p.ring_stream_stride + (int64_t)kvh * p.ring_cap * HD;
  auto slot_of = [&](int j) { return p.window > 0 ? (first_pos + j) % p.ring_cap : first_pos + j; };
  const float* q = p.q + ((int64_t)b * p.heads + h) * HD;
  for (int i = tid; i < HD; i += kRefThreads) qs[i] = __ldcg(q + i);
  __syncthreads();

  // Scores: half-warp per key; lane i holds dot lane i (elements i, i + 16, ...).
  const int hw = lane >> 4, i16 = lane & 15;
  for (int j0 = 2 * warp; j0 < count; j0 += 2 * (kRefThreads / 32)) {
    const int j = j0 + hw;
    float acc = 0.f;
    if (j < count) {
      const int64_t row = head_base + (int64_t)slot_of(j) * HD;
#pragma unroll
      for (int c = 0; c < HD / 16; c++) acc = fmaf(qs[16 * c + i16], kv_at<BF16>(p.k_ring, row + 16 * c + i16), acc);
    }
    // Pairwise tree: lane i += lane i + 8, + 4, + 2, + 1 (within each half-warp).
    acc = acc + __shfl_xor_sync(0xffffffffu, acc, 8);
    acc = acc + __shfl_xor_sync(0xffffffffu, acc, 4);
    acc = acc + __shfl_xor_sync(0xffffffffu, acc, 2);
    acc = acc + __shfl_xor_sync(0xffffffffu, acc, 1);
    if (i16 == 0 && j < count) wj[j] = p.scale * (acc + 0.0f);
  }
  __syncthreads();

  // Max (order-free).
  float m = -__int_as_float(0x7f800000);
  for (int j = tid; j < count; j += kRefThreads) m = fmaxf(m, wj[j]);
  m = warp_max(m);
  if (lane == 0) red[warp] = m;
  __syncthreads();
  if (tid == 0) {
    float mm = red[0];
    for (int w = 1; w < kRefThreads / 32; w++) mm = fmaxf(mm, red[w]);
    max_sh = mm;
  }
  __syncthreads();
  const float mx = max_sh;
  for (int j = tid; j < count; j += kRefThreads) wj[j] = exp_ref(wj[j] - mx);
  __syncthreads();

  // The key-order sum, then each key's probability e_j / sum (in place).
  if (tid == 0) {
    float s = 0.f;
    for (int j = 0; j < count; j++) s = s + wj[j];
    sum_sh = s;
  }
  __syncthreads();
  const float sum = sum_sh;
  for (int j = tid; j < count; j += kRefThreads) wj[j] = wj[j] / sum;
  __syncthreads();

  // Output dimension i: the FMA chain over keys in order.
  if (tid < HD) {
    float o = 0.f;
    int j = 0;
    for (; j + 8 <= count; j += 8) {
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; u++) v[u] = kv_at<BF16>(p.v_ring, head_base + (int64_t)slot_of(j + u) * HD + tid);
#pragma unroll
      for (int u = 0; u < 8; u++) o = fmaf(wj[j + u], v[u], o);
    }
    for (; j < count; j++) o = fmaf(wj[j], kv_at<BF16>(p.v_ring, head_base + (int64_t)slot_of(j) * HD + tid), o);
    p.out[((int64_t)b * p.heads + h) * HD + tid] = o;
  }
}

constexpr int kRefMaxSmem = 200 * 1024;  // the scores of up to 51,200 keys

template <int HD, bool BF16>
void launch_t(const AttnParams& p, cudaStream_t s) {
  attn_ref_kernel<HD, BF16><<<dim3(p.heads, p.nb), kRefThreads, (size_t)p.ring_cap * 4, s>>>(p);
}

}  // namespace

bool attention_ref_supported(int head_dim, int ring_cap) {
  return (head_dim == 64 || head_dim == 128) && (int64_t)ring_cap * 4 <= kRefMaxSmem;
}

void attention_ref_init_device() {
  cudaFuncSetAttribute(attn_ref_kernel<64, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kRefMaxSmem);
  cudaFuncSetAttribute(attn_ref_kernel<64, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kRefMaxSmem);
  cudaFuncSetAttribute(attn_ref_kernel<128, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kRefMaxSmem);
  cudaFuncSetAttribute(attn_ref_kernel<128, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kRefMaxSmem);
}

void launch_attention_ref(const AttnParams& p, cudaStream_t s) {
  if (p.head_dim == 64) {
    if (p.kv_bf16) launch_t<64, true>(p, s); else launch_t<64, false>(p, s);
  } else {
    if (p.kv_bf16) launch_t<128, true>(p, s); else launch_t<128, false>(p, s);
  }
}

}  // namespace svl
