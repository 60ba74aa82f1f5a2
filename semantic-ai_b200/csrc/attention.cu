// attention.cu — sliding-window decode attention over the per-stream KV ring.
//
// Replaces the reference's CPU kernel (nn/kernels/attention.rs:81-169) and its generic
// masked fallback on CUDA (nn/transformer.rs:346-364) for one new query per stream: query
// p sees keys p - min(p + 1, window) + 1 .. p. The keys of a (stream, head) are split into
// `splits` chunks, one CTA each, so batch 1 fills the GPU. Each warp handles KPW keys at a
// time, HD/16 lanes per key and 16 contiguous dims per lane (coalesced 16-byte loads of
// whole key rows), with an online softmax per lane group; the warps, then the chunks, are
// merged by max-rescaling. The last CTA of a (stream, head) to finish merges the chunks.
#include "common.cuh"
#include "kernels.cuh"

namespace svl {
namespace {

constexpr int kAttnWarps = 4;
constexpr int kMaxSplits = kAttnWarps * 32;

template <bool BF16>
__device__ __forceinline__ void load16(const void* base, int64_t off, float* out) {
  if (BF16) {
    const uint4* p = reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(base) + off);
    uint4 a = __ldg(p), b = __ldg(p + 1);
    uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
    for (int i = 0; i < 8; i++) {
      out[2 * i] = bf16_lo(w[i]);
      out[2 * i + 1] = bf16_hi(w[i]);
    }
  } else {
    const float4* p = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(base) + off);
#pragma unroll
    for (int i = 0; i < 4; i++) {
      float4 v = __ldg(p + i);
      out[4 * i] = v.x;
      out[4 * i + 1] = v.y;
      out[4 * i + 2] = v.z;
      out[4 * i + 3] = v.w;
    }
  }
}

// Merge (m2, l2, a2) into (m, l, a): the max-rescaled sum of two softmax partials.
__device__ __forceinline__ void merge(float& m, float& l, float* a, float m2, float l2,
                                      const float* a2) {
  float mn = fmaxf(m, m2);
  if (mn == -INFINITY) return;
  float c1 = exp_ref(m - mn), c2 = exp_ref(m2 - mn);
  l = l * c1 + l2 * c2;
#pragma unroll
  for (int i = 0; i < 16; i++) a[i] = a[i] * c1 + a2[i] * c2;
  m = mn;
}

template <int HD, bool BF16>
__global__ void __launch_bounds__(kAttnWarps * 32) attn_decode_kernel(const AttnParams p) {
  constexpr int LPK = HD / 16;   // lanes per key
  constexpr int KPW = 32 / LPK;  // keys per warp per iteration
  __shared__ float sm_m[kAttnWarps], sm_l[kAttnWarps];
  __shared__ float sm_a[kAttnWarps][HD];
  __shared__ bool last;

  const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // q and the newest key come from the previous kernel (programmatic dependent launch).
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int kk = lane / LPK, sub = lane % LPK;
  const int pos = p.pos[b];
  const int count = p.window > 0 ? min(pos + 1, p.window) : pos + 1;
  const int kps = (count + p.splits - 1) / p.splits;
  const int j0 = split * kps, j1 = min(j0 + kps, count);
  const int first_pos = pos - count + 1;
  const int kvh = h / (p.heads / p.kv_heads);
  const int64_t head_base = b * p.ring_stream_stride + (int64_t)kvh * p.ring_cap * HD;

  float q[16];
  {
    const float4* qp = reinterpret_cast<const float4*>(p.q + ((int64_t)b * p.heads + h) * HD + sub * 16);
#pragma unroll
    for (int i = 0; i < 4; i++) {
      float4 v = qp[i];
      q[4 * i] = v.x;
      q[4 * i + 1] = v.y;
      q[4 * i + 2] = v.z;
      q[4 * i + 3] = v.w;
    }
  }
  float m = -INFINITY, l = 0.f, acc[16];
#pragma unroll
  for (int i = 0; i < 16; i++) acc[i] = 0.f;

  for (int jb = j0 + warp * KPW; jb < j1; jb += kAttnWarps * KPW) {
    const int j = jb + kk;
    const bool valid = j < j1;
    const int ppos = first_pos + (valid ? j : j0);
    const int slot = p.window > 0 ? ppos % p.ring_cap : ppos;
    const int64_t off = head_base + (int64_t)slot * HD + sub * 16;
    float kv[16];
    load16<BF16>(p.k_ring, off, kv);
    float d = 0.f;
#pragma unroll
    for (int i = 0; i < 16; i++) d = fmaf(q[i], kv[i], d);
#pragma unroll
    for (int o = LPK / 2; o; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
    load16<BF16>(p.v_ring, off, kv);
    if (valid) {
      const float s = p.scale * d;
      const float mn = fmaxf(m, s);
      const float c = exp_ref(m - mn), e = exp_ref(s - mn);
      l = l * c + e;
#pragma unroll
      for (int i = 0; i < 16; i++) acc[i] = acc[i] * c + e * kv[i];
      m = mn;
    }
  }
  // Merge the KPW key groups of the warp (lanes sub, sub + LPK, ...).
#pragma unroll
  for (int o = LPK; o < 32; o <<= 1) {
    float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    float l2 = __shfl_xor_sync(0xffffffffu, l, o);
    float a2[16];
#pragma unroll
    for (int i = 0; i < 16; i++) a2[i] = __shfl_xor_sync(0xffffffffu, acc[i], o);
    merge(m, l, acc, m2, l2, a2);
  }
  if (kk == 0) {
#pragma unroll
    for (int i = 0; i < 16; i++) sm_a[warp][sub * 16 + i] = acc[i];
    if (sub == 0) {
      sm_m[warp] = m;
      sm_l[warp] = l;
    }
  }
  __syncthreads();
  // Merge the warps; thread t < HD owns output dim t.
  const int t = threadIdx.x;
  float M = -INFINITY;
  for (int w = 0; w < kAttnWarps; w++) M = fmaxf(M, sm_m[w]);
  float L = 0.f, A = 0.f;
  if (M != -INFINITY)
    for (int w = 0; w < kAttnWarps; w++) {
      if (sm_m[w] == -INFINITY) continue;
      float c = exp_ref(sm_m[w] - M);
      L = L + sm_l[w] * c;
      if (t < HD) A = A + sm_a[w][t] * c;
    }
  const int64_t bh = (int64_t)b * p.heads + h;
  __shared__ float so[HD];
  if (p.splits == 1) {
    if (t < HD) so[t] = L > 0.f ? A / L : 0.f;
  } else {
    float* part = p.part + (bh * p.splits + split) * (HD + 2);
    if (t < HD) part[2 + t] = A;
    if (t == 0) {
      part[0] = M;
      part[1] = L;
    }
    __threadfence();
    __syncthreads();
    if (t == 0) last = atomicAdd(p.tickets + bh, 1u) == (unsigned)p.splits - 1;
    __syncthreads();
    if (!last) return;
    __threadfence();
    // The last CTA of this (stream, head) merges the chunks: scale factors in shared memory
    // first, then every output dim sums its column with all loads in flight.
    const float* parts = p.part + bh * p.splits * (HD + 2);
    __shared__ float sc[kMaxSplits];
    __shared__ float sl[kMaxSplits];
    __shared__ float s_ll;
    if (t < p.splits) {
      sc[t] = __ldcg(parts + t * (HD + 2));
      sl[t] = __ldcg(parts + t * (HD + 2) + 1);
    }
    __syncthreads();
    if (t == 0) {
      float MM = -INFINITY;
      for (int s = 0; s < p.splits; s++) MM = fmaxf(MM, sc[s]);
      float LL = 0.f;
      for (int s = 0; s < p.splits; s++) {
        const float c = sc[s] == -INFINITY ? 0.f : exp_ref(sc[s] - MM);
        sc[s] = c;
        LL = LL + sl[s] * c;
      }
      s_ll = LL;
    }
    __syncthreads();
    if (t < HD) {
      float AA = 0.f;
#pragma unroll 4
      for (int s = 0; s < p.splits; s++) AA = AA + __ldcg(parts + s * (HD + 2) + 2 + t) * sc[s];
      so[t] = AA / s_ll;
    }
    if (t == 0) p.tickets[bh] = 0u;
  }
  __syncthreads();
  if (t < HD) p.out[bh * HD + t] = so[t];
}

template <int HD>
void launch_hd(const AttnParams& p, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.splits, p.heads, p.nb);
  cfg.blockDim = dim3(kAttnWarps * 32);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (p.kv_bf16)
    cudaLaunchKernelEx(&cfg, attn_decode_kernel<HD, true>, p);
  else
    cudaLaunchKernelEx(&cfg, attn_decode_kernel<HD, false>, p);
}

}  // namespace

int attention_max_splits() { return kMaxSplits; }

void launch_attention_decode(const AttnParams& p, cudaStream_t s) {
  switch (p.head_dim) {
    case 64: launch_hd<64>(p, s); break;
    case 128: launch_hd<128>(p, s); break;
    default: break;  // rejected at model creation
  }
}

}  // namespace svl
