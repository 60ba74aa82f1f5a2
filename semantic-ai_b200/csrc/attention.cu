// attention.cu — sliding-window decode attention over the per-stream KV ring.
//
// Replaces the reference's CPU kernel (nn/kernels/attention.rs:81-169) and its generic
// masked fallback on CUDA (nn/transformer.rs:346-364) for one new query per stream: query p
// sees keys p - min(p + 1, window) + 1 .. p (first_key of the reference's compacting cache
// is implied by the ring). The keys of a (stream, head) are split into `splits` chunks, one
// CTA each; the chunks of a (stream, head) form one thread-block cluster.
//
// Every key but the newest was written by an earlier step, and the in-projection of this
// step only writes the newest slot, so each CTA bulk-copies its chunk's keys and values into
// a shared-memory ring *before* griddepcontrol.wait, overlapping the previous kernel; after
// the wait it reads q and the newest row. Consumer warps score HD/16 lanes per key (16
// contiguous dims per lane) with an online softmax per lane group; lane groups and warps
// merge by max-rescaling, and the CTAs of a cluster merge through distributed shared
// memory. Every mbarrier wait is bounded (a wait that runs out sets *p.err); every CTA
// reaches both cluster barriers whatever happened, so no CTA waits on one that left.
#include "common.cuh"
#include "kernels.cuh"
#include "sm100.cuh"

namespace svl {
namespace {

constexpr int kConsumerWarps = 4;
constexpr int kThreads = (kConsumerWarps + 1) * 32;  // warp 4: producer
constexpr int kSlots = 3;
constexpr int kTileBytes = 16 * 1024;
constexpr int kMaxSplits = 8;  // portable cluster size

template <bool BF16>
__device__ __forceinline__ void unpack16(const uint8_t* src, float* out) {
  if (BF16) {
    const uint4 a = reinterpret_cast<const uint4*>(src)[0], b = reinterpret_cast<const uint4*>(src)[1];
    const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
    for (int i = 0; i < 8; i++) {
      out[2 * i] = bf16_lo(w[i]);
      out[2 * i + 1] = bf16_hi(w[i]);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const float4 v = reinterpret_cast<const float4*>(src)[i];
      out[4 * i] = v.x;
      out[4 * i + 1] = v.y;
      out[4 * i + 2] = v.z;
      out[4 * i + 3] = v.w;
    }
  }
}
template <bool BF16>
__device__ __forceinline__ void unpack16_global(const uint8_t* src, float* out) {
  if (BF16) {
    const uint4 a = __ldcg(reinterpret_cast<const uint4*>(src)), b = __ldcg(reinterpret_cast<const uint4*>(src) + 1);
    const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
    for (int i = 0; i < 8; i++) {
      out[2 * i] = bf16_lo(w[i]);
      out[2 * i + 1] = bf16_hi(w[i]);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const float4 v = __ldcg(reinterpret_cast<const float4*>(src) + i);
      out[4 * i] = v.x;
      out[4 * i + 1] = v.y;
      out[4 * i + 2] = v.z;
      out[4 * i + 3] = v.w;
    }
  }
}

// Merge (m2, l2, a2) into (m, l, a): the max-rescaled sum of two softmax partials.
__device__ __forceinline__ void merge(float& m, float& l, float* a, float m2, float l2, const float* a2) {
  const float mn = fmaxf(m, m2);
  if (mn == -INFINITY) return;
  const float c1 = exp_ref(m - mn), c2 = exp_ref(m2 - mn);
  l = l * c1 + l2 * c2;
#pragma unroll
  for (int i = 0; i < 16; i++) a[i] = a[i] * c1 + a2[i] * c2;
  m = mn;
}

template <int HD, bool BF16>
__global__ void __launch_bounds__(kThreads) attn_kernel(const AttnParams p) {
  constexpr int EL = BF16 ? 2 : 4;
  constexpr int ROW = HD * EL;             // bytes per key row
  constexpr int T = kTileBytes / ROW;      // keys per tile
  constexpr int LPK = HD / 16;             // lanes per key
  constexpr int KPW = 32 / LPK;            // keys per warp per pass
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kSlots;
  uint8_t* kbuf = smem + 128;
  uint8_t* vbuf = kbuf + kSlots * kTileBytes;
  __shared__ float sm_m[kConsumerWarps], sm_l[kConsumerWarps];
  __shared__ float sm_a[kConsumerWarps][HD];
  __shared__ float part_m, part_l;
  __shared__ float part_a[HD];
  __shared__ int failed;

  const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int pos = p.pos[b];  // advanced only by the last kernel of a step
  const int count = p.window > 0 ? min(pos + 1, p.window) : pos + 1;
  const int kps = (count + p.splits - 1) / p.splits;
  const int j0 = min(split * kps, count), j1 = min(j0 + kps, count);
  const int first_pos = pos - count + 1;
  const int ntiles = (j1 - j0 + T - 1) / T;
  const int kvh = h / (p.heads / p.kv_heads);
  const int64_t head_base = (b * p.ring_stream_stride + (int64_t)kvh * p.ring_cap * HD) * EL;
  const uint8_t* kg = static_cast<const uint8_t*>(p.k_ring) + head_base;
  const uint8_t* vg = static_cast<const uint8_t*>(p.v_ring) + head_base;
  auto slot_of_key = [&](int j) {
    const int q = first_pos + j;
    return p.window > 0 ? q % p.ring_cap : q;
  };

  if (tid == 0) {
    failed = 0;
    for (int s = 0; s < kSlots; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();

  // Tile i holds keys [j0 + i T, min(j0 + (i + 1) T, j1)); the newest key (count - 1) is read
  // from global memory after the dependency wait, so the copies stop before it.
  auto issue = [&](int i) {
    const int slot = i % kSlots;
    const int a = j0 + i * T, e = min(min(a + T, j1), count - 1);
    uint32_t bytes = 0;
    for (int j = a; j < e;) {
      const int s0 = slot_of_key(j);
      const int run = p.window > 0 ? min(e - j, p.ring_cap - s0) : e - j;  // the ring wraps once at most
      bytes += 2u * (uint32_t)run * ROW;
      j += run;
    }
    mbar_expect_tx(&full[slot], bytes);
    for (int j = a; j < e;) {
      const int s0 = slot_of_key(j);
      const int run = p.window > 0 ? min(e - j, p.ring_cap - s0) : e - j;
      const uint32_t nbytes = (uint32_t)run * ROW;
      bulk_g2s(kbuf + (size_t)slot * kTileBytes + (size_t)(j - a) * ROW, kg + (int64_t)s0 * ROW, nbytes, &full[slot]);
      bulk_g2s(vbuf + (size_t)slot * kTileBytes + (size_t)(j - a) * ROW, vg + (int64_t)s0 * ROW, nbytes, &full[slot]);
      j += run;
    }
  };
  int issued = 0;
  if (warp == kConsumerWarps && lane == 0)
    for (; issued < min(kSlots, ntiles); issued++) issue(issued);
  pdl_launch();
  pdl_wait();

  float m = -INFINITY, l = 0.f, acc[16];
#pragma unroll
  for (int i = 0; i < 16; i++) acc[i] = 0.f;
  const int kk = lane / LPK, sub = lane % LPK;

  if (warp == kConsumerWarps) {
    // ---- producer: refill each slot once all consumer warps released it.
    if (lane == 0) {
      for (; issued < ntiles; issued++) {
        const int slot = issued % kSlots;
        if (!mbar_wait(&empty[slot], (uint32_t)((issued / kSlots) - 1) & 1u)) {
          atomicExch(p.err, 1);
          failed = 1;
          break;
        }
        issue(issued);
      }
      // Every copy issued must land before the CTA exits (bounded).
      for (int i = max(0, issued - kSlots); i < issued; i++) mbar_wait(&full[i % kSlots], (uint32_t)(i / kSlots) & 1u);
    }
  } else {
    // ---- consumers.
    float q[16];
    {
      const float4* qp = reinterpret_cast<const float4*>(p.q + ((int64_t)b * p.heads + h) * HD + sub * 16);
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const float4 v = __ldcg(qp + i);
        q[4 * i] = v.x;
        q[4 * i + 1] = v.y;
        q[4 * i + 2] = v.z;
        q[4 * i + 3] = v.w;
      }
    }
    for (int i = 0; i < ntiles; i++) {
      const int slot = i % kSlots;
      if (failed || !mbar_wait(&full[slot], (uint32_t)(i / kSlots) & 1u)) {
        if (lane == 0) {
          atomicExch(p.err, 1);
          failed = 1;
        }
        break;
      }
      const int a = j0 + i * T, e = min(a + T, j1);
      for (int jb = a + warp * KPW; jb < e; jb += kConsumerWarps * KPW) {
        const int j = jb + kk;
        const bool valid = j < e;
        float kv[16], vv[16];
        if (valid && j == count - 1) {
          const int64_t off = (int64_t)slot_of_key(j) * ROW + sub * 16 * EL;
          unpack16_global<BF16>(kg + off, kv);
          unpack16_global<BF16>(vg + off, vv);
        } else {
          const size_t off = (size_t)slot * kTileBytes + (size_t)((valid ? j : a) - a) * ROW + sub * 16 * EL;
          unpack16<BF16>(kbuf + off, kv);
          unpack16<BF16>(vbuf + off, vv);
        }
        float d = 0.f;
#pragma unroll
        for (int t = 0; t < 16; t++) d = fmaf(q[t], kv[t], d);
#pragma unroll
        for (int o = LPK / 2; o; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
        if (valid) {
          const float s = p.scale * d;  // scale * dot(q, k), as the reference
          const float mn = fmaxf(m, s);
          const float c = exp_ref(m - mn), ev = exp_ref(s - mn);
          l = l * c + ev;
#pragma unroll
          for (int t = 0; t < 16; t++) acc[t] = acc[t] * c + ev * vv[t];
          m = mn;
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
    }
    // Merge the KPW key groups of the warp (lanes sub, sub + LPK, ...).
#pragma unroll
    for (int o = LPK; o < 32; o <<= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
      const float l2 = __shfl_xor_sync(0xffffffffu, l, o);
      float a2[16];
#pragma unroll
      for (int t = 0; t < 16; t++) a2[t] = __shfl_xor_sync(0xffffffffu, acc[t], o);
      merge(m, l, acc, m2, l2, a2);
    }
    if (kk == 0) {
#pragma unroll
      for (int t = 0; t < 16; t++) sm_a[warp][sub * 16 + t] = acc[t];
      if (sub == 0) {
        sm_m[warp] = m;
        sm_l[warp] = l;
      }
    }
  }
  __syncthreads();
  // This CTA's partial: merge the warps; thread t < HD owns output dim t.
  if (tid < HD) {
    float M = -INFINITY;
    for (int w = 0; w < kConsumerWarps; w++) M = fmaxf(M, sm_m[w]);
    float L = 0.f, A = 0.f;
    if (M != -INFINITY)
      for (int w = 0; w < kConsumerWarps; w++) {
        if (sm_m[w] == -INFINITY) continue;
        const float c = exp_ref(sm_m[w] - M);
        L = L + sm_l[w] * c;
        A = A + sm_a[w][tid] * c;
      }
    part_a[tid] = A;
    if (tid == 0) {
      part_m = M;
      part_l = L;
    }
  }
  const int64_t bh = (int64_t)b * p.heads + h;
  if (p.splits == 1) {
    __syncthreads();
    if (tid < HD) p.out[bh * HD + tid] = part_l > 0.f ? part_a[tid] / part_l : 0.f;
    return;
  }
  // The chunks of this (stream, head) merge in the cluster's first CTA, in chunk order.
  cluster_sync();
  if (split == 0 && tid < HD) {
    float MM = -INFINITY;
    for (int s = 0; s < p.splits; s++) MM = fmaxf(MM, dsmem_ld(dsmem_addr(&part_m, s)));
    float LL = 0.f, AA = 0.f;
    for (int s = 0; s < p.splits; s++) {
      const float ms = dsmem_ld(dsmem_addr(&part_m, s));
      if (ms == -INFINITY) continue;
      const float c = exp_ref(ms - MM);
      LL = LL + dsmem_ld(dsmem_addr(&part_l, s)) * c;
      AA = AA + dsmem_ld(dsmem_addr(&part_a[tid], s)) * c;
    }
    p.out[bh * HD + tid] = LL > 0.f ? AA / LL : 0.f;
  }
  // Keep every CTA's shared memory alive until the first CTA has read it.
  cluster_sync();
}

template <int HD, bool BF16>
void launch_t(const AttnParams& p, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.splits, p.heads, p.nb);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = 128 + 2 * kSlots * kTileBytes;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = p.splits;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  cudaLaunchKernelEx(&cfg, attn_kernel<HD, BF16>, p);
}

template <int HD, bool BF16>
void set_attr() {
  cudaFuncSetAttribute(attn_kernel<HD, BF16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       128 + 2 * kSlots * kTileBytes);
}

}  // namespace

int attention_max_splits() { return kMaxSplits; }

void attention_init_device() {
  set_attr<64, false>();
  set_attr<64, true>();
  set_attr<128, false>();
  set_attr<128, true>();
}

void launch_attention_decode(const AttnParams& p, cudaStream_t s) {
  switch (p.head_dim * 2 + p.kv_bf16) {
    case 128: launch_t<64, false>(p, s); break;
    case 129: launch_t<64, true>(p, s); break;
    case 256: launch_t<128, false>(p, s); break;
    case 257: launch_t<128, true>(p, s); break;
    default: break;  // rejected at model creation
  }
}

}  // namespace svl
