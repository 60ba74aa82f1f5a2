// attention.cu — sliding-window decode attention over the per-stream KV ring.
//
// Replaces the reference's CPU kernel (nn/kernels/attention.rs:81-169) and its generic
// masked fallback on CUDA (nn/transformer.rs:346-364) for one new query per stream: query p
// sees keys p - min(p + 1, window) + 1 .. p (first_key of the reference's compacting cache
// is implied by the ring). Three kernels, by the number of (stream, head) units:
//  - attn_flat_kernel (few units, short windows: batch 1 of the STT models): flat chunks of
//    at most 48 keys, two CTAs per SM, keys loaded into registers, merged by the last CTA;
//  - attn_kernel (few units, longer windows): the keys of a (stream, head) are split into
//    `splits` chunks, one CTA each; the chunks of a (stream, head) form one thread-block
//    cluster (described below);
//  - attn_warp_kernel + attn_merge_kernel (148 units or more): pieces of keys per warp.
//
// Every key but the newest was written by an earlier step, and the in-projection of this
// step only writes the newest slot, so each CTA bulk-copies its chunk's keys and values into
// a shared-memory ring *before* griddepcontrol.wait, overlapping the previous kernel; after
// the wait it reads q and the newest row. Consumer warps score HD/16 lanes per key (16
// contiguous dims per lane) with an online softmax whose running max is shared by the warp's
// lane groups (they merge by plain sums); warps merge by max-rescaling, and the CTAs of a
// cluster merge through distributed shared memory: each pushes its partial into the first CTA's
// shared memory, and one cluster barrier publishes them. Every mbarrier wait is bounded (a wait
// that runs out sets *p.err to 4); every CTA reaches the cluster barrier whatever happened, so
// no CTA waits on one that left.
#include <cuda.h>

#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"
#include "sm100.cuh"

namespace svl {
namespace {

constexpr int kConsumerWarps = 8;
constexpr int kThreads = (kConsumerWarps + 1) * 32;  // warp kConsumerWarps: producer
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
  // The cluster's first CTA collects every chunk's partial here (written by the chunks'
  // CTAs through distributed shared memory).
  __shared__ float gm[kMaxSplits], gl[kMaxSplits];
  __shared__ float ga[kMaxSplits][HD];
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
  if (warp == kConsumerWarps && lane == 0) {
    for (; issued < min(kSlots, ntiles); issued++) issue(issued);
    // Then this CTA's share of the later kernels' data into L2.
    const int cta = split + p.splits * (h + p.heads * b), ctas = p.splits * p.heads * p.nb;
    for (int i = 0; i < kMaxPrefetch; i++) prefetch_l2_share(p.pf[i].p, p.pf[i].bytes, cta, ctas);
  }
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
          atomicExch(p.err, 4);
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
          atomicExch(p.err, 4);
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
        // One running max per warp: the pass's KPW scores raise it (a warp-uniform branch, so
        // the accumulators are rescaled only when it rises), then each lane group adds its key.
        const float s = valid ? p.scale * d : -INFINITY;  // scale * dot(q, k), as the reference
        float mx = s;
#pragma unroll
        for (int o = LPK; o < 32; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if (mx > m) {
          const float c = exp_ref(m - mx);  // 0 while nothing was added
          l = l * c;
#pragma unroll
          for (int t = 0; t < 16; t++) acc[t] = acc[t] * c;
          m = mx;
        }
        if (valid) {
          const float ev = exp_ref(s - m);
          l = l + ev;
#pragma unroll
          for (int t = 0; t < 16; t++) acc[t] = acc[t] + ev * vv[t];
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
    }
    // The KPW key groups of the warp (lanes sub, sub + LPK, ...) share the running max: their
    // sums add up.
#pragma unroll
    for (int o = LPK; o < 32; o <<= 1) {
      l += __shfl_xor_sync(0xffffffffu, l, o);
#pragma unroll
      for (int t = 0; t < 16; t++) acc[t] += __shfl_xor_sync(0xffffffffu, acc[t], o);
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
    if (p.splits > 1) {
      // Push the partial into the first CTA's collection (stores do not wait on the remote
      // CTA; the cluster barrier below publishes them).
      dsmem_st(dsmem_addr(&ga[split][tid], 0), A);
      if (tid == 0) {
        dsmem_st(dsmem_addr(&gm[split], 0), M);
        dsmem_st(dsmem_addr(&gl[split], 0), L);
      }
    }
  }
  const int64_t bh = (int64_t)b * p.heads + h;
  if (p.splits == 1) {
    __syncthreads();
    if (tid < HD) p.out[bh * HD + tid] = part_l > 0.f ? part_a[tid] / part_l : 0.f;
    return;
  }
  // The chunks of this (stream, head) merge in the cluster's first CTA, in chunk order. After
  // the barrier no CTA touches another's shared memory, so the others may leave.
  cluster_sync();
  if (split == 0 && tid < HD) {
    float MM = -INFINITY;
    for (int s = 0; s < p.splits; s++) MM = fmaxf(MM, gm[s]);
    float LL = 0.f, AA = 0.f;
    for (int s = 0; s < p.splits; s++) {
      const float ms = gm[s];
      if (ms == -INFINITY) continue;
      const float c = exp_ref(ms - MM);
      LL = LL + gl[s] * c;
      AA = AA + ga[s][tid] * c;
    }
    p.out[bh * HD + tid] = LL > 0.f ? AA / LL : 0.f;
  }
}

// ---- few streams, short windows: flat chunks merged by the last CTA ---------------------
//
// At batch 1 one layer's keys and values (12.3 MB of f32 for STT-1b) have been pulled into L2
// by the kernel two places earlier, and the cluster kernel above is bound by its chain of
// latencies (cluster scheduling, staging, cluster barrier), not by HBM: it takes as long on
// L2-resident data as on cold data. Here each (stream, head) unit's keys are cut into
// p.splits flat chunks of at most kFlatMaxKeys keys, one CTA each (about two per SM), with no
// cluster and no staging:
//  - before the dependency wait each warp loads its keys' rows (every key but the newest,
//    which the in-projection writes) straight into registers, lane i holding dims
//    [i * DL, (i + 1) * DL) of a row;
//  - after it, q and the newest key. The warp scores its keys (the lane's DL products, then a
//    butterfly sum, which leaves the same value in every lane), takes their max and adds its
//    keys in order; the CTA merges its warps in warp order and stores the chunk's partial
//    (max, sum of weights, weighted values) in p.part;
//  - the last CTA of the unit to finish (a ticket per unit, p.ticket) merges the unit's
//    chunks in chunk order and writes the output, then clears the ticket for the next launch.
// The merge orders are fixed, so the result does not depend on timing. Nothing here waits.
constexpr int kFlatWarps = 8;
constexpr int kFlatKeysPerWarp = 6;
constexpr int kFlatMaxKeys = kFlatWarps * kFlatKeysPerWarp;  // keys per chunk at most
constexpr int kFlatMaxSplits = 2 * 148;                         // chunks per unit at most

// W 32-bit words of a key row per lane (DL dims of f32, or of bf16 pairs), loaded through L2
// with eviction policy `pol` (the window is read once per step, so its lines go first).
template <int W>
__device__ __forceinline__ void ld_row_words_hint(const uint8_t* src, uint32_t (&w)[W], uint64_t pol) {
  if constexpr (W == 4) {
    asm volatile("ld.global.cg.L2::cache_hint.v4.u32 {%0, %1, %2, %3}, [%4], %5;"
                 : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3])
                 : "l"(src), "l"(pol));
  } else if constexpr (W == 2) {
    asm volatile("ld.global.cg.L2::cache_hint.v2.u32 {%0, %1}, [%2], %3;" : "=r"(w[0]), "=r"(w[1]) : "l"(src), "l"(pol));
  } else {
    asm volatile("ld.global.cg.L2::cache_hint.u32 %0, [%1], %2;" : "=r"(w[0]) : "l"(src), "l"(pol));
  }
}
// The same without a policy.
template <int W>
__device__ __forceinline__ void ld_row_words(const uint8_t* src, uint32_t (&w)[W]) {
  if constexpr (W == 4) {
    const uint4 v = __ldcg(reinterpret_cast<const uint4*>(src));
    w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
  } else if constexpr (W == 2) {
    const uint2 v = __ldcg(reinterpret_cast<const uint2*>(src));
    w[0] = v.x; w[1] = v.y;
  } else {
    w[0] = __ldcg(reinterpret_cast<const unsigned int*>(src));
  }
}
template <int DL, bool BF16, int W>
__device__ __forceinline__ float row_dim(const uint32_t (&w)[W], int i) {
  if (BF16) return (i & 1) ? bf16_hi(w[i >> 1]) : bf16_lo(w[i >> 1]);
  return __uint_as_float(w[i]);
}

template <int HD, bool BF16>
__global__ void __launch_bounds__(kFlatWarps * 32, 3) attn_flat_kernel(const AttnParams p) {
  constexpr int DL = HD / 32;           // dims per lane
  constexpr int EL = BF16 ? 2 : 4;
  constexpr int W = DL * EL / 4;        // 32-bit words per lane per row
  constexpr int ROW = HD * EL;
  constexpr int KPW = kFlatKeysPerWarp;
  constexpr int PS = HD + 4;            // floats per partial: values, then max and sum
  __shared__ float sm_m[kFlatWarps], sm_l[kFlatWarps];
  __shared__ float sm_a[kFlatWarps][HD];
  __shared__ float fl_m[kFlatMaxSplits], fl_l[kFlatMaxSplits];  // the last CTA's merge
  __shared__ bool last;

  const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int S = p.splits;
  const int pos = p.pos[b];  // advanced only by the last kernel of a step
  const int count = p.window > 0 ? min(pos + 1, p.window) : pos + 1;
  const int kps = (count + S - 1) / S;
  const int j0 = min(split * kps, count), j1 = min(j0 + kps, count);
  const int first_pos = pos - count + 1;
  const int kvh = h / (p.heads / p.kv_heads);
  const int64_t head_base = (b * p.ring_stream_stride + (int64_t)kvh * p.ring_cap * HD) * EL;
  const uint8_t* kg = static_cast<const uint8_t*>(p.k_ring) + head_base + lane * DL * EL;
  const uint8_t* vg = static_cast<const uint8_t*>(p.v_ring) + head_base + lane * DL * EL;
  auto row_off = [&](int j) {
    const int q = first_pos + j;
    return (int64_t)(p.window > 0 ? q % p.ring_cap : q) * ROW;
  };

  // Key r of this warp: j0 + warp + r * kFlatWarps.
  const uint64_t pol = l2_evict_first();
  uint32_t kw[KPW][W], vw[KPW][W];
#pragma unroll
  for (int r = 0; r < KPW; r++) {
    const int j = j0 + warp + r * kFlatWarps;
    if (j < j1 && j != count - 1) {
      ld_row_words_hint<W>(kg + row_off(j), kw[r], pol);
      ld_row_words_hint<W>(vg + row_off(j), vw[r], pol);
    }
  }
  if (tid == 0) {
    const int cta = split + S * (h + p.heads * b), ctas = S * p.heads * p.nb;
    for (int i = 0; i < kMaxPrefetch; i++) prefetch_l2_share(p.pf[i].p, p.pf[i].bytes, cta, ctas);
  }
  pdl_launch();
  pdl_wait();

#pragma unroll
  for (int r = 0; r < KPW; r++) {
    const int j = j0 + warp + r * kFlatWarps;
    if (j < j1 && j == count - 1) {
      ld_row_words<W>(kg + row_off(j), kw[r]);
      ld_row_words<W>(vg + row_off(j), vw[r]);
    }
  }
  const int64_t unit = (int64_t)b * p.heads + h;
  float q[DL];
  {
    uint32_t qw[DL];
    ld_row_words<DL>(reinterpret_cast<const uint8_t*>(p.q + unit * HD + lane * DL), qw);
#pragma unroll
    for (int i = 0; i < DL; i++) q[i] = __uint_as_float(qw[i]);
  }
  float sc[KPW];
#pragma unroll
  for (int r = 0; r < KPW; r++) {
    float d = 0.f;
#pragma unroll
    for (int i = 0; i < DL; i++) d = fmaf(q[i], row_dim<DL, BF16, W>(kw[r], i), d);
    sc[r] = d;
  }
#pragma unroll
  for (int o = 16; o; o >>= 1)
#pragma unroll
    for (int r = 0; r < KPW; r++) sc[r] += __shfl_xor_sync(0xffffffffu, sc[r], o);
  float m = -INFINITY;
#pragma unroll
  for (int r = 0; r < KPW; r++) {
    const bool valid = j0 + warp + r * kFlatWarps < j1;
    sc[r] = valid ? p.scale * sc[r] : -INFINITY;  // scale * dot(q, k), as the reference
    m = fmaxf(m, sc[r]);
  }
  float l = 0.f, acc[DL];
#pragma unroll
  for (int i = 0; i < DL; i++) acc[i] = 0.f;
  if (m != -INFINITY) {
#pragma unroll
    for (int r = 0; r < KPW; r++) {
      if (sc[r] == -INFINITY) continue;
      const float e = exp_ref(sc[r] - m);
      l = l + e;
#pragma unroll
      for (int i = 0; i < DL; i++) acc[i] = acc[i] + e * row_dim<DL, BF16, W>(vw[r], i);
    }
  }
#pragma unroll
  for (int i = 0; i < DL; i++) sm_a[warp][lane * DL + i] = acc[i];
  if (lane == 0) {
    sm_m[warp] = m;
    sm_l[warp] = l;
  }
  __syncthreads();

  // The chunk's partial: thread t < HD merges dim t of the warps, in warp order.
  float A = 0.f, L = 0.f, M = -INFINITY;
  if (tid < HD) {
#pragma unroll
    for (int w = 0; w < kFlatWarps; w++) M = fmaxf(M, sm_m[w]);
    if (M != -INFINITY)
#pragma unroll
      for (int w = 0; w < kFlatWarps; w++) {
        if (sm_m[w] == -INFINITY) continue;
        const float c = exp_ref(sm_m[w] - M);
        L = L + sm_l[w] * c;
        A = A + sm_a[w][tid] * c;
      }
  }
  if (S == 1) {
    if (tid < HD) p.out[unit * HD + tid] = L > 0.f ? A / L : 0.f;
    return;
  }
  float* part = p.part + (unit * S + split) * PS;
  if (tid < HD) {
    part[tid] = A;
    if (tid == 0) {
      part[HD] = M;
      part[HD + 1] = L;
    }
    __threadfence();
  }
  __syncthreads();
  if (tid == 0) last = atomicAdd(p.ticket + unit, 1u) == (unsigned)S - 1;
  __syncthreads();
  if (!last) return;
  __threadfence();
  // The unit's chunks in chunk order. Dim t of the first 32 chunks (thread t < HD), and every
  // chunk's max and sum (one thread per chunk), are loaded at once; then each chunk's scale
  // exp(max_s - max) (0 for an empty chunk); further chunks come 32 per round trip.
  const float* up = p.part + unit * S * PS;
  constexpr int kU = 32;
  float a[kU];
  if (tid < HD) {
#pragma unroll
    for (int u = 0; u < kU; u++) a[u] = u < S ? __ldcg(up + (int64_t)u * PS + tid) : 0.f;
  }
  for (int i = tid; i < S; i += kFlatWarps * 32) {
    fl_m[i] = __ldcg(up + (int64_t)i * PS + HD);
    fl_l[i] = __ldcg(up + (int64_t)i * PS + HD + 1);
  }
  __syncthreads();
  float MM = -INFINITY;
  for (int i = 0; i < S; i++) MM = fmaxf(MM, fl_m[i]);
  __syncthreads();
  for (int i = tid; i < S; i += kFlatWarps * 32) fl_m[i] = fl_m[i] == -INFINITY ? 0.f : exp_ref(fl_m[i] - MM);
  __syncthreads();
  if (tid < HD) {
    float LL = 0.f, AA = 0.f;
    for (int s0 = 0; s0 < S; s0 += kU) {
      if (s0 > 0) {
#pragma unroll
        for (int u = 0; u < kU; u++) a[u] = s0 + u < S ? __ldcg(up + (int64_t)(s0 + u) * PS + tid) : 0.f;
      }
#pragma unroll
      for (int u = 0; u < kU; u++) {
        if (s0 + u >= S) break;
        const float c = fl_m[s0 + u];
        LL = LL + fl_l[s0 + u] * c;
        AA = AA + a[u] * c;
      }
    }
    p.out[unit * HD + tid] = LL > 0.f ? AA / LL : 0.f;
  }
  if (tid == 0) p.ticket[unit] = 0u;
}

// ---- many streams: pieces of a fixed key count -----------------------------------------
//
// With hundreds of streams there are thousands of (stream, head) units per layer, and their
// windows fill to different lengths (streams start at different times). A unit's window
// occupies ring slots [0, count): until the window is full the keys sit in slots 0 .. pos,
// after that every slot holds a key of the window (the ring's capacity is the window). Keys
// are independent under softmax, so a unit's keys are taken in slot order, and a chunk of KC
// consecutive slots never wraps. The slots of a unit are cut into pieces of `p.piece` (the
// last one shorter); a work item is one piece, and warp w of W takes items w, w + W, ...
// (pieces are of one size, so the warps get the same work to within a piece).
//
// The warp is its own producer. bf16 caches: lane 0 loads a chunk's keys and values with
// tensor-map copies (boxes of 64 dims x KC slots, 128-byte swizzle, so ldmatrix reads them
// without bank conflicts) into the warp's 2-slot ring, and the item's q with its first chunk;
// q.k and p.v run on the tensor cores (mma m16n8k16, f32 accumulation). The f32 operand (q,
// then the probabilities) is split into three bf16 parts x = hi + mid + lo (24 significant
// bits, the f32 value to rounding) placed in rows 0, 8 and 1 of the A tile, so a key's score
// is the sum of three exact-product rows and the arithmetic stays f32-accurate. f32 caches:
// 1-D bulk copies, and lane groups of LPK lanes score a key (16 dims per lane) on the FMA pipe.
// Either way a chunk's scores are gathered so that lane j holds key j's: the max, exp and sum
// are one warp instruction each, and the accumulators are rescaled only when the running max
// rises. Before griddepcontrol.wait only the first item's chunks are copied; the newest key
// (this step's) in them is then replaced from global memory, and q read from global.
// A unit of one piece writes its output directly; otherwise each piece writes its partial
// (max, sum, weighted values) and attn_merge_kernel, launched next, combines them in piece
// order. Every wait is bounded (a wait that runs out sets *p.err to 4).
constexpr int kWWarps = 12;                // warps per CTA (one CTA per SM)
constexpr int kWSlots = 2;                 // ring slots per warp
constexpr int kWQueue = 4;                 // item descriptors in flight per warp (> slots)
constexpr int kMergeWarps = 8;             // attn_merge_kernel: one warp per unit
constexpr int kWMaxPieces = 16;
constexpr int kWChunk = 8192;              // keys and values of a chunk
constexpr int kWSmemLimit = 227 * 1024 - 2048;  // dynamic shared memory, static arrays aside

template <int HD, bool BF16>
struct WShape {
  static constexpr int EL = BF16 ? 2 : 4;
  static constexpr int ROW = HD * EL;                   // bytes per key row in the ring
  static constexpr int KC = kWChunk / 2 / ROW;          // keys per chunk (8 .. 32)
  static constexpr int QB = HD * 4;                     // the item's q
  static constexpr int KV = kWWarps * kWSlots * kWChunk;
  static constexpr int RING = 1024 + KV + kWWarps * kWSlots * QB;  // 1024: alignment slack
  static constexpr int MAX_NB = (kWSmemLimit - RING) / 4 - 1;     // the item prefix is [nb + 1]
};

struct WItem {
  int b, h, k, npc;  // stream, head, piece, pieces of the unit
  int a0, a1;        // ring slots [a0, a1)
  int count, ns;     // keys in the window, ring slot of the newest key
};

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* tm, int c0, int c1, int c2,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_addr(bar))
      : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
// D += A B, m16n8k16, bf16 operands, f32 accumulators.
__device__ __forceinline__ void mma_bf16(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
__device__ __forceinline__ uint32_t pack_bf16(float lo_elem, float hi_elem) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo_elem, hi_elem);
  return *reinterpret_cast<const uint32_t*>(&v);
}
// A fragment (rows 0, 8: hi, mid in lanes 0-3; row 1: lo in lanes 4-7; other rows 0) of the
// pairs (x0, x1) at columns 2l, 2l + 1 and (x2, x3) at columns 8 + 2l, 9 + 2l.
__device__ __forceinline__ void split_frag(int lane, float x0, float x1, float x2, float x3, uint32_t* a) {
  const float h0 = bf16r(x0), h1 = bf16r(x1), h2 = bf16r(x2), h3 = bf16r(x3);
  const float r0 = x0 - h0, r1 = x1 - h1, r2 = x2 - h2, r3 = x3 - h3;  // exact
  const float m0 = bf16r(r0), m1 = bf16r(r1), m2 = bf16r(r2), m3 = bf16r(r3);
  if (lane < 4) {
    a[0] = pack_bf16(h0, h1);
    a[2] = pack_bf16(h2, h3);
    a[1] = pack_bf16(m0, m1);
    a[3] = pack_bf16(m2, m3);
  } else if (lane < 8) {
    a[0] = pack_bf16(r0 - m0, r1 - m1);
    a[2] = pack_bf16(r2 - m2, r3 - m3);
    a[1] = a[3] = 0u;
  } else {
    a[0] = a[1] = a[2] = a[3] = 0u;
  }
}
// Byte offset of (slot row r, 16-byte column c) in a chunk's keys or values: bf16, boxes of
// 64 dims (128 bytes) x KC rows with the 128-byte swizzle; f32, plain rows.
template <int HD, bool BF16>
__device__ __forceinline__ int chunk_off(int r, int c) {
  using S = WShape<HD, BF16>;
  if constexpr (BF16) return (c >> 3) * (S::KC * 128) + r * 128 + (((c & 7) ^ (r & 7)) << 4);
  else return r * S::ROW + (c << 4);
}

template <int HD, bool BF16>
__global__ void __launch_bounds__(kWWarps * 32, 1)
    attn_warp_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                     const AttnParams p) {
  using S = WShape<HD, BF16>;
  constexpr int EL = S::EL, ROW = S::ROW, KC = S::KC;
  constexpr int LPK = HD / 16;           // FMA path: lanes per key (16 dims each)
  constexpr int KPP = 32 / LPK;          // FMA path: keys per pass
  constexpr int NT = KC / 8, KS = HD / 16, PK = KC / 16, DT = HD / 8;  // tensor-core tiles
  constexpr int NACC = BF16 ? DT * 4 : 16;
  constexpr int PS = HD + 4;             // floats per partial: values, max, sum, pad
  static_assert(KC % KPP == 0 && KC <= 32 && (!BF16 || KC % 16 == 0), "chunk shape");
  extern __shared__ __align__(128) uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full[kWWarps][kWSlots];
  __shared__ int4 desc[kWWarps][kWQueue][2];
  __shared__ int sflag[kWWarps][kWSlots];  // bit 0: q in the slot; bit 1: the newest key is stale
  __shared__ int wsum[kWWarps];
  // The swizzled boxes want 1024-byte alignment.
  uint8_t* smem = smem_raw + ((1024 - (smem_addr(smem_raw) & 1023)) & 1023);
  int* cum = reinterpret_cast<int*>(smem_raw + S::RING);  // [nb + 1] items before stream b
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t* ring = smem + (size_t)warp * kWSlots * kWChunk;
  float* qring = reinterpret_cast<float*>(smem + S::KV) + (size_t)warp * kWSlots * HD;
  uint64_t* bar = full[warp];
  const int nb = p.nb, heads = p.heads, P = p.piece;
  const int kk = lane / LPK, sub = lane % LPK;

  // Items per stream (heads x pieces) and their prefix. Positions are advanced only by the
  // last kernel of a step, so they are read before the dependency wait.
  auto count_of = [&](int b) {
    const int pos = p.pos[b];
    return p.window > 0 ? min(pos + 1, p.window) : pos + 1;
  };
  {
    const int per = (nb + (int)blockDim.x - 1) / (int)blockDim.x;
    const int b0 = min((int)threadIdx.x * per, nb), b1 = min(b0 + per, nb);
    int local = 0;
    for (int b = b0; b < b1; b++) local += heads * ((count_of(b) + P - 1) / P);
    int x = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) wsum[warp] = x;
    if (threadIdx.x == 0) {
      for (int w = 0; w < kWWarps; w++)
        for (int i = 0; i < kWSlots; i++) mbar_init(&full[w][i], 1);
      fence_mbar_init();
    }
    __syncthreads();
    int run = x - local;
    for (int w = 0; w < warp; w++) run += wsum[w];
    for (int b = b0; b < b1; b++) {
      cum[b] = run;
      run += heads * ((count_of(b) + P - 1) / P);
    }
    if (threadIdx.x == blockDim.x - 1) cum[nb] = run;
    __syncthreads();
  }
  const int total = cum[nb];
  auto decode = [&](int t, WItem& w) {
    int lo = 0, hi = nb;  // cum[lo] <= t < cum[hi]
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (cum[mid] <= t) lo = mid;
      else hi = mid;
    }
    const int npc = (cum[lo + 1] - cum[lo]) / heads, r = t - cum[lo];
    const int pos = p.pos[lo];
    w.b = lo;
    w.h = r / npc;
    w.k = r - w.h * npc;
    w.npc = npc;
    w.count = p.window > 0 ? min(pos + 1, p.window) : pos + 1;
    w.a0 = w.k * P;
    w.a1 = min(w.a0 + P, w.count);
    w.ns = p.window > 0 ? pos % p.ring_cap : pos;
  };
  // Ring row (tensor-map coordinate, or row of the layer's ring) of slot 0 of a unit.
  auto unit_row = [&](const WItem& w) {
    return (int64_t)(w.b * p.kv_heads + w.h / (heads / p.kv_heads)) * p.ring_cap;
  };

  const int gw = blockIdx.x * kWWarps + warp, W = gridDim.x * kWWarps;
  uint32_t issued = 0, consumed = 0;  // chunks; chunk i uses slot i % kWSlots, phase (i / kWSlots) & 1
  int pq = 0, cq = 0;                 // items the producer started / the consumer started
  WItem pi{}, ci{};
  int pc = 0, pnc = 0, cc = 0, cnc = 0;  // next chunk and chunk count of pi / ci
  bool pmore = gw < total, waited = false;
  int failed = 0, next_t = gw;  // the item the producer takes next

  auto start_item = [&](int t) {
    decode(t, pi);
    pc = 0;
    pnc = (pi.a1 - pi.a0 + KC - 1) / KC;
    if (lane == 0) {
      desc[warp][pq % kWQueue][0] = make_int4(pi.b, pi.h, pi.k, pi.npc);
      desc[warp][pq % kWQueue][1] = make_int4(pi.a0, pi.a1, pi.count, pi.ns);
    }
    pq++;
  };
  // Lane 0 copies chunk pc of pi into the next slot (the slot's earlier reads are complete:
  // every lane passed __syncwarp after consuming it).
  auto issue_chunk = [&]() {
    const uint32_t slot = issued % kWSlots;
    if (lane == 0) {
      uint8_t* dst = ring + (size_t)slot * kWChunk;
      const int a = pi.a0 + pc * KC, e = min(a + KC, pi.a1);
      const bool stale = !waited && pi.ns >= a && pi.ns < e;  // written by this step's in-projection
      const bool qcopy = pc == 0 && waited;
      sflag[warp][slot] = (qcopy ? 1 : 0) | (stale ? 2 : 0);
      const int64_t row = unit_row(pi) + a;
      if constexpr (BF16) {
        mbar_expect_tx(&bar[slot], (uint32_t)kWChunk + (qcopy ? HD * 4u : 0u));
#pragma unroll
        for (int hb = 0; hb < HD / 64; hb++) {
          tma_load_3d(dst + hb * KC * 128, &tmk, 64 * hb, (int)(p.ring_row0 + row), p.layer, &bar[slot]);
          tma_load_3d(dst + kWChunk / 2 + hb * KC * 128, &tmv, 64 * hb, (int)(p.ring_row0 + row), p.layer,
                      &bar[slot]);
        }
      } else {
        const uint32_t bytes = (uint32_t)(e - a) * ROW;
        mbar_expect_tx(&bar[slot], 2u * bytes + (qcopy ? HD * 4u : 0u));
        bulk_g2s(dst, static_cast<const uint8_t*>(p.k_ring) + row * ROW, bytes, &bar[slot]);
        bulk_g2s(dst + kWChunk / 2, static_cast<const uint8_t*>(p.v_ring) + row * ROW, bytes, &bar[slot]);
      }
      if (qcopy)
        bulk_g2s(qring + (size_t)slot * HD, p.q + ((int64_t)pi.b * heads + pi.h) * HD, HD * 4u, &bar[slot]);
    }
    pc++;
    issued++;
  };
  // Keep the ring full: before the dependency wait only the first item's chunks.
  auto produce = [&]() {
    while (!failed && pmore && issued - consumed < (uint32_t)kWSlots) {
      if (pc == pnc) {
        if (!waited) break;
        next_t += W;
        if (next_t >= total) {
          pmore = false;
          break;
        }
        start_item(next_t);
      }
      issue_chunk();
    }
  };

  float M = -INFINITY, L = 0.f, acc[NACC];
  float q[16];             // FMA path: this lane's 16 dims of q
  uint32_t qa[KS][4];      // tensor-core path: A fragments of q
#pragma unroll
  for (int t = 0; t < NACC; t++) acc[t] = 0.f;
#pragma unroll
  for (int t = 0; t < 16; t++) q[t] = 0.f;
#pragma unroll
  for (int t = 0; t < KS; t++) qa[t][0] = qa[t][1] = qa[t][2] = qa[t][3] = 0u;

  auto load_q = [&](const float* src, bool global) {
    if constexpr (BF16) {
      const int l2 = 2 * (lane & 3);
#pragma unroll
      for (int ks = 0; ks < KS; ks++) {
        const float* s0 = src + 16 * ks + l2;
        const float2 x01 = global ? __ldcg(reinterpret_cast<const float2*>(s0)) : *reinterpret_cast<const float2*>(s0);
        const float2 x23 = global ? __ldcg(reinterpret_cast<const float2*>(s0 + 8)) : *reinterpret_cast<const float2*>(s0 + 8);
        split_frag(lane, x01.x, x01.y, x23.x, x23.y, qa[ks]);
      }
    } else {
      const float4* qp = reinterpret_cast<const float4*>(src) + sub * 4;
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const float4 v = global ? __ldcg(qp + i) : qp[i];
        q[4 * i] = v.x;
        q[4 * i + 1] = v.y;
        q[4 * i + 2] = v.z;
        q[4 * i + 3] = v.w;
      }
    }
  };
  // Online-softmax update for the chunk's scores (lane j: key j, -inf past the chunk); returns
  // this lane's weight exp(s - M) and rescales the accumulators when the max rises.
  auto softmax = [&](float sc, int n) {
    const float mn = fmaxf(M, warp_max(sc));
    const float e = lane < n ? exp_ref(sc - mn) : 0.f;
    if (mn != M) {  // uniform: M and mn are the same in every lane
      const float c = M == -INFINITY ? 0.f : exp_ref(M - mn);
      L *= c;
#pragma unroll
      for (int t = 0; t < NACC; t++) acc[t] *= c;
      M = mn;
    }
    L += warp_sum(e);
    return e;
  };
  // Scores and values of the chunk's first n keys (n <= KC) at kb / vb.
  auto consume = [&](const uint8_t* kb, const uint8_t* vb, int n) {
    if constexpr (BF16) {
      const int l = lane & 3;
      float c[NT][4];
#pragma unroll
      for (int t = 0; t < NT; t++) {
        c[t][0] = c[t][1] = c[t][2] = c[t][3] = 0.f;
        const int r = 8 * t + (lane & 7);
#pragma unroll
        for (int ks = 0; ks < KS; ks += 2) {
          uint32_t b[4];  // keys 8t .. 8t + 7; dims 16 ks .. 16 ks + 31
          ldsm_x4(smem_addr(kb + chunk_off<HD, BF16>(r, 2 * ks + (lane >> 3))), b);
          mma_bf16(c[t], qa[ks], b[0], b[1]);
          mma_bf16(c[t], qa[ks + 1], b[2], b[3]);
        }
      }
      // Lanes 0-3 hold keys 8t + 2l + {0, 1}: rows hi (c0, c1), mid (c2, c3), lo (lane + 4).
      float sc = -INFINITY;
#pragma unroll
      for (int t = 0; t < NT; t++)
#pragma unroll
        for (int e = 0; e < 2; e++) {
          const float lo = __shfl_down_sync(0xffffffffu, c[t][e], 4);
          const float full_s = (lo + c[t][2 + e]) + c[t][e];
          const float x = __shfl_sync(0xffffffffu, full_s, (lane & 7) >> 1);
          if ((lane >> 3) == t && (lane & 1) == e) sc = x;
        }
      sc = lane < n ? p.scale * sc : -INFINITY;  // scale * dot(q, k), as the reference
      const float w = softmax(sc, n);
#pragma unroll
      for (int pk = 0; pk < PK; pk++) {
        const int kb0 = 16 * pk + 2 * l;
        const float w0 = __shfl_sync(0xffffffffu, w, kb0), w1 = __shfl_sync(0xffffffffu, w, kb0 + 1);
        const float w2 = __shfl_sync(0xffffffffu, w, kb0 + 8), w3 = __shfl_sync(0xffffffffu, w, kb0 + 9);
        uint32_t pa[4];
        split_frag(lane, w0, w1, w2, w3, pa);
        const int r = 16 * pk + 8 * ((lane >> 3) & 1) + (lane & 7);
#pragma unroll
        for (int dt = 0; dt < DT; dt += 2) {
          uint32_t b[4];  // keys 16 pk .. 16 pk + 15; dims 8 dt .. 8 dt + 15
          ldsm_x4_t(smem_addr(vb + chunk_off<HD, BF16>(r, dt + (lane >> 4))), b);
          mma_bf16(&acc[4 * dt], pa, b[0], b[1]);
          mma_bf16(&acc[4 * (dt + 1)], pa, b[2], b[3]);
        }
      }
    } else {
      float sc = -INFINITY;
#pragma unroll
      for (int pass = 0; pass < KC / KPP; pass++) {
        const int j = pass * KPP + kk;
        float d = 0.f;
        if (j < n) {
          float kv[16];
          unpack16<BF16>(kb + (size_t)j * ROW + sub * 16 * EL, kv);
#pragma unroll
          for (int t = 0; t < 16; t++) d = fmaf(q[t], kv[t], d);
        }
#pragma unroll
        for (int o = LPK / 2; o; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
        const float sp = __shfl_sync(0xffffffffu, d, (lane % KPP) * LPK);
        if (lane / KPP == pass && lane < n) sc = p.scale * sp;  // scale * dot(q, k)
      }
      const float w = softmax(sc, n);
#pragma unroll
      for (int pass = 0; pass < KC / KPP; pass++) {
        const int j = pass * KPP + kk;
        const float wj = __shfl_sync(0xffffffffu, w, j & 31);
        if (j < n) {
          float vv[16];
          unpack16<BF16>(vb + (size_t)j * ROW + sub * 16 * EL, vv);
#pragma unroll
          for (int t = 0; t < 16; t++) acc[t] = fmaf(wj, vv[t], acc[t]);
        }
      }
    }
  };
  // The item's keys are all in (M, L, acc): write the output, or the partial.
  auto finish_item = [&]() {
    const int64_t u = (int64_t)ci.b * heads + ci.h;
    const bool direct = ci.npc == 1;
    float* dst = direct ? p.out + u * HD : p.part + (u * p.npieces + ci.k) * PS;
    const float inv = direct ? 1.f / L : 1.f;
    if constexpr (BF16) {
      // Lanes 0-3: dims 8 dt + 2l + {0, 1} = hi + mid + lo rows.
#pragma unroll
      for (int dt = 0; dt < DT; dt++) {
        const float lo0 = __shfl_down_sync(0xffffffffu, acc[4 * dt], 4);
        const float lo1 = __shfl_down_sync(0xffffffffu, acc[4 * dt + 1], 4);
        if (lane < 4) {
          const float o0 = (lo0 + acc[4 * dt + 2]) + acc[4 * dt], o1 = (lo1 + acc[4 * dt + 3]) + acc[4 * dt + 1];
          __stcg(reinterpret_cast<float2*>(dst + 8 * dt + 2 * lane), make_float2(o0 * inv, o1 * inv));
        }
      }
    } else {
      // Lane groups hold disjoint keys under the same running max: their sums add up.
#pragma unroll
      for (int o = LPK; o < 32; o <<= 1)
#pragma unroll
        for (int t = 0; t < 16; t++) acc[t] += __shfl_xor_sync(0xffffffffu, acc[t], o);
      if (kk == 0) {
#pragma unroll
        for (int t = 0; t < 16; t += 4)
          __stcg(reinterpret_cast<float4*>(dst + sub * 16 + t),
                 make_float4(acc[t] * inv, acc[t + 1] * inv, acc[t + 2] * inv, acc[t + 3] * inv));
      }
    }
    if (!direct && lane == 0) __stcg(reinterpret_cast<float2*>(dst + HD), make_float2(M, L));
  };

  if (pmore) start_item(gw);
  produce();
  pdl_launch();
  pdl_wait();  // q and the newest keys of this step come from the previous kernels
  waited = true;
  while (true) {
    produce();
    if (failed || consumed == issued) break;
    const uint32_t slot = consumed % kWSlots;
    if (!mbar_wait(&bar[slot], (consumed / kWSlots) & 1u)) {
      if (lane == 0) atomicExch(p.err, 4);
      failed = 1;
      break;
    }
    uint8_t* kb = ring + (size_t)slot * kWChunk;
    uint8_t* vb = kb + kWChunk / 2;
    const int flags = sflag[warp][slot];
    if (cc == cnc) {  // the first chunk of the next item
      const int4 d0 = desc[warp][cq % kWQueue][0], d1 = desc[warp][cq % kWQueue][1];
      ci = WItem{d0.x, d0.y, d0.z, d0.w, d1.x, d1.y, d1.z, d1.w};
      cq++;
      cc = 0;
      cnc = (ci.a1 - ci.a0 + KC - 1) / KC;
      M = -INFINITY;
      L = 0.f;
#pragma unroll
      for (int t = 0; t < NACC; t++) acc[t] = 0.f;
      if (flags & 1) load_q(qring + (size_t)slot * HD, false);
      else load_q(p.q + ((int64_t)ci.b * heads + ci.h) * HD, true);
    }
    const int a = ci.a0 + cc * KC, n = min(KC, ci.a1 - a);
    bool touched = false;
    if (flags & 2) {
      // The newest key was copied before this step wrote it: its row again, from global.
      const int r = ci.ns - a;
      const int64_t off = (unit_row(ci) + ci.ns) * ROW;
      for (int i = lane; i < 2 * (ROW / 16); i += 32) {
        const int isv = i >= ROW / 16, c = i - (isv ? ROW / 16 : 0);
        const uint4 v = __ldcg(reinterpret_cast<const uint4*>(
            static_cast<const uint8_t*>(isv ? p.v_ring : p.k_ring) + off + c * 16));
        *reinterpret_cast<uint4*>((isv ? vb : kb) + chunk_off<HD, BF16>(r, c)) = v;
      }
      touched = true;
    }
    if (BF16 && n < KC) {
      // Rows past the window (another unit's keys, or never written) get weight 0: make their
      // values 0 so that they add nothing whatever they hold.
      for (int i = lane; i < (KC - n) * (ROW / 16); i += 32) {
        const int r = n + i / (ROW / 16), c = i % (ROW / 16);
        *reinterpret_cast<uint4*>(vb + chunk_off<HD, BF16>(r, c)) = make_uint4(0u, 0u, 0u, 0u);
      }
      touched = true;
    }
    if (touched) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // before a copy overwrites them
      __syncwarp();
    }
    consume(kb, vb, n);
    __syncwarp();
    consumed++;
    cc++;
    if (cc == cnc) finish_item();
  }
  // Copies still in flight (a failed wait) land before the CTA exits (bounded).
  if (failed && lane == 0)
    for (uint32_t i = consumed; i < issued; i++) mbar_wait(&bar[i % kWSlots], (i / kWSlots) & 1u);
}

// The units of several pieces: their partials merged in piece order, one warp per unit.
template <int HD>
__global__ void __launch_bounds__(kMergeWarps * 32) attn_merge_kernel(const AttnParams p) {
  constexpr int PS = HD + 4, DL = HD / 32;
  const int lane = threadIdx.x & 31;
  const int64_t u = (int64_t)blockIdx.x * kMergeWarps + (threadIdx.x >> 5);
  pdl_launch();
  pdl_wait();
  if (u >= (int64_t)p.nb * p.heads) return;
  const int pos = p.pos[u / p.heads];
  const int count = p.window > 0 ? min(pos + 1, p.window) : pos + 1;
  const int npc = (count + p.piece - 1) / p.piece;
  if (npc == 1) return;  // written by the attention kernel
  const float* base = p.part + u * p.npieces * PS;
  float MM = -INFINITY;
  for (int k = 0; k < npc; k++) MM = fmaxf(MM, __ldcg(base + k * PS + HD));
  float LL = 0.f, A[DL];
#pragma unroll
  for (int i = 0; i < DL; i++) A[i] = 0.f;
  for (int k = 0; k < npc; k++) {
    const float2 ml = __ldcg(reinterpret_cast<const float2*>(base + k * PS + HD));
    const float c = exp_ref(ml.x - MM);
    LL = LL + ml.y * c;
    const float* a = base + k * PS + lane * DL;
    if constexpr (DL == 4) {
      const float4 v = __ldcg(reinterpret_cast<const float4*>(a));
      A[0] = A[0] + v.x * c;
      A[1] = A[1] + v.y * c;
      A[2] = A[2] + v.z * c;
      A[3] = A[3] + v.w * c;
    } else {
      const float2 v = __ldcg(reinterpret_cast<const float2*>(a));
      A[0] = A[0] + v.x * c;
      A[1] = A[1] + v.y * c;
    }
  }
  float* out = p.out + u * HD + lane * DL;
#pragma unroll
  for (int i = 0; i < DL; i++) out[i] = A[i] / LL;
}

template <int HD, bool BF16>
bool launch_w(const AttnParams& p, cudaStream_t s) {
  using S = WShape<HD, BF16>;
  if (p.nb > S::MAX_NB || (BF16 && !p.kmap)) return false;
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t items = (int64_t)p.nb * p.heads * p.npieces;
  const int grid = (int)std::min<int64_t>(sms, (items + kWWarps - 1) / kWWarps);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kWWarps * 32);
  cfg.dynamicSmemBytes = S::RING + (p.nb + 1) * 4;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  CUtensorMap none{};
  const CUtensorMap& tk = p.kmap ? *reinterpret_cast<const CUtensorMap*>(p.kmap) : none;
  const CUtensorMap& tv = p.vmap ? *reinterpret_cast<const CUtensorMap*>(p.vmap) : none;
  cudaLaunchKernelEx(&cfg, attn_warp_kernel<HD, BF16>, tk, tv, p);
  if (p.npieces > 1) {
    cfg.gridDim = dim3((unsigned)(((int64_t)p.nb * p.heads + kMergeWarps - 1) / kMergeWarps));
    cfg.blockDim = dim3(kMergeWarps * 32);
    cfg.dynamicSmemBytes = 0;
    cudaLaunchKernelEx(&cfg, attn_merge_kernel<HD>, p);
  }
  return true;
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
void launch_f(const AttnParams& p, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.splits, p.heads, p.nb);
  cfg.blockDim = dim3(kFlatWarps * 32);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, attn_flat_kernel<HD, BF16>, p);
}

template <int HD, bool BF16>
void set_attr() {
  cudaFuncSetAttribute(attn_kernel<HD, BF16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       128 + 2 * kSlots * kTileBytes);
  cudaFuncSetAttribute(attn_kernel<HD, BF16>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
  cudaFuncSetAttribute(attn_warp_kernel<HD, BF16>, cudaFuncAttributeMaxDynamicSharedMemorySize, kWSmemLimit);
}

}  // namespace

int attention_max_splits() { return kMaxSplits; }

int attention_flat_max_keys() { return kFlatMaxKeys; }

void attention_init_device() {
  set_attr<64, false>();
  set_attr<64, true>();
  set_attr<128, false>();
  set_attr<128, true>();
}

int attention_chunk_keys(int head_dim, int kv_bf16) { return kWChunk / 2 / (head_dim * (kv_bf16 ? 2 : 4)); }

int attention_piece(int head_dim, int kv_bf16, int ring_cap, int* npieces) {
  const int kc = kWChunk / 2 / (head_dim * (kv_bf16 ? 2 : 4));
  const int per = (ring_cap + kWMaxPieces - 1) / kWMaxPieces;  // at most kWMaxPieces pieces
  const int piece = std::max(4 * kc, (per + kc - 1) / kc * kc);
  *npieces = (ring_cap + piece - 1) / piece;
  return piece;
}

void launch_attention_decode(const AttnParams& p, cudaStream_t s) {
  // Few streams, short windows: flat chunks (p.ticket set at state creation).
  if (p.ticket) {
    switch (p.head_dim * 2 + p.kv_bf16) {
      case 128: launch_f<64, false>(p, s); return;
      case 129: launch_f<64, true>(p, s); return;
      case 256: launch_f<128, false>(p, s); return;
      case 257: launch_f<128, true>(p, s); return;
      default: return;  // rejected at model creation
    }
  }
  if (p.splits == 1 && p.part) {
    // Enough (stream, head) units to cover the GPU: pieces handed out to warps (up to the
    // stream count whose item prefix fits in shared memory).
    bool ok = false;
    switch (p.head_dim * 2 + p.kv_bf16) {
      case 128: ok = launch_w<64, false>(p, s); break;
      case 129: ok = launch_w<64, true>(p, s); break;
      case 256: ok = launch_w<128, false>(p, s); break;
      case 257: ok = launch_w<128, true>(p, s); break;
      default: break;
    }
    if (ok) return;
  }
  switch (p.head_dim * 2 + p.kv_bf16) {
    case 128: launch_t<64, false>(p, s); break;
    case 129: launch_t<64, true>(p, s); break;
    case 256: launch_t<128, false>(p, s); break;
    case 257: launch_t<128, true>(p, s); break;
    default: break;  // rejected at model creation
  }
}

}  // namespace svl
