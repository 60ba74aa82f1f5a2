// gemv.cu — weight-streaming matrix-vector products for small stream counts.
//
// At small batch the step is bound by reading every weight once (the reference runs the
// same products on the CPU through kernels::matvec, nn/kernels/matvec.rs:29-58, and
// candle's QMatMul, nn/mod.rs:97). Two kernels:
//
//  - gemv_kernel (f32 / bf16 weights): each warp owns a contiguous range of row groups (R
//    rows) and streams them straight from global memory into registers, 16 bytes per lane
//    and U loads per row in flight.
//  - qgemv_kernel (Q8_0 / Q4_1 weights): the rows are stored in super-blocks (see
//    gemv_common.cuh) so that lane (r, l) of a warp -- row r of a group of 4, slot l of 8 --
//    streams slot l of every block of its row and runs the reference CPU dot's FMA chain for
//    that slot in block order; the warp's three xor-shuffles are the reference's horizontal
//    sum tree. The result is the reference CPU's value bit for bit on identical inputs.
//
// Both launch with programmatic dependent launch: each warp issues its first loads before
// griddepcontrol.wait (weights do not depend on the previous kernel), and one thread per CTA
// pulls its share of a later kernel's weights into L2 (cp.async.bulk.prefetch.L2). After the
// wait, every CTA turns the input row(s) into records in shared memory -- the layer's norm
// (candle rms_norm / layer_norm) and the conversion for the weight format (bf16 rounding, or
// the Q8_0 / Q8_1 activation blocks candle's QMatMul builds) -- while those first weight
// loads are in flight. Each row group ends with the fused epilogue (RoPE + KV-ring write,
// SwiGLU, GELU, SiLU, residual add, logits + argmax).
#include "common.cuh"
#include "gemv_common.cuh"
#include "kernels.cuh"
#include "sm100.cuh"

#include <algorithm>
#include <climits>

namespace svl {

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kCtasPerSm = 2;
constexpr int kGrid = 148 * kCtasPerSm;
// The argmax scratch (the state's and the no-allocation head's) holds one candidate per CTA.
static_assert(kGrid <= kLogitsGrid, "the argmax scratch holds kLogitsGrid CTAs per stream");

// 16 bytes of weights, read once per step: kept out of L1, evicted first from L2 (pol from
// l2_evict_first()).
__device__ __forceinline__ uint4 ldg_weights(const void* p, uint64_t pol) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p), "l"(pol));
  return r;
}
__device__ __forceinline__ uint32_t word_of(const uint4& v, int j) {
  return j == 0 ? v.x : j == 1 ? v.y : j == 2 ? v.z : v.w;
}
// Each CTA pulls its share of the later kernels' ranges into L2.
__device__ __forceinline__ void prefetch_share(const GemvParams& p) {
  if (threadIdx.x == 0)
#pragma unroll
    for (int i = 0; i < kMaxPrefetch; i++) prefetch_l2_share(p.pf[i].p, p.pf[i].bytes, blockIdx.x, gridDim.x);
}

// Argmax of a logits product: the CTA's best per stream (from am_v / am_i in shared memory,
// one entry per warp), then the last CTA to finish reduces the CTAs' bests; the lowest index
// wins ties and NaN never wins (candle argmax; stt/model.rs:257).
template <int NB>
__device__ __forceinline__ void argmax_finish(const GemvParams& p, float (*am_v)[NB], int (*am_i)[NB],
                                              bool* last_cta) {
  const int tid = threadIdx.x, nb = p.nb;
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
  if (tid == 0) *last_cta = atomicAdd(p.am_ticket, 1u) == gridDim.x - 1;
  __syncthreads();
  if (*last_cta) {
    __threadfence();
    if (tid < nb && tid < NB) {
      float bv = 0.f;
      int bi = INT_MAX;
      for (int g = 0; g < (int)gridDim.x; g++) {
        const float v = __ldcg(p.am_val + tid * gridDim.x + g);
        const int ix = __ldcg(p.am_idx + tid * gridDim.x + g);
        if (ix != INT_MAX && better(v, ix, bv, bi)) {
          bv = v;
          bi = ix;
        }
      }
      p.tokens[tid] = bi == INT_MAX ? 0u : (uint32_t)bi;
      if (p.pos_advance) p.pos_advance[tid] += 1;
    }
    if (tid == 0) *p.am_ticket = 0u;
  }
}

// ---- f32 / bf16 weights ------------------------------------------------------------------

__host__ __device__ inline int dense_chunks(int wt, int k) { return wt == W_F32 ? k / 4 : k / 8; }

// Accumulates chunks [c0, c0 + 32 U) of R rows (weights already in wv) against the NB input
// records in shared memory.
template <int WT, int NB, int R, int U>
__device__ __forceinline__ void dot_chunks(const uint4 (&wv)[R][U], const GemvParams& p, int c0,
                                           const uint8_t* xsm, int rec, int lane, float (&acc)[R][NB]) {
  const int nch = dense_chunks(WT, p.k);
#pragma unroll
  for (int u = 0; u < U; u++) {
    const int c = c0 + lane + 32 * u;
    if (c >= nch) continue;
    if (WT == W_F32) {
#pragma unroll
      for (int b = 0; b < NB; b++) {
        const float4 x = reinterpret_cast<const float4*>(xsm + (size_t)b * rec)[c];
#pragma unroll
        for (int r = 0; r < R; r++) {
          const float4 w = *reinterpret_cast<const float4*>(&wv[r][u]);
          float a = acc[r][b];
          a = fmaf(w.x, x.x, a);
          a = fmaf(w.y, x.y, a);
          a = fmaf(w.z, x.z, a);
          a = fmaf(w.w, x.w, a);
          acc[r][b] = a;
        }
      }
    } else {
#pragma unroll
      for (int b = 0; b < NB; b++) {
        const float4 x0 = reinterpret_cast<const float4*>(xsm + (size_t)b * rec)[2 * c];
        const float4 x1 = reinterpret_cast<const float4*>(xsm + (size_t)b * rec)[2 * c + 1];
#pragma unroll
        for (int r = 0; r < R; r++) {
          const uint4 w = wv[r][u];
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
  }
}

template <int WT, int NB, int R, int U>
__global__ void __launch_bounds__(kThreads, kCtasPerSm) gemv_kernel(const GemvParams p) {
  extern __shared__ __align__(16) uint8_t xsm[];
  __shared__ float am_v[kWarps][NB];
  __shared__ int am_i[kWarps][NB];
  __shared__ float red[NB][2][kWarps];
  __shared__ float stat[NB][2];
  __shared__ bool last_cta;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nb = p.nb, nch = dense_chunks(WT, p.k), rec = dense_rec_bytes(p.k);
  // Row groups of R rows (R even keeps the RoPE / SwiGLU pairs in one group), split into
  // contiguous ranges per warp.
  const int groups = (p.n + R - 1) / R;
  const int total_w = gridDim.x * kWarps;
  const int gw = blockIdx.x * kWarps + warp;
  const int g0 = (int)((int64_t)gw * groups / total_w), g1 = (int)((int64_t)(gw + 1) * groups / total_w);

  uint4 wv[R][U];
  const uint64_t pol = l2_evict_first();
  // Loads chunks [c0, c0 + 32 U) of group g's rows: every load of the group is in flight at once.
  auto issue = [&](int g, int c0) {
#pragma unroll
    for (int r = 0; r < R; r++)
#pragma unroll
      for (int u = 0; u < U; u++) {
        const int c = c0 + lane + 32 * u;
        const int row = g * R + r;
        const bool on = g < g1 && c < nch && row < p.n;
        wv[r][u] = on ? ldg_weights(p.w + (int64_t)row * p.row_stride + (int64_t)c * 16, pol) : make_uint4(0, 0, 0, 0);
      }
  };
  issue(g0, 0);
  prefetch_share(p);
  NormPre pre;
  norm_preload<kThreads>(p, pre);
  pdl_launch();
  pdl_wait();
  build_dense_records<WT, NB>(p, pre, xsm, rec, red, stat);

  float best_v = 0.f;
  int best_i = INT_MAX;
  for (int g = g0; g < g1; g++) {
    float acc[R][NB];
#pragma unroll
    for (int r = 0; r < R; r++)
#pragma unroll
      for (int b = 0; b < NB; b++) acc[r][b] = 0.f;
    for (int c0 = 0; c0 < nch; c0 += 32 * U) {
      if (c0 > 0) issue(g, c0);
      dot_chunks<WT, NB, R, U>(wv, p, c0, xsm, rec, lane, acc);
    }
    // The next group's first loads fly while this group reduces and runs its epilogue.
    if (g + 1 < g1) issue(g + 1, 0);
#pragma unroll
    for (int r = 0; r < R; r++)
#pragma unroll
      for (int b = 0; b < NB; b++) acc[r][b] = warp_sum(acc[r][b]);
    const int row = g * R;
    if (p.epi == EPI_LOGITS && lane < NB && lane < nb) {
#pragma unroll
      for (int r = 0; r < R; r++) {
        float v = 0.f;
#pragma unroll
        for (int b = 0; b < NB; b++)
          if (b == lane) v = acc[r][b];
        if (row + r < p.n) {
          v = v + (p.bias ? p.bias[row + r] : 0.f);
          if (better(v, row + r, best_v, best_i)) {
            best_v = v;
            best_i = row + r;
          }
        }
      }
    }
    // Lane j < R NB runs the epilogue of (row + j / NB, stream j % NB); all at once.
    {
      float v = 0.f, v_lo = 0.f, v_hi = 0.f;
#pragma unroll
      for (int jj = 0; jj < R * NB; jj++)
        if (lane == jj) {
          v = acc[jj / NB][jj % NB];
          v_lo = acc[(jj / NB) & ~1][jj % NB];
          v_hi = acc[((jj / NB) | 1) % R][jj % NB];
        }
      const int r = lane / NB, b = lane % NB;
      if (lane < R * NB && b < nb && row + r < p.n) epilogue(p, b, row + r, v, v_lo, v_hi);
    }
  }

  if (p.epi == EPI_LOGITS) {
    if (lane < NB) {
      am_v[warp][lane] = best_v;
      am_i[warp][lane] = best_i;
    }
    argmax_finish<NB>(p, am_v, am_i, &last_cta);
  }
}

// ---- Q8_0 / Q4_1 weights -------------------------------------------------------------------
//
// Staged through shared memory with bulk copies: four consecutive rows (a group) are one
// contiguous run of memory, so one cp.async.bulk moves a group. CTA c takes a contiguous
// range of groups; its thread 0 issues the copies of as many groups as its stage area holds
// (for the STT shapes: all of them) before griddepcontrol.wait, so the whole share is in
// flight at once, in the shadow of the previous kernel, with no registers held. After the
// wait and the input records, warp w folds groups w, w + 8, ... from shared memory and,
// when a later group shares the stage it just read, refills it.

// Folds super-block sb of the lane's row (its bytes at `row` in shared memory) into the slot
// accumulators acc[b] (and, for Q4_1, the m * s sums ms[b]) of the NB records: for each block
// j in order, acc = fma(d_w * d_x, sum of the slot's four products, acc).
template <int WT, int NB>
__device__ __forceinline__ void fold_sb(const uint8_t* row, int sb, int nblk, int nsb, int l,
                                        const uint8_t* xsm, int rec, int nb, float (&acc)[NB],
                                        float (&ms)[NB]) {
  constexpr int SBB = WT == W_Q8 ? kQ8SbBytes : kQ4SbBytes;
  const uint8_t* sp = row + sb * SBB;
  uint4 wa, wb;
  float dw[kSbBlocks], mw[kSbBlocks];
  if (WT == W_Q8) {
    wa = *reinterpret_cast<const uint4*>(sp + 16 * l);
    wb = *reinterpret_cast<const uint4*>(sp + 128 + 16 * l);
    const uint4 sc = *reinterpret_cast<const uint4*>(sp + 256);
    const uint32_t w4[4] = {sc.x, sc.y, sc.z, sc.w};
#pragma unroll
    for (int q = 0; q < 4; q++) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w4[q]));
      dw[2 * q] = f.x;
      dw[2 * q + 1] = f.y;
      mw[2 * q] = mw[2 * q + 1] = 0.f;
    }
  } else {
    wa = *reinterpret_cast<const uint4*>(sp + 32 * (l & 3));
    wb = *reinterpret_cast<const uint4*>(sp + 32 * (l & 3) + 16);
    const uint4 s0 = *reinterpret_cast<const uint4*>(sp + 128);
    const uint4 s1 = *reinterpret_cast<const uint4*>(sp + 144);
    const uint32_t w8[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w8[j]));
      dw[j] = f.x;
      mw[j] = f.y;
    }
  }
  const int sh = (WT == W_Q4 && l >= 4) ? 4 : 0;
  const int nj = min(kSbBlocks, nblk - sb * kSbBlocks);
#pragma unroll
  for (int b = 0; b < NB; b++) {
    if (b >= nb) break;
    const uint8_t* xr = xsm + (size_t)b * rec;
    const uint4 xa = *reinterpret_cast<const uint4*>(xr + sb * 256 + 16 * l);
    const uint4 xb = *reinterpret_cast<const uint4*>(xr + sb * 256 + 128 + 16 * l);
    const float* dx = reinterpret_cast<const float*>(xr + nsb * 256) + sb * kSbBlocks;
    const float4 dx0 = reinterpret_cast<const float4*>(dx)[0], dx1 = reinterpret_cast<const float4*>(dx)[1];
    const float dxs[8] = {dx0.x, dx0.y, dx0.z, dx0.w, dx1.x, dx1.y, dx1.z, dx1.w};
    float sxs[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (WT == W_Q4) {
      const float* sx = dx + nsb * kSbBlocks;
      const float4 s0 = reinterpret_cast<const float4*>(sx)[0], s1 = reinterpret_cast<const float4*>(sx)[1];
      sxs[0] = s0.x; sxs[1] = s0.y; sxs[2] = s0.z; sxs[3] = s0.w;
      sxs[4] = s1.x; sxs[5] = s1.y; sxs[6] = s1.z; sxs[7] = s1.w;
    }
#pragma unroll
    for (int j = 0; j < kSbBlocks; j++) {
      if (j >= nj) break;
      uint32_t wq = j < 4 ? word_of(wa, j) : word_of(wb, j - 4);
      const uint32_t xq = j < 4 ? word_of(xa, j) : word_of(xb, j - 4);
      if (WT == W_Q4) wq = (wq >> sh) & 0x0f0f0f0fu;
      const int si = __dp4a((int)wq, (int)xq, 0);
      const float dd = __fmul_rn(dw[j], dxs[j]);
      acc[b] = fmaf(dd, (float)si, acc[b]);
      if (WT == W_Q4) ms[b] = __fadd_rn(ms[b], __fmul_rn(mw[j], sxs[j]));
    }
  }
}

constexpr int kQMaxStages = 64;      // mbarriers of the stage ring
constexpr int kQHeader = kQMaxStages * 8 + 64;  // barriers + the stages' issue counts
// Shared memory of one CTA of the quantised kernel: header, records, stages.
constexpr size_t kQSmemBudget = 110 * 1024;

__host__ __device__ inline size_t q_records_area(int wtype, int k, int nb) {
  return ((size_t)nb * q_rec_bytes(wtype, k) + 127) / 128 * 128;
}

// At most 80 registers per thread (launch bounds of 3 CTAs per SM; launched 2 per SM): measured
// 0.647 ms per STT-1b q8_0 step against 0.659 ms at 106 registers. A next kernel that fits
// beside two CTAs (the attention after in_proj, at 72 registers) does start early, but its
// copies then queue behind this kernel's on the same SMs: no faster.
template <int WT, int NB>
__global__ void __launch_bounds__(kThreads, 3) qgemv_kernel(const GemvParams p, int nst_max) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ float am_v[kWarps][NB];
  __shared__ int am_i[kWarps][NB];
  __shared__ float red[NB][2][kWarps];
  __shared__ float stat[NB][2];
  __shared__ bool last_cta;
  __shared__ int failed;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int l = lane & 7, r = lane >> 3;
  const int nb = p.nb, nblk = p.k / QBLK, nsb = super_blocks(p.k), rec = q_rec_bytes(WT, p.k);
  const int64_t gbytes = 4 * p.row_stride;
  const int groups = (p.n + 3) / 4;
  const int G0 = (int)((int64_t)blockIdx.x * groups / gridDim.x);
  const int ng = (int)((int64_t)(blockIdx.x + 1) * groups / gridDim.x) - G0;
  // Every group has a stage of its own when they fit (each stage filled once, any warp reads
  // it). Otherwise the stages are reused: W consumer warps, W dividing nst, so that stage
  // st is always read by warp st % W, which waits on its phases one after another (an
  // mbarrier parity wait for a phase two ahead of the barrier would succeed at once).
  const bool ring = ng > nst_max;
  const int nst = !ring ? ng : nst_max >= kWarps ? nst_max / kWarps * kWarps : nst_max;
  const int W = ring ? min(kWarps, nst) : kWarps;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  int* issued = reinterpret_cast<int*>(smem + kQMaxStages * 8);  // copies issued per stage
  uint8_t* xsm = smem + kQHeader;
  uint8_t* stg = xsm + q_records_area(WT, p.k, NB);

  // Group G0 + i into stage i % nst (the failure drill withholds CTA 0's first copy).
  const bool withhold = p.test_withhold && blockIdx.x == 0;
  const uint32_t limit = p.wait_limit ? p.wait_limit : kWaitLimit;
  // The weights are read once per step: their L2 lines go first.
  const uint64_t pol = l2_evict_first();
  auto copy_group = [&](int i) {
    if (withhold && i == 0) return;
    const int g = G0 + i, st = i % nst;
    const uint32_t bytes = (uint32_t)(min(4, p.n - 4 * g) * p.row_stride);
    mbar_expect_tx(&full[st], bytes);
    bulk_g2s_hint(stg + (size_t)st * gbytes, p.w + (int64_t)g * gbytes, bytes, &full[st], pol);
    issued[st]++;
  };
  if (tid == 0) {
    failed = 0;
    for (int st = 0; st < nst; st++) {
      mbar_init(&full[st], 1);
      issued[st] = 0;
    }
    fence_mbar_init();
    for (int i = 0; i < nst; i++) copy_group(i);
  }
  prefetch_share(p);
  NormPre pre;
  norm_preload<kThreads>(p, pre);
  __syncthreads();
  pdl_launch();
  pdl_wait();
  build_q_records<WT, NB>(p, pre, xsm, rec, red, stat);

  float best_v = 0.f;
  int best_i = INT_MAX;
  for (int i = warp; warp < W && i < ng; i += W) {
    const int st = i % nst;
    if (failed || !mbar_wait(&full[st], (uint32_t)(i / nst) & 1u, limit)) {
      if (lane == 0) {
        if (p.err) atomicExch(p.err, 2);
        failed = 1;
      }
      break;
    }
    const int g = G0 + i;
    const uint8_t* rowp = stg + (size_t)st * gbytes + (size_t)r * p.row_stride;
    float acc[NB], ms[NB];
#pragma unroll
    for (int b = 0; b < NB; b++) acc[b] = ms[b] = 0.f;
#pragma unroll 4
    for (int sb = 0; sb < nsb; sb++) fold_sb<WT, NB>(rowp, sb, nblk, nsb, l, xsm, rec, nb, acc, ms);
    // The stage is read: refill it with the group that comes nst later, which this warp reads
    // next (the refill is ordered after this warp's reads of the stage).
    __syncwarp();
    if (lane == 0 && i + nst < ng) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      copy_group(i + nst);
    }
    // The 8 slot lanes of each row meet in the reference's sum tree
    // ((l0 + l4) + (l2 + l6)) + ((l1 + l5) + (l3 + l7)) (+ the m * s sum for Q4_1); every lane
    // of the row ends with the total.
    float res[NB];
#pragma unroll
    for (int b = 0; b < NB; b++) {
      float t = acc[b];
      t = t + __shfl_xor_sync(0xffffffffu, t, 4);
      t = t + __shfl_xor_sync(0xffffffffu, t, 2);
      t = t + __shfl_xor_sync(0xffffffffu, t, 1);
      if (WT == W_Q4) t = t + ms[b];
      res[b] = t;
    }
    // Lane (r, l) runs the epilogue of row 4 g + r for stream l; rows 2i, 2i+1 pair up.
    float v = 0.f;
#pragma unroll
    for (int b = 0; b < NB; b++)
      if (b == l) v = res[b];
    const float vo = __shfl_xor_sync(0xffffffffu, v, 8);
    const int row = g * 4 + r;
    const bool mine = l < nb && row < p.n;
    if (p.epi == EPI_LOGITS && mine) {
      const float vb = v + (p.bias ? p.bias[row] : 0.f);
      if (better(vb, row, best_v, best_i)) {
        best_v = vb;
        best_i = row;
      }
    }
    if (mine) epilogue(p, l, row, v, (r & 1) ? vo : v, (r & 1) ? v : vo);
  }
  // A wait that ran out: every copy issued must still land before the CTA exits (bounded).
  __syncthreads();
  if (failed && tid == 0)
    for (int st = 0; st < nst; st++)
      if (issued[st] > 0) mbar_wait(&full[st], (uint32_t)(issued[st] - 1) & 1u);

  if (p.epi == EPI_LOGITS) {
    // The 4 rows' lanes of each stream meet first, then the warps.
#pragma unroll
    for (int off = 8; off < 32; off <<= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best_v, off);
      const int oi = __shfl_xor_sync(0xffffffffu, best_i, off);
      if (oi != INT_MAX && better(ov, oi, best_v, best_i)) {
        best_v = ov;
        best_i = oi;
      }
    }
    if (lane < NB) {
      am_v[warp][lane] = best_v;
      am_i[warp][lane] = best_i;
    }
    argmax_finish<NB>(p, am_v, am_i, &last_cta);
  }
}

// ---- f32 / bf16 weights in the reference's dot order (reference-order states) -----------
//
// kernels::dot (nn/kernels/mod.rs:68-91), which kernels::matvec runs per row: 16 FMA lanes,
// lane i over elements i, i + 16, ... in order, then the pairwise tree (lane i += lane i + 8,
// + 4, + 2, + 1). Lane (r, j) of a warp -- row r of a group of 8, quarter j -- holds dot
// lanes 4j..4j+3 of its row; xor-shuffles 2 and 1 are the tree's first two levels, the
// last two run in the lane.
template <int WT, int NB>
__global__ void __launch_bounds__(kThreads, kCtasPerSm) rgemv_kernel(const GemvParams p) {
  extern __shared__ __align__(16) uint8_t xsm[];
  __shared__ float am_v[kWarps][NB];
  __shared__ int am_i[kWarps][NB];
  __shared__ float red[NB][2][kWarps];
  __shared__ float stat[NB][2];
  __shared__ bool last_cta;
  constexpr int U = 8;  // chunks of 16 values in flight per lane
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, r = lane >> 2, j = lane & 3;
  const int nb = p.nb, nch = p.k / 16, rec = dense_rec_bytes(p.k);
  const int groups = (p.n + 7) / 8;
  const int total_w = gridDim.x * kWarps;
  const int gw = blockIdx.x * kWarps + warp;
  const int g0 = (int)((int64_t)gw * groups / total_w), g1 = (int)((int64_t)(gw + 1) * groups / total_w);
  const uint64_t pol = l2_evict_first();
  prefetch_share(p);
  NormPre pre;
  norm_preload<kThreads>(p, pre);
  pdl_launch();
  pdl_wait();
  build_dense_records<WT, NB>(p, pre, xsm, rec, red, stat);

  float best_v[2] = {0.f, 0.f};  // streams j and j + 4
  int best_i[2] = {INT_MAX, INT_MAX};
  for (int g = g0; g < g1; g++) {
    const int row = g * 8 + r;
    const bool on = row < p.n;
    const uint8_t* wrow = p.w + (int64_t)(on ? row : 0) * p.row_stride;
    float acc[NB][4];
#pragma unroll
    for (int b = 0; b < NB; b++)
#pragma unroll
      for (int s = 0; s < 4; s++) acc[b][s] = 0.f;
    for (int c0 = 0; c0 < nch; c0 += U) {
      float w[U][4];
#pragma unroll
      for (int u = 0; u < U; u++) {
        const int c = c0 + u;
        if (WT == W_F32) {
          const uint4 v = on && c < nch ? ldg_weights(wrow + (int64_t)(16 * c + 4 * j) * 4, pol) : make_uint4(0, 0, 0, 0);
          w[u][0] = __uint_as_float(v.x); w[u][1] = __uint_as_float(v.y);
          w[u][2] = __uint_as_float(v.z); w[u][3] = __uint_as_float(v.w);
        } else {
          uint2 v = make_uint2(0, 0);
          if (on && c < nch) v = __ldcs(reinterpret_cast<const uint2*>(wrow + (int64_t)(16 * c + 4 * j) * 2));
          w[u][0] = bf16_lo(v.x); w[u][1] = bf16_hi(v.x); w[u][2] = bf16_lo(v.y); w[u][3] = bf16_hi(v.y);
        }
      }
#pragma unroll
      for (int u = 0; u < U; u++) {
        const int c = c0 + u;
        if (c >= nch) break;
#pragma unroll
        for (int b = 0; b < NB; b++) {
          if (b >= nb) break;
          const float4 x = *reinterpret_cast<const float4*>(xsm + (size_t)b * rec + (16 * c + 4 * j) * 4);
          acc[b][0] = fmaf(x.x, w[u][0], acc[b][0]);
          acc[b][1] = fmaf(x.y, w[u][1], acc[b][1]);
          acc[b][2] = fmaf(x.z, w[u][2], acc[b][2]);
          acc[b][3] = fmaf(x.w, w[u][3], acc[b][3]);
        }
      }
    }
    float res[NB];
#pragma unroll
    for (int b = 0; b < NB; b++) {
      float a[4];
#pragma unroll
      for (int s = 0; s < 4; s++) {
        a[s] = acc[b][s];
        a[s] = a[s] + __shfl_xor_sync(0xffffffffu, a[s], 2);  // lane i += lane i + 8
        a[s] = a[s] + __shfl_xor_sync(0xffffffffu, a[s], 1);  // lane i += lane i + 4
      }
      res[b] = ((a[0] + a[2]) + (a[1] + a[3])) + 0.0f;  // + 2, + 1, then the (empty) tail
    }
    // Lane (r, j) runs the epilogue of row 8 g + r for streams j and j + 4; rows 2i, 2i+1 pair up.
#pragma unroll
    for (int h = 0; h < 2; h++) {
      const int sb = j + 4 * h;
      float v = 0.f;
#pragma unroll
      for (int b = 0; b < NB; b++)
        if (b == sb) v = res[b];
      const float vo = __shfl_xor_sync(0xffffffffu, v, 4);
      const bool mine = sb < nb && sb < NB && on;
      if (p.epi == EPI_LOGITS && mine) {
        const float vb = v + (p.bias ? p.bias[row] : 0.f);
        if (better(vb, row, best_v[h], best_i[h])) {
          best_v[h] = vb;
          best_i[h] = row;
        }
      }
      if (mine) epilogue(p, sb, row, v, (r & 1) ? vo : v, (r & 1) ? v : vo);
    }
  }
  if (p.epi == EPI_LOGITS) {
    // The 8 rows' lanes of each stream meet; lanes 0-3 then hold streams j and j + 4.
#pragma unroll
    for (int h = 0; h < 2; h++) {
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best_v[h], off);
        const int oi = __shfl_xor_sync(0xffffffffu, best_i[h], off);
        if (oi != INT_MAX && better(ov, oi, best_v[h], best_i[h])) {
          best_v[h] = ov;
          best_i[h] = oi;
        }
      }
      if (lane < 4 && j + 4 * h < NB) {
        am_v[warp][j + 4 * h] = best_v[h];
        am_i[warp][j + 4 * h] = best_i[h];
      }
    }
    argmax_finish<NB>(p, am_v, am_i, &last_cta);
  }
}

constexpr size_t kMaxSmem = 96 * 1024;  // input records; 2 CTAs per SM

// Rows per warp group of the dense kernel: the fewest (of 1, 2, 4) whose groups fit in one
// wave of warps, so the whole matrix is in flight at once; 2 at least when the epilogue pairs
// rows.
int pick_r(const GemvParams& p) {
  const int warps = kGrid * kWarps;
  const bool pairs = p.epi == EPI_QKV_ROPE || p.epi == EPI_SWIGLU;
  if (!pairs && p.n <= warps) return 1;
  if (p.n <= 2 * warps) return 2;
  return 4;
}

// Loads per row in flight per lane for the dense kernel: 8 (f32), else 4, or 2 for
// four-row groups.
template <int WT, int R>
constexpr int kU = WT == W_F32 ? 8 : R == 4 ? 2 : 4;
// 16 streams per launch (f32 weights only, see max_nb): 4 loads per row in flight, so that
// the weights in flight and the 16 streams' accumulators fit the registers.
template <int WT, int NB, int R>
constexpr int kUn = NB == 16 ? 4 : kU<WT, R>;
// CTAs of a quantised product: one group at least each, at most kGrid.
constexpr int kQGrid = kGrid;

int rec_bytes(const GemvParams& p) {
  return (p.wtype == W_Q8 || p.wtype == W_Q4) ? q_rec_bytes(p.wtype, p.k) : dense_rec_bytes(p.k);
}

template <class K>
void launch_k(K kernel, const GemvParams& p, int grid, size_t smem, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, kernel, p);
}

template <int WT, int NB, int R>
void launch_r(const GemvParams& p, cudaStream_t s) {
  const int groups = (p.n + R - 1) / R;
  const int grid = std::min((groups + kWarps - 1) / kWarps, kGrid);
  launch_k(gemv_kernel<WT, NB, R, kUn<WT, NB, R>>, p, grid, (size_t)NB * rec_bytes(p), s);
}

// Four-row groups only where their registers fit without spilling (one stream, bf16).
template <int WT, int NB>
constexpr bool kAllowR4 = NB == 1 && WT == W_BF16;

template <int WT, int NB>
void launch_t(const GemvParams& p, cudaStream_t s) {
  if constexpr (WT == W_Q8 || WT == W_Q4) {
    const int groups = (p.n + 3) / 4;
    const int grid = std::min(groups, kQGrid);
    const size_t gbytes = 4 * (size_t)p.row_stride;
    const int per_cta = (groups + grid - 1) / grid;  // the most groups a CTA takes
    const size_t fixed = kQHeader + q_records_area(WT, p.k, NB);
    const int nst = (int)std::min<size_t>({(size_t)per_cta, (size_t)kQMaxStages, (kQSmemBudget - fixed) / gbytes});
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = fixed + (size_t)nst * gbytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, qgemv_kernel<WT, NB>, p, nst);
    return;
  } else {
  if (p.ref_order) {
    const int groups = (p.n + 7) / 8;
    const int grid = std::min((groups + kWarps - 1) / kWarps, kGrid);
    launch_k(rgemv_kernel<WT, NB>, p, grid, (size_t)NB * rec_bytes(p), s);
    return;
  }
  int r = pick_r(p);
  if (!kAllowR4<WT, NB> && r == 4) r = 2;
  if constexpr (kAllowR4<WT, NB>) {
    if (r == 4) {
      launch_r<WT, NB, 4>(p, s);
      return;
    }
  }
  if (r == 2)
    launch_r<WT, NB, 2>(p, s);
  else
    launch_r<WT, NB, 1>(p, s);
  }
}

template <int WT, int NB>
void set_attrs_nb() {
  if constexpr (WT == W_Q8 || WT == W_Q4) {
    cudaFuncSetAttribute(qgemv_kernel<WT, NB>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kQSmemBudget);
    // The whole carveout as shared memory (the attention kernel asks for the same), so that
    // consecutive kernels can share an SM without reconfiguring it.
    cudaFuncSetAttribute(qgemv_kernel<WT, NB>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
  } else {
    cudaFuncSetAttribute(rgemv_kernel<WT, NB>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem);
    cudaFuncSetAttribute(gemv_kernel<WT, NB, 1, kU<WT, 1>>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem);
    cudaFuncSetAttribute(gemv_kernel<WT, NB, 2, kU<WT, 2>>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem);
    if constexpr (kAllowR4<WT, NB>)
      cudaFuncSetAttribute(gemv_kernel<WT, NB, 4, kU<WT, 4>>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem);
  }
}

template <int WT>
void set_attrs() {
  set_attrs_nb<WT, 1>();
  set_attrs_nb<WT, 2>();
  set_attrs_nb<WT, 4>();
  set_attrs_nb<WT, 8>();
  if constexpr (WT == W_F32) {
    cudaFuncSetAttribute(gemv_kernel<WT, 16, 1, kUn<WT, 16, 1>>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem);
    cudaFuncSetAttribute(gemv_kernel<WT, 16, 2, kUn<WT, 16, 2>>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem);
  }
}

// 9 to 16 streams of an f32 product in one launch (max_nb decides when).
void launch_t16(const GemvParams& p, cudaStream_t s) {
  if (pick_r(p) == 1)
    launch_r<W_F32, 16, 1>(p, s);
  else
    launch_r<W_F32, 16, 2>(p, s);
}

// Streams per launch: the widest template whose input records fit (with, for the quantised
// kernel, at least one staged group of rows). f32 weights with many streams (Mimi's
// transformers, f32 models) take 16 per launch where the records fit, halving the passes over
// the weights; not for the logits head (its argmax scratch holds 8 streams per launch) nor in
// reference order.
int max_nb(const GemvParams& p) {
  if (p.wtype == W_F32 && p.nb > 8 && p.epi != EPI_LOGITS && !p.ref_order &&
      (size_t)16 * rec_bytes(p) <= kMaxSmem)
    return 16;
  const bool q = p.wtype == W_Q8 || p.wtype == W_Q4;
  for (int nb : {8, 4, 2}) {
    if (q ? kQHeader + q_records_area(p.wtype, p.k, nb) + 4 * (size_t)p.row_stride <= kQSmemBudget
          : (size_t)nb * rec_bytes(p) <= kMaxSmem)
      return nb;
  }
  return 1;
}

template <int WT>
void launch_w(const GemvParams& p0, cudaStream_t s) {
  const int cap = max_nb(p0);
  for (int b0 = 0; b0 < p0.nb; b0 += cap) {
    GemvParams p = p0;
    p.nb = p0.nb - b0 < cap ? p0.nb - b0 : cap;
    p.x = p0.x + b0 * p0.x_stride;
    if (p0.out) p.out = p0.out + b0 * p0.out_stride;
    if (p0.pos) p.pos = p0.pos + b0;
    if (p0.tokens) p.tokens = p0.tokens + b0;
    if (p0.pos_advance) p.pos_advance = p0.pos_advance + b0;
    if (p0.k_ring) {
      const size_t el = p0.kv_bf16 ? 2 : 4;
      p.k_ring = static_cast<uint8_t*>(p0.k_ring) + b0 * p0.ring_stream_stride * el;
      p.v_ring = static_cast<uint8_t*>(p0.v_ring) + b0 * p0.ring_stream_stride * el;
    }
    if (b0 > 0)
      for (auto& r : p.pf) r = PrefetchRange{};
    if constexpr (WT == W_F32) {
      if (p.nb > 8) {
        launch_t16(p, s);
        continue;
      }
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

int gemv_launches(const GemvParams& p) {
  const int cap = max_nb(p);
  return (p.nb + cap - 1) / cap;
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
