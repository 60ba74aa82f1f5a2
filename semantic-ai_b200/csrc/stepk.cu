// stepk.cu — the whole STT step of one stream as one persistent kernel.
//
// At batch 1 the step reads ~0.9 GB of weights (q8_0) plus the KV window, and nothing else
// of size: it is HBM-bound, and a chain of ~80 dependent kernels loses the bandwidth at every
// link (launch, ramp-up, input prologue, tail). Here one CTA per SM runs the whole step:
//
//  * a producer warp streams this CTA's share of every phase's bytes -- its rows of each
//    weight matrix, its key range of each layer's KV window -- with 1-D bulk copies
//    (cp.async.bulk) into a ring of shared-memory slots. Weights and past KV do not depend on
//    the step's activations, so the producer never waits for data: only for a free slot. It
//    runs ahead of the consumers by the whole ring (~160 KB per SM, ~24 MB across the GPU),
//    through the phase boundaries;
//  * eight consumer warps run the phases in order. A phase starts when every CTA has
//    finished the previous one (a counter per phase in global memory, acquire / release),
//    builds its input record in shared memory (the layer norm and the weight format's
//    activation conversion, as the matrix-vector kernel does), then consumes its slots: one
//    warp per row (row pairs for RoPE / SwiGLU), and the same fused epilogues.
//
// Phases: embedding sum; per layer in_proj (+RoPE, KV-ring write), attention, out_proj
// (+residual), linear_in (+SwiGLU / GELU), linear_out (+residual); the head (logits, argmax,
// position advance). Attention splits each head's keys over `splits` CTAs; each writes a
// partial softmax (max, sum, weighted values) and the last CTA of the head (a counter per
// layer and head) merges them into the attention output.
//
// The launch is cooperative (every CTA resident), and every wait is bounded: one that runs
// out sets the error flag and the CTA carries on, so the grid always finishes.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "common.cuh"
#include "gemv_common.cuh"
#include "kernels.cuh"
#include "sm100.cuh"

namespace svl {
namespace {

constexpr int kCons = 384;               // consumer threads: 12 warps
constexpr int kConsWarps = kCons / 32;
constexpr int kSThreads = kCons + 32;    // plus the producer warp
constexpr int kMaxSlots = 16;
constexpr int kMaxKeysPerPart = 1024;

__device__ __forceinline__ void cons_sync() { asm volatile("bar.sync 1, 384;" ::: "memory"); }

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Any failure recorded for this launch (a wait that ran out, a bad token): later waits give
// up at once, so a failed step still ends promptly.
__device__ __forceinline__ bool failed(const int* err) {
  return *reinterpret_cast<const volatile int*>(err) != 0;
}

// Bounded wait until *c >= target.
__device__ bool wait_count(const unsigned* c, unsigned target, const int* err) {
  for (uint32_t i = 0; i < kWaitLimit; i++) {
    if (ld_acquire(c) >= target) return true;
    if ((i & 255) == 255 && failed(err)) return false;
    __nanosleep(32);
  }
  return false;
}

// Bounded wait on an mbarrier phase, giving up once the launch has failed.
__device__ bool wait_bar(uint64_t* bar, uint32_t parity, const int* err) {
  for (uint32_t i = 0; i < kWaitLimit; i++) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255) == 255 && failed(err)) return false;
  }
  return false;
}

__device__ __forceinline__ bool pair_epi(int epi) { return epi == EPI_QKV_ROPE || epi == EPI_SWIGLU; }

// Rows [r0, r1) of a product for CTA c of G (whole row pairs for the pair epilogues).
__device__ __forceinline__ void rows_of(const GemvParams& g, int c, int G, int& r0, int& r1) {
  if (pair_epi(g.epi)) {
    const int np = g.n / 2;
    r0 = 2 * (int)((int64_t)np * c / G);
    r1 = 2 * (int)((int64_t)np * (c + 1) / G);
  } else {
    r0 = (int)((int64_t)g.n * c / G);
    r1 = (int)((int64_t)g.n * (c + 1) / G);
  }
}
__device__ __forceinline__ int rows_per_slot(const GemvParams& g, int slot_bytes) {
  int r = slot_bytes / (int)g.row_stride;
  if (pair_epi(g.epi)) r &= ~1;
  return r < 1 ? 1 : r;
}

// Keys of attention unit `part` of a head: positions [j0, j1) of the visible window of the
// newest position pos (the newest key itself is read from global memory: this step wrote it).
__device__ __forceinline__ void keys_of(const AttnParams& a, int pos, int part, int splits, int& j0,
                                        int& j1) {
  const int count = a.window > 0 ? min(pos + 1, a.window) : pos + 1;
  const int first = pos + 1 - count;
  j0 = first + (int)((int64_t)count * part / splits);
  j1 = first + (int)((int64_t)count * (part + 1) / splits);
}
__device__ __forceinline__ int ring_slot(const AttnParams& a, int j) {
  return a.window > 0 ? j % a.ring_cap : j;
}

// The lane's share of one row's dot product against the input record (one stream): 16-byte
// chunks c = lane + 32 i of the row, as the matrix-vector kernel's dot_chunks.
// Q8_0: lane l takes whole 32-element blocks l, l + 32, ...: 32 weight bytes against the
// record's 32 activation bytes (an exact integer dot), scaled by both f16-valued scales.
__device__ __forceinline__ float q8_block(const uint8_t* wrow, const uint8_t* rec, int k, int b) {
  // Lanes of odd groups of four read the block's second half first: with 32-byte strides
  // between lanes, this spreads a warp's 16-byte loads over all banks.
  const int h = (b >> 2) & 1;
  const uint4 w0 = *reinterpret_cast<const uint4*>(wrow + (size_t)b * 32 + 16 * h);
  const uint4 w1 = *reinterpret_cast<const uint4*>(wrow + (size_t)b * 32 + 16 * (1 - h));
  const int4 x0 = reinterpret_cast<const int4*>(rec)[2 * b + h];
  const int4 x1 = reinterpret_cast<const int4*>(rec)[2 * b + 1 - h];
  int s = __dp4a((int)w0.x, x0.x, 0);
  s = __dp4a((int)w0.y, x0.y, s);
  s = __dp4a((int)w0.z, x0.z, s);
  s = __dp4a((int)w0.w, x0.w, s);
  s = __dp4a((int)w1.x, x1.x, s);
  s = __dp4a((int)w1.y, x1.y, s);
  s = __dp4a((int)w1.z, x1.z, s);
  s = __dp4a((int)w1.w, x1.w, s);
  const float dw = __half2float(reinterpret_cast<const __half*>(wrow + k)[b]);
  const float dx = reinterpret_cast<const float*>(rec + k)[b];
  return (dw * dx) * (float)s;
}
__device__ __forceinline__ float q8_dot(const uint8_t* wrow, const uint8_t* rec, int k, int lane) {
  float acc = 0.f;
  for (int b = lane; b < k / QBLK; b += 32) acc += q8_block(wrow, rec, k, b);
  return acc;
}

template <int WT>
__device__ __forceinline__ float row_dot(const uint8_t* wrow, const uint8_t* rec, int k, int lane) {
  if (WT == W_Q8) return q8_dot(wrow, rec, k, lane);
  const int nch = chunks_per_row(WT, k);
  float acc = 0.f;
  for (int c0 = 0; c0 < nch; c0 += 32) {
    const int c = c0 + lane;
    const bool valid = c < nch;
    const uint4 w = valid ? *reinterpret_cast<const uint4*>(wrow + (size_t)c * 16) : make_uint4(0, 0, 0, 0);
    if (WT == W_F32) {
      if (valid) {
        const float4 x = reinterpret_cast<const float4*>(rec)[c];
        const float4 wf = *reinterpret_cast<const float4*>(&w);
        acc = fmaf(wf.x, x.x, acc);
        acc = fmaf(wf.y, x.y, acc);
        acc = fmaf(wf.z, x.z, acc);
        acc = fmaf(wf.w, x.w, acc);
      }
    } else if (WT == W_BF16) {
      if (valid) {
        const float4 x0 = reinterpret_cast<const float4*>(rec)[2 * c];
        const float4 x1 = reinterpret_cast<const float4*>(rec)[2 * c + 1];
        acc = fmaf(bf16_lo(w.x), x0.x, acc);
        acc = fmaf(bf16_hi(w.x), x0.y, acc);
        acc = fmaf(bf16_lo(w.y), x0.z, acc);
        acc = fmaf(bf16_hi(w.y), x0.w, acc);
        acc = fmaf(bf16_lo(w.z), x1.x, acc);
        acc = fmaf(bf16_hi(w.z), x1.y, acc);
        acc = fmaf(bf16_lo(w.w), x1.z, acc);
        acc = fmaf(bf16_hi(w.w), x1.w, acc);
      }
    } else if (WT == W_Q8) {
      // (not reached: Q8 rows use q8_dot below)
    } else {  // W_Q4: chunk c is block c, 16 bytes of nibbles (ggml Q4_1 order).
      if (valid) {
        const int nblk = k / QBLK;
        const float2 dm = __half22float2(reinterpret_cast<const __half2*>(wrow + k / 2)[c]);
        const int4* xb = reinterpret_cast<const int4*>(rec + (size_t)c * QBLK);
        const int4 lo = xb[0], hi = xb[1];
        const float dx = reinterpret_cast<const float*>(rec + k)[c];
        const float sx = reinterpret_cast<const float*>(rec + k)[nblk + c];
        int s = __dp4a((int)(w.x & 0x0f0f0f0fu), lo.x, 0);
        s = __dp4a((int)(w.y & 0x0f0f0f0fu), lo.y, s);
        s = __dp4a((int)(w.z & 0x0f0f0f0fu), lo.z, s);
        s = __dp4a((int)(w.w & 0x0f0f0f0fu), lo.w, s);
        s = __dp4a((int)((w.x >> 4) & 0x0f0f0f0fu), hi.x, s);
        s = __dp4a((int)((w.y >> 4) & 0x0f0f0f0fu), hi.y, s);
        s = __dp4a((int)((w.z >> 4) & 0x0f0f0f0fu), hi.z, s);
        s = __dp4a((int)((w.w >> 4) & 0x0f0f0f0fu), hi.w, s);
        acc += (dm.x * dx) * (float)s + dm.y * sx;
      }
    }
  }
  return acc;
}

struct Smem {
  StepPhase cur;                   // the running phase's parameters (read often, off global memory)
  uint64_t full[kMaxSlots], empty[kMaxSlots];
  float red[2][kConsWarps];
  float stat[2];
  float best_v[kConsWarps];
  int best_i[kConsWarps];
  float sc[kMaxKeysPerPart];       // attention scores / weights of this CTA's keys
  float2 rope[64];                 // (cos, sin)(pos * inv_freq[i]) of the running in_proj phase
  float acc[kConsWarps][128];      // attention: per-warp weighted value sums (head_dim <= 128)
  int flag;
};

// Per-phase ring bookkeeping shared by producer and consumers: slot it % nslots, fill round
// it / nslots.
struct Ring {
  uint8_t* base;
  int slot_bytes, nslots;
  __device__ uint8_t* slot(uint32_t it) const { return base + (size_t)(it % nslots) * slot_bytes; }
};

// ---- producer --------------------------------------------------------------------------

__device__ bool produce(Smem& sm, const Ring& ring, uint32_t& it, const void* src, uint32_t bytes,
                        int* err) {
  const uint32_t s = it % ring.nslots;
  if (it >= (uint32_t)ring.nslots && !wait_bar(&sm.empty[s], ((it / ring.nslots) - 1) & 1, err)) {
    atomicExch(err, 3);
    return false;
  }
  mbar_expect_tx(&sm.full[s], bytes);
  bulk_g2s(ring.slot(it), src, bytes, &sm.full[s]);
  it++;
  return true;
}

__device__ void producer(const StepProgram& pg, Smem& sm, const Ring& ring) {
  const int G = gridDim.x, cta = blockIdx.x;
  uint32_t it = 0;
  for (int p = 0; p < pg.nph; p++) {
    const StepPhase& P = pg.ph[p];
    if (P.type == PH_GEMV) {
      const GemvParams& g = P.g;
      int r0, r1;
      rows_of(g, cta, G, r0, r1);
      const int rps = rows_per_slot(g, ring.slot_bytes);
      for (int r = r0; r < r1; r += rps) {
        const int nr = min(rps, r1 - r);
        if (!produce(sm, ring, it, g.w + (int64_t)r * g.row_stride, (uint32_t)(nr * g.row_stride), pg.err)) return;
      }
    } else if (P.type == PH_ATTN) {
      const AttnParams& a = P.a;
      const int units = a.heads * pg.splits;
      if (cta >= units) continue;
      const int h = cta / pg.splits, part = cta % pg.splits;
      const int pos = a.pos[0];
      int j0, j1;
      keys_of(a, pos, part, pg.splits, j0, j1);
      if (j1 > pos) j1 = pos;  // the newest key comes from global memory
      const int kvh = h / (a.heads / a.kv_heads);
      const int rowb = a.head_dim * (a.kv_bf16 ? 2 : 4);
      const int kps = ring.slot_bytes / rowb;
      for (int t = 0; t < 2; t++) {
        const uint8_t* base = static_cast<const uint8_t*>(t == 0 ? a.k_ring : a.v_ring) +
                              (int64_t)kvh * a.ring_cap * rowb;
        for (int j = j0; j < j1;) {
          // A run of consecutive ring slots, at most one slot of the shared-memory ring.
          const int sl = ring_slot(a, j);
          int n = min(j1 - j, kps);
          if (a.window > 0) n = min(n, a.ring_cap - sl);
          if (!produce(sm, ring, it, base + (int64_t)sl * rowb, (uint32_t)(n * rowb), pg.err)) return;
          j += n;
        }
      }
    }
  }
}

// ---- consumers -------------------------------------------------------------------------

__device__ __forceinline__ bool take(Smem& sm, const Ring& ring, uint32_t it, int* err) {
  if (!wait_bar(&sm.full[it % ring.nslots], (it / ring.nslots) & 1, err)) {
    atomicExch(err, 3);
    return false;
  }
  return true;
}
__device__ __forceinline__ void give(Smem& sm, const Ring& ring, uint32_t it, int lane) {
  __syncwarp();
  if (lane == 0) mbar_arrive(&sm.empty[it % ring.nslots]);
}

// Both rows of a pair in one pass over the chunks, so their dependency chains interleave.
template <int WT>
__device__ __forceinline__ void row_dot2(const uint8_t* w0, const uint8_t* w1, const uint8_t* rec, int k,
                                         int lane, float& a0, float& a1) {
  if (WT == W_Q8) {
    float acc0 = 0.f, acc1 = 0.f;
    for (int b = lane; b < k / QBLK; b += 32) {
      acc0 += q8_block(w0, rec, k, b);
      acc1 += q8_block(w1, rec, k, b);
    }
    a0 = acc0;
    a1 = acc1;
  } else {
    a0 = row_dot<WT>(w0, rec, k, lane);
    a1 = row_dot<WT>(w1, rec, k, lane);
  }
}

// One product phase: this CTA's rows [r0, r1) arrive slot by slot; warp w takes items (rows,
// or row pairs for RoPE / SwiGLU) w, w + 8, ... of the phase, so all warps work on different
// slots at once. Every warp arrives once on each slot's `empty` barrier (those with no item
// in a slot without waiting for it).
template <int WT>
__device__ void gemv_phase(const StepProgram& pg, const GemvParams& g, Smem& sm, const Ring& ring,
                           uint8_t* rec, uint32_t& it) {
  const int G = gridDim.x, cta = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int recb = rec_bytes_of(WT, g.k);
  build_records<WT, 1, kCons>(g, rec, recb, sm.red, sm.stat, [] { cons_sync(); });
  int r0, r1;
  rows_of(g, cta, G, r0, r1);
  const int rps = rows_per_slot(g, ring.slot_bytes);
  const bool pairs = pair_epi(g.epi);
  const int per_item = pairs ? 2 : 1;
  float best_v = 0.f;
  int best_i = INT_MAX;
  int item = warp;  // next item of this warp (phase-relative, in rows / per_item)
  const int n_items = (r1 - r0) / per_item;
  for (int r = r0; r < r1; r += rps, it++) {
    const int nr = min(rps, r1 - r);
    const int i_end = (r - r0 + nr) / per_item;  // items [.., i_end) lie in this slot
    if (item < i_end && item < n_items) {
      const bool ok = take(sm, ring, it, pg.err);
      const uint8_t* slot = ring.slot(it);
      for (; item < i_end; item += kConsWarps) {
        const int row = r0 + item * per_item;
        const uint8_t* wr = slot + (size_t)(row - r) * g.row_stride;
        if (pairs) {
          float a0 = 0.f, a1 = 0.f;
          if (ok) row_dot2<WT>(wr, wr + g.row_stride, rec, g.k, lane, a0, a1);
          const float v0 = warp_sum(a0), v1 = warp_sum(a1);
          if (g.epi == EPI_QKV_ROPE) {
            // rope_i (nn/transformer.rs:339-340) with the phase's (cos, sin) table; q to its
            // buffer, k and v into the KV ring at the position's slot.
            if (lane < 2) {
              const int hd = g.head_dim;
              const bool is_v = row >= g.q_dim + g.kv_dim;
              float val;
              int rr;
              if (!is_v) {
                const int dim = row % hd;
                const float2 cs = sm.rope[dim >> 1];
                val = lane == 0 ? v0 * cs.x - v1 * cs.y : v0 * cs.y + v1 * cs.x;
                rr = row < g.q_dim ? row : row - g.q_dim;
              } else {
                val = lane == 0 ? v0 : v1;
                rr = row - g.q_dim - g.kv_dim;
              }
              const int rw = row + lane;
              if (rw < g.q_dim) {
                g.out[rw] = val;
              } else {
                const int r2 = rr + lane, kh = r2 / hd, dim = r2 % hd;
                const int pos = g.pos[0];
                const int slot = g.windowed ? pos % g.ring_cap : pos;
                const int64_t off = ((int64_t)kh * g.ring_cap + slot) * hd + dim;
                void* ringp = is_v ? g.v_ring : g.k_ring;
                if (g.kv_bf16)
                  reinterpret_cast<__nv_bfloat16*>(ringp)[off] = __float2bfloat16_rn(val);
                else
                  reinterpret_cast<float*>(ringp)[off] = val;
              }
            }
          } else if (lane == 0) {
            epilogue(g, 0, row, v0, v0, v1);
          } else if (lane == 1) {
            epilogue(g, 0, row + 1, v1, v0, v1);
          }
        } else {
          // The residual's old value is loaded before the dot, so its latency overlaps it.
          const bool resid = g.epi == EPI_RESIDUAL;
          const float xold = (resid && lane == 0) ? __ldcg(g.out + row) : 0.f;
          const float v = ok ? warp_sum(row_dot<WT>(wr, rec, g.k, lane)) : 0.f;
          if (lane == 0 && resid) {
            float u = g.bias ? v + g.bias[row] : v;
            if (g.ls) u = u * g.ls[row];
            g.out[row] = xold + u;
          } else if (lane == 0) {
            epilogue(g, 0, row, v, v, v);
            if (g.epi == EPI_LOGITS) {
              const float lv = v + (g.bias ? g.bias[row] : 0.f);
              if (better(lv, row, best_v, best_i)) {
                best_v = lv;
                best_i = row;
              }
            }
          }
        }
      }
    }
    give(sm, ring, it, lane);
  }
  if (g.epi == EPI_LOGITS) {
    // Argmax: CTA best, then the last CTA of the grid reduces the CTA bests (lowest row on ties).
    if (lane == 0) {
      sm.best_v[warp] = best_v;
      sm.best_i[warp] = best_i;
    }
    cons_sync();
    if (tid == 0) {
      float bv = 0.f;
      int bi = INT_MAX;
      for (int w = 0; w < kConsWarps; w++)
        if (sm.best_i[w] != INT_MAX && better(sm.best_v[w], sm.best_i[w], bv, bi)) {
          bv = sm.best_v[w];
          bi = sm.best_i[w];
        }
      g.am_val[cta] = bv;
      g.am_idx[cta] = bi;
      __threadfence();
      sm.flag = atomicAdd(g.am_ticket, 1u) == (unsigned)G - 1;
    }
    cons_sync();
    if (sm.flag && tid == 0) {
      __threadfence();
      float bv = 0.f;
      int bi = INT_MAX;
      for (int c = 0; c < G; c++) {
        const float v = __ldcg(g.am_val + c);
        const int ix = __ldcg(g.am_idx + c);
        if (ix != INT_MAX && better(v, ix, bv, bi)) {
          bv = v;
          bi = ix;
        }
      }
      g.tokens[0] = bi == INT_MAX ? 0u : (uint32_t)bi;
      if (g.pos_advance) g.pos_advance[0] += 1;
      *g.am_ticket = 0u;
    }
  }
}

__device__ void attn_phase(const StepProgram& pg, const AttnParams& a, int layer, Smem& sm,
                           const Ring& ring, uint32_t& it) {
  const int cta = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int units = a.heads * pg.splits;
  if (cta >= units) return;
  const int h = cta / pg.splits, part = cta % pg.splits, hd = a.head_dim;
  const int pos = a.pos[0];
  int j0, j1;
  keys_of(a, pos, part, pg.splits, j0, j1);
  const bool newest = j1 > pos;  // this part holds the newest key
  const int jr = newest ? pos : j1;  // keys [j0, jr) come through the ring
  const int nk = j1 - j0;
  const int kvh = h / (a.heads / a.kv_heads);
  const int elt = a.kv_bf16 ? 2 : 4, rowb = hd * elt;
  const int kps = ring.slot_bytes / rowb;
  const float* q = a.q + (int64_t)h * hd;
  const int per = hd / 32;  // head-dim elements per lane (head_dim 64 or 128)
  float qv[4];
  for (int e = 0; e < 4; e++) qv[e] = e < per ? __ldcg(q + lane + 32 * e) : 0.f;
  auto key_elt = [&](const uint8_t* row, int e) -> float {
    return a.kv_bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(row)[lane + 32 * e])
                     : reinterpret_cast<const float*>(row)[lane + 32 * e];
  };
  // Scores (nn/kernels/attention.rs:100-127): scale * q.k.
  for (int j = j0; j < jr;) {
    const int sl = ring_slot(a, j);
    int n = min(jr - j, kps);
    if (a.window > 0) n = min(n, a.ring_cap - sl);
    const bool ok = take(sm, ring, it, pg.err);
    const uint8_t* slot = ring.slot(it);
    for (int t = warp; t < n; t += kConsWarps) {
      float d = 0.f;
      for (int e = 0; e < per; e++) d = fmaf(qv[e], ok ? key_elt(slot + (size_t)t * rowb, e) : 0.f, d);
      d = warp_sum(d);
      if (lane == 0) sm.sc[j - j0 + t] = a.scale * d;
    }
    give(sm, ring, it, lane);
    it++;
    j += n;
  }
  const uint8_t* kbase = static_cast<const uint8_t*>(a.k_ring) + (int64_t)kvh * a.ring_cap * rowb;
  const uint8_t* vbase = static_cast<const uint8_t*>(a.v_ring) + (int64_t)kvh * a.ring_cap * rowb;
  if (newest && warp == 0) {
    const uint8_t* row = kbase + (int64_t)ring_slot(a, pos) * rowb;
    float d = 0.f;
    for (int e = 0; e < per; e++)
      d = fmaf(qv[e], a.kv_bf16 ? __bfloat162float(__ldcg(reinterpret_cast<const __nv_bfloat16*>(row) + lane + 32 * e))
                                : __ldcg(reinterpret_cast<const float*>(row) + lane + 32 * e), d);
    d = warp_sum(d);
    if (lane == 0) sm.sc[nk - 1] = a.scale * d;
  }
  cons_sync();
  // Max, then exp_ref(s - max) and their sum (attention.rs:128-137).
  float mx = -INFINITY;
  for (int t = tid; t < nk; t += kCons) mx = fmaxf(mx, sm.sc[t]);
  mx = warp_max(mx);
  if (lane == 0) sm.red[0][warp] = mx;
  cons_sync();
  mx = sm.red[0][0];
  for (int w = 1; w < kConsWarps; w++) mx = fmaxf(mx, sm.red[0][w]);
  float sum = 0.f;
  for (int t = tid; t < nk; t += kCons) {
    const float e = exp_ref(sm.sc[t] - mx);
    sm.sc[t] = e;
    sum += e;
  }
  sum = warp_sum(sum);
  if (lane == 0) sm.red[1][warp] = sum;
  cons_sync();
  sum = 0.f;
  for (int w = 0; w < kConsWarps; w++) sum += sm.red[1][w];
  // Weighted values: warp w sums its keys, lane l dims l + 32 e.
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int j = j0; j < jr;) {
    const int sl = ring_slot(a, j);
    int n = min(jr - j, kps);
    if (a.window > 0) n = min(n, a.ring_cap - sl);
    const bool ok = take(sm, ring, it, pg.err);
    const uint8_t* slot = ring.slot(it);
    for (int t = warp; t < n; t += kConsWarps) {
      const float wt = sm.sc[j - j0 + t];
      for (int e = 0; e < per; e++) acc[e] = fmaf(wt, ok ? key_elt(slot + (size_t)t * rowb, e) : 0.f, acc[e]);
    }
    give(sm, ring, it, lane);
    it++;
    j += n;
  }
  if (newest && warp == 0) {
    const uint8_t* row = vbase + (int64_t)ring_slot(a, pos) * rowb;
    const float wt = sm.sc[nk - 1];
    for (int e = 0; e < per; e++)
      acc[e] = fmaf(wt, a.kv_bf16 ? __bfloat162float(__ldcg(reinterpret_cast<const __nv_bfloat16*>(row) + lane + 32 * e))
                                  : __ldcg(reinterpret_cast<const float*>(row) + lane + 32 * e), acc[e]);
  }
  for (int e = 0; e < per; e++) sm.acc[warp][lane + 32 * e] = acc[e];
  cons_sync();
  // Partial (max, sum, weighted values) of this part; the head's last part merges.
  float* part_out = pg.part + ((int64_t)h * pg.splits + part) * (hd + 2);
  for (int dd = tid; dd < hd; dd += kCons) {
    float v = 0.f;
    for (int w = 0; w < kConsWarps; w++) v += sm.acc[w][dd];
    part_out[2 + dd] = v;
  }
  if (tid == 0) {
    part_out[0] = mx;
    part_out[1] = sum;
  }
  __threadfence();
  cons_sync();
  if (tid == 0) {
    unsigned* cnt = pg.head_cnt + (int64_t)layer * a.heads + h;
    sm.flag = atomicAdd(cnt, 1u) == (unsigned)pg.splits - 1;
    if (sm.flag) *cnt = 0u;
  }
  cons_sync();
  if (!sm.flag) return;
  __threadfence();
  // Merge (flash-decoding style): M = max of the part maxima, w_s = exp(m_s - M) for parts
  // with keys, L = sum l_s w_s, out = sum acc_s w_s / L, parts in order.
  const float* parts = pg.part + (int64_t)h * pg.splits * (hd + 2);
  float* pm = sm.sc;            // part maxima
  float* pw = sm.sc + 256;      // part weights
  float* pl = sm.sc + 512;      // part sums
  for (int t = tid; t < pg.splits; t += kCons) {
    pm[t] = __ldcg(parts + (int64_t)t * (hd + 2));
    pl[t] = __ldcg(parts + (int64_t)t * (hd + 2) + 1);
  }
  cons_sync();
  float M = -INFINITY;
  for (int t = 0; t < pg.splits; t++) M = fmaxf(M, pm[t]);
  for (int t = tid; t < pg.splits; t += kCons) pw[t] = pl[t] > 0.f ? exp_ref(pm[t] - M) : 0.f;
  cons_sync();
  float L = 0.f;
  for (int t = 0; t < pg.splits; t++) L += pl[t] * pw[t];
  for (int dd = tid; dd < hd; dd += kCons) {
    float v = 0.f;
#pragma unroll 4
    for (int t = 0; t < pg.splits; t++) v += __ldcg(parts + (int64_t)t * (hd + 2) + 2 + dd) * pw[t];
    a.out[(int64_t)h * hd + dd] = __fdiv_rn(v, L);
  }
}

// LanguageModel::step's input sum (stt/model.rs:246-250) for this CTA's columns: the
// 1 + n_q rows are loaded at once into shared memory (the record area, free until the next
// phase), then each column is summed in the reference's order.
__device__ void embed_phase(const EmbedParams& e, float4* stage) {
  const int G = gridDim.x, cta = blockIdx.x, tid = threadIdx.x;
  const int c0 = (int)((int64_t)(e.d / 4) * cta / G), c1 = (int)((int64_t)(e.d / 4) * (cta + 1) / G);
  const int nc = c1 - c0, rows = 1 + e.n_q;
  for (int t = tid; t < rows * nc; t += kCons) {
    const int r = t / nc, c4 = c0 + t % nc;
    uint32_t tok = r == 0 ? e.text_tok[0] : e.audio_tok[r - 1];
    const uint32_t lim = r == 0 ? (uint32_t)e.text_card : (uint32_t)e.card;
    if (tok > lim) {
      atomicExch(e.error_flag, 1);
      tok = 0;
    }
    const void* table = r == 0 ? e.text_table : e.audio_tables;
    const int64_t row = r == 0 ? (int64_t)tok : (int64_t)(r - 1) * (e.card + 1) + tok;
    float4 v;
    if (e.tables_bf16) {
      const uint2 u = reinterpret_cast<const uint2*>(reinterpret_cast<const __nv_bfloat16*>(table) + row * e.d)[c4];
      v = make_float4(bf16_lo(u.x), bf16_hi(u.x), bf16_lo(u.y), bf16_hi(u.y));
    } else {
      v = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(table) + row * e.d)[c4];
    }
    stage[t] = v;
  }
  cons_sync();
  for (int c = tid; c < nc; c += kCons) {
    float4 acc = stage[c];
    for (int r = 1; r < rows; r++) {
      const float4 v = stage[r * nc + c];
      acc.x = acc.x + v.x;
      acc.y = acc.y + v.y;
      acc.z = acc.z + v.z;
      acc.w = acc.w + v.w;
    }
    reinterpret_cast<float4*>(e.x)[c0 + c] = acc;
  }
}

template <int WT>
__global__ void __launch_bounds__(kSThreads, 1) step_kernel(const StepProgram pg) {
  extern __shared__ __align__(128) uint8_t dsm[];
  __shared__ Smem sm;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  Ring ring{dsm, pg.slot_bytes, pg.nslots};
  uint8_t* rec = dsm + (size_t)pg.slot_bytes * pg.nslots;  // pg.rec_bytes of input record
  if (tid == 0) {
    for (int i = 0; i < pg.nslots; i++) {
      mbar_init(&sm.full[i], 1);
      mbar_init(&sm.empty[i], kConsWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();
  if (warp == kConsWarps) {
    if (lane == 0) producer(pg, sm, ring);
    return;
  }
  uint32_t it = 0;
  int layer = 0;
  for (int p = 0; p < pg.nph; p++) {
    // The phase's parameters into shared memory: the epilogues and dot loops read them for
    // every row, and global loads would miss L1 after each phase's acquire.
    {
      static_assert(sizeof(StepPhase) % 4 == 0, "phase copy");
      const uint32_t* src = reinterpret_cast<const uint32_t*>(pg.ph + p);
      uint32_t* dst = reinterpret_cast<uint32_t*>(&sm.cur);
      for (int i = tid; i < (int)(sizeof(StepPhase) / 4); i += kCons) dst[i] = src[i];
    }
    const StepPhase& P = sm.cur;
    cons_sync();
    if (P.type == PH_GEMV && P.g.epi == EPI_QKV_ROPE) {
      // The (cos, sin) of this position for each RoPE frequency, once per phase (the position
      // was written by the previous step: stable here).
      const int pos = P.g.pos[0];
      for (int i = tid; i < P.g.head_dim / 2; i += kCons) {
        float sn, c;
        sincosf((float)pos * P.g.inv_freq[i], &sn, &c);
        sm.rope[i] = make_float2(c, sn);
      }
    }
    if (p > 0 && tid == 0 && !wait_count(pg.done + p - 1, gridDim.x, pg.err)) atomicExch(pg.err, 3);
    cons_sync();
    if (P.type == PH_EMBED) {
      embed_phase(P.e, reinterpret_cast<float4*>(rec));
    } else if (P.type == PH_GEMV) {
      gemv_phase<WT>(pg, P.g, sm, ring, rec, it);
    } else {
      attn_phase(pg, P.a, layer, sm, ring, it);
      layer++;
    }
    __threadfence();
    cons_sync();
    if (tid == 0) atomicAdd(pg.done + p, 1u);
  }
}

template <int WT>
void setup_kernel() {
  cudaFuncSetAttribute(step_kernel<WT>, cudaFuncAttributeMaxDynamicSharedMemorySize, kStepDynSmem);
}

}  // namespace

int step_kernel_ctas(int wtype) {
  int dev = 0, sms = 0, per = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaError_t e = cudaSuccess;
  switch (wtype) {
    case W_F32: e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, step_kernel<W_F32>, kSThreads, kStepDynSmem); break;
    case W_BF16: e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, step_kernel<W_BF16>, kSThreads, kStepDynSmem); break;
    case W_Q8: e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, step_kernel<W_Q8>, kSThreads, kStepDynSmem); break;
    default: e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, step_kernel<W_Q4>, kSThreads, kStepDynSmem); break;
  }
  if (e != cudaSuccess || per < 1) {
    cudaGetLastError();
    return 0;
  }
  return sms;
}

void step_kernel_init_device() {
  setup_kernel<W_F32>();
  setup_kernel<W_BF16>();
  setup_kernel<W_Q8>();
  setup_kernel<W_Q4>();
}

void launch_step_kernel(const StepProgram& pg, int wtype, int ctas, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ctas);
  cfg.blockDim = dim3(kSThreads);
  cfg.dynamicSmemBytes = kStepDynSmem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  switch (wtype) {
    case W_F32: cudaLaunchKernelEx(&cfg, step_kernel<W_F32>, pg); break;
    case W_BF16: cudaLaunchKernelEx(&cfg, step_kernel<W_BF16>, pg); break;
    case W_Q8: cudaLaunchKernelEx(&cfg, step_kernel<W_Q8>, pg); break;
    default: cudaLaunchKernelEx(&cfg, step_kernel<W_Q4>, pg); break;
  }
}

}  // namespace svl
