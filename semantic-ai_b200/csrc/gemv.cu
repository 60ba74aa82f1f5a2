// gemv.cu — weight-streaming matrix-vector products for small stream counts.
//
// At small batch the step is bound by reading every weight once (the reference runs the
// same products on the CPU through kernels::matvec, nn/kernels/matvec.rs:29-58, and
// candle's QMatMul, nn/mod.rs:97). Each warp owns a contiguous range of row groups (R rows)
// and streams them straight from global memory into registers, 16 bytes per lane and U
// loads per row in flight (with the block formats' scales), with 2 CTAs of 8 warps per SM.
// With programmatic dependent launch, each warp issues its first group's loads before
// griddepcontrol.wait (weights do not depend on the previous kernel), and one thread per CTA
// pulls its share of a later kernel's weights into L2 (cp.async.bulk.prefetch.L2). After the
// wait, every CTA turns the input row(s) into records in shared memory -- the layer's norm
// (candle rms_norm / layer_norm) and the conversion for the weight format (bf16 rounding, or
// the Q8_0 / Q8_1 activation blocks candle's QMatMul builds) -- while those first weight
// loads are still in flight. Each row group ends with the fused epilogue (RoPE + KV-ring
// write, SwiGLU, GELU, SiLU, residual add, logits + argmax), one lane per (row, stream).
#include "common.cuh"
#include "gemv_common.cuh"
#include "kernels.cuh"

#include <climits>

namespace svl {

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kCtasPerSm = 2;
constexpr int kGrid = 148 * kCtasPerSm;

__device__ __forceinline__ uint4 ldg_weights(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// Accumulates chunks [c0, c0 + 32 U) of R rows (weights already in wv, and for the block
// formats their scales in ws) against the NB input records in shared memory (record b at
// xsm + b * rec: see input_rec_bytes).
template <int WT, int NB, int R, int U>
__device__ __forceinline__ void dot_chunks(const uint4 (&wv)[R][U], const uint32_t (&ws)[R][U],
                                           const GemvParams& p, int g, int c0, const uint8_t* xsm,
                                           int rec, int lane, float (&acc)[R][NB]) {
  const int k = p.k, nch = chunks_per_row(WT, k), nblk = k / QBLK;
#pragma unroll
  for (int u = 0; u < U; u++) {
    const int c = c0 + lane + 32 * u;
    const bool valid = c < nch;
    if (WT == W_F32) {
      if (valid) {
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
      }
    } else if (WT == W_BF16) {
      if (valid) {
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
    } else if (WT == W_Q8) {
      // Chunk c is half of block c/2: lanes 2j and 2j+1 share a block and its scales.
      const int blk = c >> 1;
      float dw[R];
#pragma unroll
      for (int r = 0; r < R; r++) dw[r] = __half2float(__ushort_as_half((unsigned short)ws[r][u]));
#pragma unroll
      for (int b = 0; b < NB; b++) {
        const uint8_t* xr = xsm + (size_t)b * rec;
        const int4 x = valid ? reinterpret_cast<const int4*>(xr)[c] : make_int4(0, 0, 0, 0);
        const float dx = valid ? reinterpret_cast<const float*>(xr + k)[blk] : 0.f;
#pragma unroll
        for (int r = 0; r < R; r++) {
          const uint4 w = wv[r][u];
          int s = __dp4a((int)w.x, x.x, 0);
          s = __dp4a((int)w.y, x.y, s);
          s = __dp4a((int)w.z, x.z, s);
          s = __dp4a((int)w.w, x.w, s);
          s += __shfl_xor_sync(0xffffffffu, s, 1);
          if (valid && !(lane & 1)) acc[r][b] = fmaf(dw[r] * dx, (float)s, acc[r][b]);
        }
      }
    } else {  // W_Q4: chunk c is block c, 16 bytes of nibbles (ggml Q4_1 order).
      if (valid) {
        float2 dm[R];
#pragma unroll
        for (int r = 0; r < R; r++) {
          const uint32_t h = ws[r][u];
          dm[r] = __half22float2(*reinterpret_cast<const __half2*>(&h));
        }
#pragma unroll
        for (int b = 0; b < NB; b++) {
          const uint8_t* xr = xsm + (size_t)b * rec;
          const int4* xb = reinterpret_cast<const int4*>(xr + (size_t)c * QBLK);
          const int4 lo = xb[0], hi = xb[1];
          const float dx = reinterpret_cast<const float*>(xr + k)[c];
          const float sx = reinterpret_cast<const float*>(xr + k)[nblk + c];
#pragma unroll
          for (int r = 0; r < R; r++) {
            const uint4 w = wv[r][u];
            int s = __dp4a((int)(w.x & 0x0f0f0f0fu), lo.x, 0);
            s = __dp4a((int)(w.y & 0x0f0f0f0fu), lo.y, s);
            s = __dp4a((int)(w.z & 0x0f0f0f0fu), lo.z, s);
            s = __dp4a((int)(w.w & 0x0f0f0f0fu), lo.w, s);
            s = __dp4a((int)((w.x >> 4) & 0x0f0f0f0fu), hi.x, s);
            s = __dp4a((int)((w.y >> 4) & 0x0f0f0f0fu), hi.y, s);
            s = __dp4a((int)((w.z >> 4) & 0x0f0f0f0fu), hi.z, s);
            s = __dp4a((int)((w.w >> 4) & 0x0f0f0f0fu), hi.w, s);
            acc[r][b] += (dm[r].x * dx) * (float)s + dm[r].y * sx;
          }
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
  __shared__ float red[2][kWarps];
  __shared__ float stat[2];
  __shared__ bool last_cta;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nb = p.nb, nch = chunks_per_row(WT, p.k), rec = rec_bytes_of(WT, p.k);
  // Row groups of R rows (R even keeps the RoPE / SwiGLU pairs in one group), split into
  // contiguous ranges per warp.
  const int groups = (p.n + R - 1) / R;
  const int total_w = gridDim.x * kWarps;
  const int gw = blockIdx.x * kWarps + warp;
  const int g0 = (int)((int64_t)gw * groups / total_w), g1 = (int)((int64_t)(gw + 1) * groups / total_w);

  uint4 wv[R][U];
  uint32_t ws[R][U];  // block formats: the scale (q8_0: d) or scale and min (q4_1) of each chunk
  // Loads chunks [c0, c0 + 32 U) of group g's rows, with their block scales: every load of
  // the group is in flight at once.
  auto issue = [&](int g, int c0) {
#pragma unroll
    for (int r = 0; r < R; r++)
#pragma unroll
      for (int u = 0; u < U; u++) {
        const int c = c0 + lane + 32 * u;
        const int row = g * R + r;
        const bool on = g < g1 && c < nch && row < p.n;
        const uint8_t* wrow = p.w + (int64_t)row * p.row_stride;
        wv[r][u] = on ? ldg_weights(wrow + (int64_t)c * 16) : make_uint4(0, 0, 0, 0);
        ws[r][u] = 0u;
        if (WT == W_Q8 && on)
          ws[r][u] = reinterpret_cast<const unsigned short*>(wrow + p.k)[c >> 1];
        else if (WT == W_Q4 && on)
          ws[r][u] = reinterpret_cast<const uint32_t*>(wrow + p.k / 2)[c];
      }
  };
  // Weights do not depend on the previous kernel: first group's loads and the L2 prefetch
  // of a later kernel's weights go out before the dependency wait.
  issue(g0, 0);
  if (tid == 0 && p.pf && p.pf_bytes > 0) {
    const int64_t share = (p.pf_bytes / gridDim.x + 15) / 16 * 16;
    const int64_t a = (int64_t)blockIdx.x * share;
    const int64_t e = min(a + share, p.pf_bytes / 16 * 16);
    for (int64_t o = a; o < e; o += 65536) prefetch_l2(p.pf + o, (uint32_t)(e - o < 65536 ? e - o : 65536));
  }
  pdl_launch();
  pdl_wait();
  build_records<WT, NB>(p, xsm, rec, red, stat, [] { __syncthreads(); });

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
      dot_chunks<WT, NB, R, U>(wv, ws, p, g, c0, xsm, rec, lane, acc);
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

  // Argmax: CTA best per stream, then the last CTA reduces the CTA bests.
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
    if (tid == 0) last_cta = atomicAdd(p.am_ticket, 1u) == gridDim.x - 1;
    __syncthreads();
    if (last_cta) {
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

}

constexpr size_t kMaxSmem = 96 * 1024;  // input records; 2 CTAs per SM

// Rows per warp group: the fewest (of 1, 2, 4) whose groups fit in one wave of warps, so the
// whole matrix is in flight at once; 2 at least when the epilogue pairs rows.
int pick_r(const GemvParams& p) {
  const int warps = kGrid * kWarps;
  const bool pairs = p.epi == EPI_QKV_ROPE || p.epi == EPI_SWIGLU;
  if (!pairs && p.n <= warps) return 1;
  if (p.n <= 2 * warps) return 2;
  return 4;
}

// Loads per row in flight per lane: 8 (f32), 4, or 2 for four-row groups (whose block
// scales ride along in registers).
template <int WT, int R>
constexpr int kU = WT == W_F32 ? 8 : R == 4 ? 2 : 4;

template <int WT, int NB, int R>
void launch_r(const GemvParams& p, cudaStream_t s) {
  constexpr int U = kU<WT, R>;
  const int groups = (p.n + R - 1) / R;
  int grid = (groups + kWarps - 1) / kWarps;
  if (grid > kGrid) grid = kGrid;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = (size_t)NB * rec_bytes_of(WT, p.k);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, gemv_kernel<WT, NB, R, U>, p);
}

// Four-row groups only where their registers fit without spilling (one stream, 16-byte
// formats with U = 4).
template <int WT, int NB>
constexpr bool kAllowR4 = NB == 1 && WT != W_F32;

template <int WT, int NB>
void launch_t(const GemvParams& p, cudaStream_t s) {
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

template <int WT, int NB>
void set_attrs_nb() {
  cudaFuncSetAttribute(gemv_kernel<WT, NB, 1, kU<WT, 1>>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem);
  cudaFuncSetAttribute(gemv_kernel<WT, NB, 2, kU<WT, 2>>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem);
  if constexpr (kAllowR4<WT, NB>)
    cudaFuncSetAttribute(gemv_kernel<WT, NB, 4, kU<WT, 4>>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem);
}

template <int WT>
void set_attrs() {
  set_attrs_nb<WT, 1>();
  set_attrs_nb<WT, 2>();
  set_attrs_nb<WT, 4>();
  set_attrs_nb<WT, 8>();
}

// Streams per launch: the widest template whose input records fit.
int max_nb(const GemvParams& p) {
  for (int nb : {8, 4, 2})
    if ((size_t)nb * rec_bytes_of(p.wtype, p.k) <= kMaxSmem) return nb;
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
    if (b0 > 0) p.pf = nullptr;
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
