// gemm.cu — the weight products of many concurrent streams on the 5th-generation tensor
// cores: Y[s][r] = epilogue(sum_k W[r][k] * X[s][k]) with W the bf16 weights [n][k] and X the
// bf16 operand rows of the streams [nb][k].
//
// With a few hundred streams per GPU the step's products stop being matrix-vector work: at
// 256 streams one pass over 1.68 GB of bf16 weights does 429 GFLOP, right at the B200's
// ridge point, so the weights must stream at HBM speed AND the tensor pipe must stay busy.
//
// One CTA owns a tile of 128 weight rows (the MMA's M) times up to 256 streams (its N), and a
// range of K. Per 64-wide K block, one thread issues two TMA tile loads (W 128x64 and X
// BNx64, both 128-byte swizzled) into a ring of shared-memory stages; another issues four
// tcgen05.mma (K = 16 each) accumulating in tensor memory, and frees the stage with
// tcgen05.commit. Narrow matrices (out_proj, linear_out: 16 row tiles) split K over a
// thread-block cluster so that every SM streams weights; the partial tiles are pushed into
// the owning CTA's shared memory over DSMEM and summed in a fixed order, so results do not
// depend on timing. The epilogue reads the accumulator with tcgen05.ld (one weight row per
// thread, 32 streams per load) and applies the same fused epilogues as the matrix-vector
// kernel: RoPE + KV-ring write, SwiGLU, GELU, residual with layer scale, logits + argmax.
//
// No TMA load here uses cluster multicast: clusters only share partial sums through DSMEM.
#include <cuda.h>
#include <cuda_bf16.h>
#include <climits>

#include "common.cuh"
#include "kernels.cuh"
#include "sm100.cuh"

namespace svl {
namespace {

constexpr int kBM = 128;              // weight rows per tile (MMA M)
constexpr int kBK = 64;               // K per stage: 128 bytes of bf16, one swizzle row
constexpr int kGThreads = 256;        // 8 warps: producer lane, MMA lane, then all epilogue
constexpr uint32_t kWTile = kBM * kBK * 2;  // 16 KB
constexpr int kMaxClusterSplit = 8;

template <int BN>
struct Cfg {
  // 128-stream tiles: a 96 KB stage ring, so that two CTAs share an SM and one's epilogue
  // overlaps the other's main loop (the next product's CTA can start its weight loads while
  // this one finishes). 256-stream tiles: 192 KB, one CTA per SM.
  static constexpr size_t kPipeBytes = BN <= 128 ? 96 * 1024 : 192 * 1024;
  static constexpr int kMinBlocks = BN <= 128 ? 2 : 1;
  static constexpr uint32_t kXTile = BN * kBK * 2;
  static constexpr uint32_t kStage = kWTile + kXTile;
  static constexpr int kStages = (int)(kPipeBytes / kStage) > 8 ? 8 : (int)(kPipeBytes / kStage);
  static constexpr uint32_t kCols = BN <= 32 ? 32 : BN <= 64 ? 64 : BN <= 128 ? 128 : 256;
  static constexpr size_t kSmem = (size_t)kStages * kStage + 1024;  // + alignment slack
  // The epilogue's tile (kBM rows x BN streams of f32) reuses the stage ring.
  static_assert((size_t)kBM * BN * 4 <= (size_t)kStages * kStage, "epilogue must fit the ring");
};

// ---- tcgen05 / TMA wrappers ---------------------------------------------------------------

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | (1ull << 16) | (64ull << 32) | (1ull << 46) |
         (2ull << 61);
}
// Instruction descriptor of kind::f16: f32 accumulator, A and B both bf16 (fmt 1) or both
// f16 (fmt 0), both K-major.
__host__ __device__ constexpr uint32_t idesc_f16kind(int m, int n, uint32_t fmt) {
  return (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t)(n >> 3) << 17) |
         ((uint32_t)(m >> 4) << 24);
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* tm, int c0, int c1,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(c0), "r"(c1), "r"(smem_addr(bar))
      : "memory");
}
__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_addr(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// 16 consecutive f32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}
// Order-preserving map of a float onto an unsigned key (larger float, larger key).
__device__ __forceinline__ uint32_t order_key(float v) {
  const uint32_t u = __float_as_uint(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
  return v > bv || (v == bv && i < bi) || bi == INT_MAX;
}

// Activations of the tensor-core path. Their outputs become bf16 GEMM operands (rounded to 8
// significant bits), so they use the hardware exp2 and fast division; the f32 path keeps the
// reference's exp (exp_ref) for bit-level parity.
__device__ __forceinline__ float silu_fast(float x) { return __fdividef(x, 1.0f + __expf(-x)); }
__device__ __forceinline__ float gelu_tanh_fast(float x) {
  const float y = 0.7978846f * fmaf(0.044715f * x, x * x, x);
  return __fdividef(x, 1.0f + __expf(-2.0f * y));
}

// Phase B of the epilogue: rows [r0, r0 + 8) of one stream, whose full sums are y[0..7]
// (weight rows tile_row0 + r0 ...; RoPE and SwiGLU pair rows 2i, 2i+1 inside the 8). Reads
// and writes are 16-byte vectors along the rows, so 16 consecutive threads cover a stream's
// 128 rows with contiguous 512-byte accesses. Same arithmetic as the matrix-vector kernel's
// epilogue, with fast activations (their outputs become bf16 operands) and RoPE's cos / sin
// read from the step's table.
template <int EPI>
__device__ __forceinline__ void finish8(const GemvParams& p, int out_bf16, int b, int row0,
                                        float (&y)[8], int slot) {
  const int nrow = p.n - row0 < 8 ? p.n - row0 : 8;  // rows of this chunk that exist
  if (nrow <= 0) return;
  if (p.bias && EPI != EPI_SWIGLU && EPI != EPI_QKV_ROPE) {
#pragma unroll
    for (int e = 0; e < 8; e++) y[e] = y[e] + (e < nrow ? p.bias[row0 + e] : 0.f);
  }
  auto put8 = [&](int64_t i, const float (&z)[8]) {  // out[i .. i + 8)
    if (out_bf16) {
      __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(p.out) + i;
      if (nrow == 8) {
        __nv_bfloat162 h[4];
#pragma unroll
        for (int e = 0; e < 4; e++) h[e] = __floats2bfloat162_rn(z[2 * e], z[2 * e + 1]);
        *reinterpret_cast<uint4*>(o) = *reinterpret_cast<uint4*>(h);
      } else {
        for (int e = 0; e < nrow; e++) o[e] = __float2bfloat16_rn(z[e]);
      }
    } else {
      float* o = p.out + i;
      if (nrow == 8) {
        reinterpret_cast<float4*>(o)[0] = make_float4(z[0], z[1], z[2], z[3]);
        reinterpret_cast<float4*>(o)[1] = make_float4(z[4], z[5], z[6], z[7]);
      } else {
        for (int e = 0; e < nrow; e++) o[e] = z[e];
      }
    }
  };
  if constexpr (EPI == EPI_RESIDUAL) {
    float* o = p.out + b * p.out_stride + row0;
    if (nrow == 8) {
      float4 a0 = reinterpret_cast<float4*>(o)[0], a1 = reinterpret_cast<float4*>(o)[1];
      float ls[8] = {1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f};
      if (p.ls) {
        const float4 l0 = reinterpret_cast<const float4*>(p.ls + row0)[0];
        const float4 l1 = reinterpret_cast<const float4*>(p.ls + row0)[1];
        ls[0] = l0.x; ls[1] = l0.y; ls[2] = l0.z; ls[3] = l0.w;
        ls[4] = l1.x; ls[5] = l1.y; ls[6] = l1.z; ls[7] = l1.w;
      }
      float u[8];
#pragma unroll
      for (int e = 0; e < 8; e++) u[e] = p.ls ? y[e] * ls[e] : y[e];
      a0.x = a0.x + u[0]; a0.y = a0.y + u[1]; a0.z = a0.z + u[2]; a0.w = a0.w + u[3];
      a1.x = a1.x + u[4]; a1.y = a1.y + u[5]; a1.z = a1.z + u[6]; a1.w = a1.w + u[7];
      reinterpret_cast<float4*>(o)[0] = a0;
      reinterpret_cast<float4*>(o)[1] = a1;
    } else {
      for (int e = 0; e < nrow; e++) o[e] = o[e] + (p.ls ? y[e] * p.ls[row0 + e] : y[e]);
    }
  } else if constexpr (EPI == EPI_STORE || EPI == EPI_LOGITS || EPI == EPI_GELU_TANH ||
                       EPI == EPI_GELU_ERF || EPI == EPI_SILU) {
    if (!p.out) return;
    float z[8];
#pragma unroll
    for (int e = 0; e < 8; e++)
      z[e] = EPI == EPI_GELU_TANH ? gelu_tanh_fast(y[e])
             : EPI == EPI_GELU_ERF ? gelu_erf_ref(y[e])
             : EPI == EPI_SILU ? silu_fast(y[e]) : y[e];
    put8(b * p.out_stride + row0, z);
  } else if constexpr (EPI == EPI_SWIGLU) {
    // Packed row 2i is gate row i, 2i+1 value row i (FeedForwardLayer::Gated,
    // nn/transformer.rs:457-461): 4 outputs at row0 / 2.
    float z[4];
#pragma unroll
    for (int e = 0; e < 4; e++) z[e] = silu_fast(y[2 * e]) * y[2 * e + 1];
    const int64_t i = b * p.out_stride + row0 / 2;
    if (out_bf16) {
      __nv_bfloat162 h[2] = {__floats2bfloat162_rn(z[0], z[1]), __floats2bfloat162_rn(z[2], z[3])};
      __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(p.out) + i;
      if (nrow == 8)
        *reinterpret_cast<uint2*>(o) = *reinterpret_cast<uint2*>(h);
      else
        for (int e = 0; e < nrow / 2; e++) o[e] = __float2bfloat16_rn(z[e]);
    } else {
      float* o = p.out + i;
      if (nrow == 8)
        *reinterpret_cast<float4*>(o) = make_float4(z[0], z[1], z[2], z[3]);
      else
        for (int e = 0; e < nrow / 2; e++) o[e] = z[e];
    }
  } else if constexpr (EPI == EPI_QKV_ROPE) {
    // Chunks of 8 rows never straddle the q / k / v regions or a head (all multiples of 8).
    const int hd = p.head_dim;
    const bool is_v = row0 >= p.q_dim + p.kv_dim, is_q = row0 < p.q_dim;
    const int rr = is_v ? row0 - p.q_dim - p.kv_dim : is_q ? row0 : row0 - p.q_dim;
    const int dim0 = rr % hd, kh = rr / hd;
    float z[8];
    if (!is_v) {
      // rope_i (candle; nn/transformer.rs:339-340): pairs (2i, 2i+1) rotate by pos * f_i.
      const float4* cs4 = reinterpret_cast<const float4*>(p.rope_cs + (int64_t)b * (hd >> 1) + (dim0 >> 1));
      const float4 c01 = cs4[0], c23 = cs4[1];
      const float c[4] = {c01.x, c01.z, c23.x, c23.z}, sn[4] = {c01.y, c01.w, c23.y, c23.w};
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const float lo = y[2 * e], hi = y[2 * e + 1];
        z[2 * e] = lo * c[e] - hi * sn[e];
        z[2 * e + 1] = lo * sn[e] + hi * c[e];
      }
    } else {
#pragma unroll
      for (int e = 0; e < 8; e++) z[e] = y[e];
    }
    if (is_q) {
      float* o = p.out + b * p.out_stride + row0;
      reinterpret_cast<float4*>(o)[0] = make_float4(z[0], z[1], z[2], z[3]);
      reinterpret_cast<float4*>(o)[1] = make_float4(z[4], z[5], z[6], z[7]);
    } else {
      void* ring = is_v ? p.v_ring : p.k_ring;
      const int64_t off = b * p.ring_stream_stride + ((int64_t)kh * p.ring_cap + slot) * hd + dim0;
      if (p.kv_bf16) {
        __nv_bfloat162 h[4];
#pragma unroll
        for (int e = 0; e < 4; e++) h[e] = __floats2bfloat162_rn(z[2 * e], z[2 * e + 1]);
        *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(ring) + off) = *reinterpret_cast<uint4*>(h);
      } else {
        float* o = reinterpret_cast<float*>(ring) + off;
        reinterpret_cast<float4*>(o)[0] = make_float4(z[0], z[1], z[2], z[3]);
        reinterpret_cast<float4*>(o)[1] = make_float4(z[4], z[5], z[6], z[7]);
      }
    }
  }
}

struct GemmArgs {
  GemvParams p;      // sizes and epilogue (x / norm unused: the operand is the bf16 X map)
  int kblocks;       // ceil(k / 64)
  int split;         // CTAs of a cluster, each a contiguous range of K blocks
  int x_row0;        // first X row of this launch's streams
  int out_bf16;      // STORE / SWIGLU / GELU / SILU outputs as bf16
  int* err;          // set when a bounded wait runs out
  float* ws;         // split exchange: [CTA][BN streams][128 rows] f32 partial tiles
  uint32_t idesc;    // instruction descriptor (operand type)
};


// Bounded wait with back-off, for the epilogue warps that idle through the main loop.
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < kWaitLimit; i++) {
    if (mbar_try_wait(bar, parity)) return true;
    __nanosleep(128);
  }
  return false;
}

template <int BN, int EPI>
__global__ void __launch_bounds__(kGThreads, Cfg<BN>::kMinBlocks)
    gemm_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                const GemmArgs ga) {
  using C = Cfg<BN>;
  constexpr bool kLogits = EPI == EPI_LOGITS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* w_s = smem;
  uint8_t* x_s = smem + (size_t)C::kStages * kWTile;
  float* xch = reinterpret_cast<float*>(smem);  // split-K exchange, after the main loop
  __shared__ __align__(8) uint64_t full_bar[C::kStages], empty_bar[C::kStages], accum_bar;
  __shared__ uint32_t tmem_slot;
  __shared__ int failed;
  __shared__ int slot_sm[BN];
  __shared__ bool last_cta;

  const GemvParams& p = ga.p;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int S = ga.split;
  const uint32_t crank = S > 1 ? cluster_rank() : 0;
  const int tile = blockIdx.x / S;
  const int s0 = blockIdx.y * BN;  // first stream of this CTA (relative to the launch)
  const int kb0 = (int)(crank * ga.kblocks / S), kb1 = (int)((crank + 1) * ga.kblocks / S);
  const int nkb = kb1 - kb0;

  if (tid == 0) {
    for (int i = 0; i < C::kStages; i++) {
      mbar_init(&full_bar[i], 1);
      mbar_init(&empty_bar[i], 1);
    }
    mbar_init(&accum_bar, 1);
    failed = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_addr(&tmem_slot)),
                 "r"(C::kCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;

  if (warp == 0 && lane == 0) {
    // Producer. Weights do not depend on the previous kernel: the first stages' weight tiles
    // go out before the dependency wait, their X tiles after it.
    const int pre = nkb < C::kStages ? nkb : C::kStages;
    for (int i = 0; i < pre; i++) {
      mbar_expect_tx(&full_bar[i], C::kStage);
      tma_load_2d(w_s + (size_t)i * kWTile, &tm_w, (kb0 + i) * kBK, tile * kBM, &full_bar[i]);
    }
    pdl_wait();
    for (int i = 0; i < pre; i++)
      tma_load_2d(x_s + (size_t)i * C::kXTile, &tm_x, (kb0 + i) * kBK, ga.x_row0 + s0, &full_bar[i]);
    for (int i = pre; i < nkb; i++) {
      const int st = i % C::kStages;
      if (!mbar_wait(&empty_bar[st], ((i / C::kStages) - 1) & 1)) {
        failed = 1;
        break;
      }
      mbar_expect_tx(&full_bar[st], C::kStage);
      tma_load_2d(w_s + (size_t)st * kWTile, &tm_w, (kb0 + i) * kBK, tile * kBM, &full_bar[st]);
      tma_load_2d(x_s + (size_t)st * C::kXTile, &tm_x, (kb0 + i) * kBK, ga.x_row0 + s0, &full_bar[st]);
    }
  } else if (warp == 1 && lane == 0) {
    // MMA issuer.
    const uint32_t idesc = ga.idesc;
    for (int i = 0; i < nkb; i++) {
      const int st = i % C::kStages;
      if (!mbar_wait(&full_bar[st], (i / C::kStages) & 1)) {
        failed = 1;
        break;
      }
      tc_fence_after();
      const uint32_t wa = smem_addr(w_s + (size_t)st * kWTile);
      const uint32_t xa = smem_addr(x_s + (size_t)st * C::kXTile);
#pragma unroll
      for (int k = 0; k < kBK / 16; k++)
        umma_bf16(tmem, sw128_desc(wa + k * 32), sw128_desc(xa + k * 32), idesc, (i | k) != 0);
      umma_commit(&empty_bar[st]);
    }
    umma_commit(&accum_bar);
  }
  pdl_launch();
  pdl_wait();
  __syncwarp();
  if (EPI == EPI_QKV_ROPE) {
    for (int j = tid; j < BN; j += kGThreads) {
      const int s = s0 + j;
      const int pos = s < p.nb ? p.pos[s] : 0;
      slot_sm[j] = p.windowed ? pos % p.ring_cap : pos;
    }
  }

  const bool ok = mbar_wait_sleep(&accum_bar, 0);
  tc_fence_after();
  __syncthreads();  // slot_sm ready
  if ((!ok || failed) && tid == 0 && ga.err) atomicExch(ga.err, 2);

  // Phase A: the accumulator leaves tensor memory. Warp w reads TMEM lanes [32 (w % 4), +32)
  // (its row quarter) for half w / 4 of the stream columns and stores the tile as
  // [stream][row] f32: into this CTA's shared memory without a split; with one, into this
  // CTA's slot of the global exchange (L2-resident), from which each CTA of the cluster then
  // sums its slice of streams over all ranks, in rank order.
  const int quarter = warp & 3, half = warp >> 2;
  const int row_l = quarter * 32 + lane;
  const uint32_t trow = tmem + ((uint32_t)(quarter * 32) << 16);
  constexpr int kHalf = BN / 2;
  const int slice = BN / S;  // streams each CTA finishes
  const int nb_cta = p.nb - s0;
  const int cta_lin = blockIdx.y * gridDim.x + blockIdx.x;
  float* tile_out = S == 1 ? xch : ga.ws + (size_t)cta_lin * BN * kBM;
  for (int c = half * kHalf; c < (half + 1) * kHalf; c += 16) {
    if (c >= nb_cta) break;
    float v[16];
    tmem_ld16(trow + c, v);
    float* dst = tile_out + ((size_t)c * kBM + row_l);
#pragma unroll
    for (int j = 0; j < 16; j++) dst[(size_t)j * kBM] = v[j];
  }
  if (S > 1)
    cluster_sync();  // release / acquire at cluster scope: the ranks' partial tiles are visible
  else
    __syncthreads();

  // Phase B: streams [sb, sb + slice) of this CTA. Item (stream, 8-row chunk): the S partials
  // summed in rank order, then the epilogue; 16 consecutive threads share a stream, so reads
  // and writes run along contiguous rows.
  const int sb = S > 1 ? (int)crank * slice : 0;
  const int row_t = tile * kBM;
  const int n_fin = (p.nb - s0 - sb) < slice ? (p.nb - s0 - sb) : slice;
  const int cta0 = cta_lin - (int)crank;  // rank 0 of this cluster
  for (int it = tid; it < n_fin * (kBM / 8); it += kGThreads) {
    const int sw = it >> 4, c8 = it & 15;
    float y[8];
    if (S == 1) {
      const float4* src = reinterpret_cast<const float4*>(xch + ((size_t)sw * kBM + c8 * 8));
      const float4 a0 = src[0], a1 = src[1];
      y[0] = a0.x; y[1] = a0.y; y[2] = a0.z; y[3] = a0.w;
      y[4] = a1.x; y[5] = a1.y; y[6] = a1.z; y[7] = a1.w;
    } else {
#pragma unroll
      for (int e = 0; e < 8; e++) y[e] = 0.f;
      for (int q = 0; q < S; q++) {
        const float4* src = reinterpret_cast<const float4*>(
            ga.ws + ((size_t)(cta0 + q) * BN + sb + sw) * kBM + c8 * 8);
        const float4 a0 = __ldcg(src), a1 = __ldcg(src + 1);
        y[0] += a0.x; y[1] += a0.y; y[2] += a0.z; y[3] += a0.w;
        y[4] += a1.x; y[5] += a1.y; y[6] += a1.z; y[7] += a1.w;
      }
    }
    if (kLogits) {
      // Keep the full sums (plus bias) in shared memory for the argmax pass below.
      float* keep = xch + ((size_t)sw * kBM + c8 * 8);
#pragma unroll
      for (int e = 0; e < 8; e++) {
        const int r = row_t + c8 * 8 + e;
        keep[e] = y[e] + ((p.bias && r < p.n) ? p.bias[r] : 0.f);
      }
    }
    finish8<EPI>(p, ga.out_bf16, s0 + sb + sw, row_t + c8 * 8, y,
                 EPI == EPI_QKV_ROPE ? slot_sm[sb + sw] : 0);
  }

  if constexpr (kLogits) {
    // Per finished stream (one warp each): the CTA's best (value, row) over its 128 rows,
    // lowest row on ties; then the last CTA of the grid reduces the per-tile candidates.
    __syncthreads();
    const int tiles = gridDim.x / S;
    for (int sw = warp; sw < n_fin; sw += kGThreads / 32) {
      float bv = 0.f;
      int bi = INT_MAX;
      for (int r = lane; r < kBM && row_t + r < p.n; r += 32) {
        const float v = xch[(size_t)sw * kBM + r];
        if (bi == INT_MAX || v > bv) {
          bv = v;
          bi = row_t + r;
        }
      }
      const uint32_t key = bi == INT_MAX ? 0u : order_key(bv);
      const uint32_t kmax = __reduce_max_sync(0xffffffffu, key);
      const uint32_t imin =
          __reduce_min_sync(0xffffffffu, (bi != INT_MAX && key == kmax) ? (uint32_t)bi : 0xffffffffu);
      const float wv = __shfl_sync(0xffffffffu, bv, (int)((imin - (uint32_t)row_t) & 31u));
      if (lane == 0) {
        const int s = s0 + sb + sw;
        p.am_val[(int64_t)s * tiles + tile] = wv;
        p.am_idx[(int64_t)s * tiles + tile] = imin == 0xffffffffu ? INT_MAX : (int)imin;
      }
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) last_cta = atomicAdd(p.am_ticket, 1u) == gridDim.x * gridDim.y - 1;
    __syncthreads();
    if (last_cta) {
      __threadfence();
      // One warp per stream: lanes take tiles lane, lane + 32, ...; the best value, then the
      // lowest row among equals (per-tile candidates are already lowest-row winners).
      for (int s = warp; s < p.nb; s += kGThreads / 32) {
        float bv = 0.f;
        int bi = INT_MAX;
        for (int t = lane; t < tiles; t += 32) {
          const float v = __ldcg(p.am_val + (int64_t)s * tiles + t);
          const int ix = __ldcg(p.am_idx + (int64_t)s * tiles + t);
          if (ix != INT_MAX && better(v, ix, bv, bi)) {
            bv = v;
            bi = ix;
          }
        }
        const uint32_t key = bi == INT_MAX ? 0u : order_key(bv);
        const uint32_t kmax = __reduce_max_sync(0xffffffffu, key);
        const uint32_t imin =
            __reduce_min_sync(0xffffffffu, (bi != INT_MAX && key == kmax) ? (uint32_t)bi : 0xffffffffu);
        if (lane == 0) {
          p.tokens[s] = imin == 0xffffffffu ? 0u : imin;
          if (p.pos_advance) p.pos_advance[s] += 1;
        }
      }
      if (tid == 0) *p.am_ticket = 0u;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::kCols)
                 : "memory");
}

// One CTA per stream: the norm of x[b] (RMS, Layer or none), rounded to bf16 into the GEMM
// operand row out[b][0:k]. Same formulas as the matrix-vector kernel's input prologue.
constexpr int kPrepThreads = 256;
__global__ void __launch_bounds__(kPrepThreads) prep_kernel(const float* x, int64_t x_stride,
                                                            int norm, const float* nw,
                                                            const float* nbias, float eps, int k,
                                                            uint16_t* out, int64_t out_stride,
                                                            int quant, int f16) {
  __shared__ float red[2][kPrepThreads / 32];
  __shared__ float stat[2];
  pdl_launch();
  pdl_wait();
  const int b = blockIdx.x, t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const float* xr = x + b * x_stride;
  uint16_t* o = out + b * out_stride;
  if (norm != NORM_NONE) {
    float s = 0.f, s2 = 0.f;
    for (int i = t * 4; i < k; i += kPrepThreads * 4) {
      const float4 v = __ldcg(reinterpret_cast<const float4*>(xr + i));
      s += v.x + v.y + v.z + v.w;
      s2 += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    }
    s = warp_sum(s);
    s2 = warp_sum(s2);
    if (lane == 0) {
      red[0][warp] = s;
      red[1][warp] = s2;
    }
    __syncthreads();
    if (t == 0) {
      float a = 0.f, c = 0.f;
      for (int w = 0; w < kPrepThreads / 32; w++) {
        a += red[0][w];
        c += red[1][w];
      }
      if (norm == NORM_RMS) {
        stat[0] = sqrtf(c / (float)k + eps);  // candle rms_norm: sqrt(mean(x^2) + eps)
      } else {
        const float mean = a / (float)k;      // candle layer_norm: E[x^2] - mean^2
        stat[0] = mean;
        stat[1] = 1.0f / sqrtf(c / (float)k - mean * mean + eps);
      }
    }
    __syncthreads();
  }
  for (int i = t * 4; i < k; i += kPrepThreads * 4) {
    float4 v = __ldcg(reinterpret_cast<const float4*>(xr + i));
    float e[4] = {v.x, v.y, v.z, v.w};
    if (norm == NORM_RMS) {
      const float4 w = *reinterpret_cast<const float4*>(nw + i);
      const float w4[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int j = 0; j < 4; j++) e[j] = e[j] / stat[0] * w4[j];
    } else if (norm == NORM_LAYER) {
      const float4 w = *reinterpret_cast<const float4*>(nw + i);
      const float4 bb = *reinterpret_cast<const float4*>(nbias + i);
      const float w4[4] = {w.x, w.y, w.z, w.w}, b4[4] = {bb.x, bb.y, bb.z, bb.w};
#pragma unroll
      for (int j = 0; j < 4; j++) e[j] = (e[j] - stat[0]) * stat[1] * w4[j] + b4[j];
    }
    if (quant) {
      // The activation blocks of the quantised dot products (ggml Q8_0 / Q8_1, as candle's
      // QMatMul builds them): d = amax / 127 (stored f16), q = round(x / d); the operand is
      // q * d, the value those products multiply. A block is 8 consecutive threads.
      // (k % 32 == 0: the threads still in this loop form whole 8-thread blocks.)
      const unsigned act = __activemask();
      float amax = fmaxf(fmaxf(fabsf(e[0]), fabsf(e[1])), fmaxf(fabsf(e[2]), fabsf(e[3])));
      amax = fmaxf(amax, __shfl_xor_sync(act, amax, 1));
      amax = fmaxf(amax, __shfl_xor_sync(act, amax, 2));
      amax = fmaxf(amax, __shfl_xor_sync(act, amax, 4));
      const float d = amax / 127.0f;
      const float id = d != 0.0f ? 1.0f / d : 0.0f;
      const float dq = f16_round(d);
#pragma unroll
      for (int j = 0; j < 4; j++) e[j] = dq * (float)(int)roundf(e[j] * id);
    }
    uint2 pk;
    if (f16) {
      __half2 lo = __floats2half2_rn(e[0], e[1]), hi = __floats2half2_rn(e[2], e[3]);
      pk.x = *reinterpret_cast<uint32_t*>(&lo);
      pk.y = *reinterpret_cast<uint32_t*>(&hi);
    } else {
      __nv_bfloat162 lo = __floats2bfloat162_rn(e[0], e[1]), hi = __floats2bfloat162_rn(e[2], e[3]);
      pk.x = *reinterpret_cast<uint32_t*>(&lo);
      pk.y = *reinterpret_cast<uint32_t*>(&hi);
    }
    *reinterpret_cast<uint2*>(o + i) = pk;
  }
}

// ---- host side ----------------------------------------------------------------------------

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                 const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                 const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                 CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encoder() {
  static EncodeTiled fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return (EncodeTiled) nullptr;
    return reinterpret_cast<EncodeTiled>(f);
  }();
  return fn;
}

template <int BN, int EPI>
void launch_be(const GemmOperand& w, const GemmOperand& x, const GemmArgs& ga, int tiles,
               int stream_tiles, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(tiles * ga.split, stream_tiles);
  cfg.blockDim = dim3(kGThreads);
  cfg.dynamicSmemBytes = Cfg<BN>::kSmem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = ga.split;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  cudaLaunchKernelEx(&cfg, gemm_kernel<BN, EPI>, *reinterpret_cast<const CUtensorMap*>(w.map),
                     *reinterpret_cast<const CUtensorMap*>(x.map), ga);
}

template <int BN>
void launch_bn(const GemmOperand& w, const GemmOperand& x, const GemmArgs& ga, int tiles,
               int stream_tiles, cudaStream_t s) {
  switch (ga.p.epi) {
    case EPI_STORE: launch_be<BN, EPI_STORE>(w, x, ga, tiles, stream_tiles, s); break;
    case EPI_RESIDUAL: launch_be<BN, EPI_RESIDUAL>(w, x, ga, tiles, stream_tiles, s); break;
    case EPI_QKV_ROPE: launch_be<BN, EPI_QKV_ROPE>(w, x, ga, tiles, stream_tiles, s); break;
    case EPI_SWIGLU: launch_be<BN, EPI_SWIGLU>(w, x, ga, tiles, stream_tiles, s); break;
    case EPI_GELU_TANH: launch_be<BN, EPI_GELU_TANH>(w, x, ga, tiles, stream_tiles, s); break;
    case EPI_GELU_ERF: launch_be<BN, EPI_GELU_ERF>(w, x, ga, tiles, stream_tiles, s); break;
    case EPI_SILU: launch_be<BN, EPI_SILU>(w, x, ga, tiles, stream_tiles, s); break;
    default: launch_be<BN, EPI_LOGITS>(w, x, ga, tiles, stream_tiles, s); break;
  }
}

template <int BN>
void set_attrs_bn() {
  const int smem = (int)Cfg<BN>::kSmem;
  cudaFuncSetAttribute(gemm_kernel<BN, EPI_STORE>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  cudaFuncSetAttribute(gemm_kernel<BN, EPI_RESIDUAL>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  cudaFuncSetAttribute(gemm_kernel<BN, EPI_QKV_ROPE>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  cudaFuncSetAttribute(gemm_kernel<BN, EPI_SWIGLU>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  cudaFuncSetAttribute(gemm_kernel<BN, EPI_GELU_TANH>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  cudaFuncSetAttribute(gemm_kernel<BN, EPI_GELU_ERF>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  cudaFuncSetAttribute(gemm_kernel<BN, EPI_SILU>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  cudaFuncSetAttribute(gemm_kernel<BN, EPI_LOGITS>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
}

}  // namespace

bool make_gemm_operand(GemmOperand& op, const void* base, int rows, int k, int64_t row_bytes,
                       int box_rows, int f16) {
  static_assert(sizeof(op.map) >= sizeof(CUtensorMap), "tensor map storage");
  EncodeTiled enc = encoder();
  if (!enc || !base || rows <= 0 || k <= 0 || row_bytes % 16 || box_rows > 256 || box_rows < 8 ||
      reinterpret_cast<uintptr_t>(base) % 16)
    return false;
  const cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
  const cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(reinterpret_cast<CUtensorMap*>(op.map),
                   f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                   const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  op.rows = rows;
  op.k = k;
  op.box_rows = box_rows;
  op.f16 = f16;
  op.valid = r == CUDA_SUCCESS;
  return op.valid;
}

bool make_ring_map(unsigned char* map128, const void* base, int64_t rows, int head_dim, int layers,
                   int64_t layer_stride, int box_rows) {
  EncodeTiled enc = encoder();
  if (!enc || !base || rows <= 0 || head_dim % 64 || layers <= 0 || (layer_stride * 2) % 16 ||
      box_rows > 256 || box_rows < 1 || reinterpret_cast<uintptr_t>(base) % 16)
    return false;
  const cuuint64_t dims[3] = {(cuuint64_t)head_dim, (cuuint64_t)rows, (cuuint64_t)layers};
  const cuuint64_t strides[2] = {(cuuint64_t)head_dim * 2, (cuuint64_t)layer_stride * 2};
  const cuuint32_t box[3] = {64, (cuuint32_t)box_rows, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  return enc(reinterpret_cast<CUtensorMap*>(map128), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3,
             const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int gemm_stream_tile(int nb) { return nb > 0 ? 128 : 128; }

int gemm_split(int n, int k, int nb, int bn) {
  const int tiles = (n + kBM - 1) / kBM;
  const int stream_tiles = (nb + bn - 1) / bn;
  const int kblocks = (k + kBK - 1) / kBK;
  const int slots = bn <= 128 ? 2 * 148 : 148;  // resident CTAs of the whole GPU
  int split = slots / (tiles * stream_tiles);
  if (split > kMaxClusterSplit) split = kMaxClusterSplit;
  // Each cluster rank keeps at least 2 K blocks and finishes a 16-wide slice of streams.
  while (split > 1 && (kblocks / split < 2 || (bn / split) % 16 != 0)) split--;
  return split < 1 ? 1 : split;
}

size_t gemm_workspace_bytes() { return (size_t)2 * 148 * 128 * kBM * 4; }

void launch_gemm(const GemvParams& p, const GemmOperand& w, const GemmOperand& x, int x_row0,
                 int out_bf16, int* err, float* ws, cudaStream_t s) {
  GemmArgs ga{};
  ga.p = p;
  ga.kblocks = (p.k + kBK - 1) / kBK;
  ga.split = gemm_split(p.n, p.k, p.nb, x.box_rows);
  ga.x_row0 = x_row0;
  ga.out_bf16 = out_bf16;
  ga.err = err;
  ga.ws = ws;
  ga.idesc = idesc_f16kind(kBM, x.box_rows, w.f16 ? 0u : 1u);
  if (w.f16 != x.f16) return;  // mixed operand types are not an MMA kind::f16 form
  const int bn = x.box_rows;
  const int tiles = (p.n + kBM - 1) / kBM;
  const int stream_tiles = (p.nb + bn - 1) / bn;
  if (bn == 128)
    launch_bn<128>(w, x, ga, tiles, stream_tiles, s);
  else
    launch_bn<256>(w, x, ga, tiles, stream_tiles, s);
}

void launch_prep_bf16(const float* x, int64_t x_stride, int nb, int norm, const float* norm_w,
                      const float* norm_b, float eps, int k, void* out, int64_t out_stride,
                      cudaStream_t s, int quant, int f16) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(nb);
  cfg.blockDim = dim3(kPrepThreads);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (quant && k % 32) quant = 0;  // quantised models have k % 32 == 0
  cudaLaunchKernelEx(&cfg, prep_kernel, x, x_stride, norm, norm_w, norm_b, eps, k,
                     static_cast<uint16_t*>(out), out_stride, quant, f16);
}

void gemm_init_device() {
  set_attrs_bn<128>();
  set_attrs_bn<256>();
}

}  // namespace svl
