// common.cuh — device helpers shared by the sm_100a kernels of the streaming LM step.
//
// The library is compiled with -fmad=false: a*b+c is never contracted implicitly, so the
// element-wise arithmetic rounds like the reference CPU path (Rust never contracts).
// Kernels ask for FMAs explicitly with fmaf() where they want them.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace svl {

enum WeightType { W_F32 = 0, W_BF16 = 1, W_Q8 = 2, W_Q4 = 3 };
enum NormKind { NORM_NONE = 0, NORM_RMS = 1, NORM_LAYER = 2 };

constexpr int QBLK = 32;  // quantisation block (ggml QK8_0 / QK4_1)

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ int warp_sum_int(int v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// exp as the reference CPU kernels compute it (nn/kernels/mod.rs:96-131): Cody-Waite
// reduction x = k ln2 + r with ln2 split in two parts, expm1(r) by its degree-8 Taylor
// polynomial in Horner form, 2^k assembled in the exponent field. Restated from that
// source so the GPU softmax and SiLU round like the reference's.
__device__ __forceinline__ float exp_ref(float x) {
  const float LN2_HI = 0.69314575f;
  const float LN2_LO = 1.4286068e-6f;
  const float ROUND = 12582912.0f;
  const float LOG2E = 1.44269504088896340736f;
  float c = x != x ? x : fminf(fmaxf(x, -87.0f), 88.0f);
  float shifted = fmaf(c, LOG2E, ROUND);
  float k = __fsub_rn(shifted, ROUND);
  int k_int = (int)(__float_as_uint(shifted) - __float_as_uint(ROUND));
  float r = fmaf(-k, LN2_LO, fmaf(-k, LN2_HI, c));
  float p = 1.0f / 40320.0f;
  p = fmaf(p, r, 1.0f / 5040.0f);
  p = fmaf(p, r, 1.0f / 720.0f);
  p = fmaf(p, r, 1.0f / 120.0f);
  p = fmaf(p, r, 1.0f / 24.0f);
  p = fmaf(p, r, 1.0f / 6.0f);
  p = fmaf(p, r, 0.5f);
  p = fmaf(p, r, 1.0f);
  float two_k = __uint_as_float((uint32_t)(k_int + 127) << 23);
  float y = fmaf(two_k, __fmul_rn(p, r), two_k);
  if (x > 88.72f) y = __int_as_float(0x7f800000);
  return x < -87.0f ? 0.0f : y;
}

// Activation::Silu and GeluTanh (nn/kernels/activation.rs:71-83).
__device__ __forceinline__ float silu_ref(float x) { return __fdiv_rn(x, 1.0f + exp_ref(-x)); }
__device__ __forceinline__ float gelu_tanh_ref(float x) {
  float y = 0.7978846f * fmaf(0.044715f * x, x * x, x);
  return __fdiv_rn(x, 1.0f + exp_ref(-2.0f * y));
}
__device__ __forceinline__ float gelu_erf_ref(float x) {
  double v = x;
  return (float)((v * (1.0 + erf(v * 0.70710678118654752440))) / 2.0);
}

// 16-byte streaming load: weights are read once per step, so keep them out of L1.
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ float bf16_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }
__device__ __forceinline__ float round_bf16(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}
__device__ __forceinline__ float f16_round(float x) { return __half2float(__float2half_rn(x)); }

}  // namespace svl
