// Device helpers shared by the kernels.
#pragma once
#include <cuda_bf16.h>
#include <cstdint>
#include "kernels.h"

namespace qasr {

__device__ __forceinline__ float bf16_bits_to_f32(uint32_t bits16) { return __uint_as_float(bits16 << 16); }

__device__ __forceinline__ void bf16x8_to_f32(const uint4& v, float* f) {
  f[0] = __uint_as_float(v.x << 16);
  f[1] = __uint_as_float(v.x & 0xFFFF0000u);
  f[2] = __uint_as_float(v.y << 16);
  f[3] = __uint_as_float(v.y & 0xFFFF0000u);
  f[4] = __uint_as_float(v.z << 16);
  f[5] = __uint_as_float(v.z & 0xFFFF0000u);
  f[6] = __uint_as_float(v.w << 16);
  f[7] = __uint_as_float(v.w & 0xFFFF0000u);
}

// Tanh GELU with the reference's constants (kernels/mod.rs:1283-1288), exact tanhf.
__device__ __forceinline__ float gelu_tanh(float x) {
  float x3 = __fmul_rn(__fmul_rn(x, x), x);
  float inner = __fmul_rn(0.7978845608028654f, __fadd_rn(x, __fmul_rn(0.044715f, x3)));
  return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, tanhf(inner)));
}

// silu(g) * u = g / (1 + exp(-g)) * u (kernels/mod.rs:1335-1337).
__device__ __forceinline__ float silu_mul(float g, float u) {
  return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
}

// f32 -> three bf16 planes with v = hi + mid + lo: each plane is the bf16 rounding of what
// the planes before it left over (both subtractions are exact), so together they hold all 24
// significand bits of v. The tensor-core GEMM multiplies each plane by bf16 weights.
__device__ __forceinline__ void split3_bf16(float v, __nv_bfloat16& hi, __nv_bfloat16& mid, __nv_bfloat16& lo) {
  hi = __float2bfloat16_rn(v);
  const float r = __fsub_rn(v, __bfloat162float(hi));
  mid = __float2bfloat16_rn(r);
  lo = __float2bfloat16_rn(__fsub_rn(r, __bfloat162float(mid)));
}

// Monotonic float <-> int mapping for atomicMax on floats.
__device__ __forceinline__ int float_to_ordered(float f) {
  int i = __float_as_int(f);
  return i >= 0 ? i : i ^ 0x7FFFFFFF;
}
__device__ __forceinline__ float ordered_to_float(int i) { return __int_as_float(i >= 0 ? i : i ^ 0x7FFFFFFF); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Block-wide sum/max for blockDim.x <= 1024; `red` needs 32 floats of shared memory.
__device__ __forceinline__ float block_sum(float v, float* red) {
  int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  float t = lane < nw ? red[lane] : 0.f;
  return warp_sum(t);
}
__device__ __forceinline__ float block_max(float v, float* red) {
  int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  float t = lane < nw ? red[lane] : -3.0e38f;
  return warp_max(t);
}

__device__ __forceinline__ float apply_epi(const GemmArgs& a, int m, int n, float v) {
  switch (a.epi) {
    case EPI_BIAS:
      return __fadd_rn(v, a.bias[n]);
    case EPI_BIAS_GELU:
      return gelu_tanh(__fadd_rn(v, a.bias[n]));
    case EPI_RESID: {
      float r = a.resid[(size_t)m * a.ldr + n];
      if (a.bias) r = __fadd_rn(r, a.bias[n]);
      return __fadd_rn(v, r);
    }
    case EPI_LOG10_MAX: {
      float l = log10f(fmaxf(v, 1e-10f));
      atomicMax(a.gmax, float_to_ordered(l));
      return l;
    }
    default:
      return v;
  }
}

// Streaming 16-byte load that does not allocate in L1 (weights are read once per step).
__device__ __forceinline__ uint4 ld_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

}  // namespace qasr
