// Element loads shared by the forward kernels (forward.cu, prefill.cu).
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "common.cuh"

namespace skcq {

__device__ __forceinline__ float ld_any(const void* p, int64_t i, int dtype) {
  if (dtype == SKCQ_DTYPE_BF16) return __uint_as_float((uint32_t) static_cast<const uint16_t*>(p)[i] << 16);
  return static_cast<const float*>(p)[i];
}
// Stored scale -> f32 (codebook_experts.py:328-331: int scales times scale_q_scale).
__device__ __forceinline__ float ld_scale(const void* p, int64_t i, int dtype, float q_scale) {
  switch (dtype) {
    case SKCQ_DTYPE_BF16: return __uint_as_float((uint32_t) static_cast<const uint16_t*>(p)[i] << 16);
    case SKCQ_DTYPE_F16: return __half2float(static_cast<const __half*>(p)[i]);
    case SKCQ_DTYPE_I8: return __fmul_rn((float)static_cast<const int8_t*>(p)[i], q_scale);
    case SKCQ_DTYPE_I16: return __fmul_rn((float)static_cast<const int16_t*>(p)[i], q_scale);
    default: return static_cast<const float*>(p)[i];
  }
}

__device__ __forceinline__ void st_any(void* p, int64_t i, int dtype, float v) {
  if (dtype == SKCQ_DTYPE_BF16) {
    __nv_bfloat16 h = __float2bfloat16_rn(v);
    static_cast<uint16_t*>(p)[i] = *reinterpret_cast<uint16_t*>(&h);
  } else {
    static_cast<float*>(p)[i] = v;
  }
}

// Elements [i, i + 8) of a bf16 array (i * 2 bytes 16-byte aligned) -> f32.
__device__ __forceinline__ void ld_bf16x8(const void* p, int64_t i, float (&v)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p) + i);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    v[2 * j] = __uint_as_float(w[j] << 16);
    v[2 * j + 1] = __uint_as_float(w[j] & 0xffff0000u);
  }
}

// Elements [i, i + 8) of an f32 | bf16 array (16-byte aligned), rounded as st_any.
__device__ __forceinline__ void st_x8(void* p, int64_t i, int dtype, const float (&v)[8]) {
  if (dtype == SKCQ_DTYPE_BF16) {
    uint32_t w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      __nv_bfloat16 lo = __float2bfloat16_rn(v[2 * j]), hi = __float2bfloat16_rn(v[2 * j + 1]);
      w[j] = (uint32_t)*reinterpret_cast<uint16_t*>(&lo) | ((uint32_t)*reinterpret_cast<uint16_t*>(&hi) << 16);
    }
    *reinterpret_cast<uint4*>(static_cast<uint16_t*>(p) + i) = make_uint4(w[0], w[1], w[2], w[3]);
  } else {
    float4* q = reinterpret_cast<float4*>(static_cast<float*>(p) + i);
    q[0] = make_float4(v[0], v[1], v[2], v[3]);
    q[1] = make_float4(v[4], v[5], v[6], v[7]);
  }
}

// Centroid vector of BS elements at p -> f32 registers, with the widest
// aligned vector loads (p is aligned to BS * sizeof(T)).
template <int BS, typename T>
__device__ __forceinline__ void load_centroid(const T* __restrict__ p, float (&w)[BS]) {
  constexpr int BYTES = BS * (int)sizeof(T);
  if constexpr (BYTES % 4 == 0) {
    uint32_t u[BYTES / 4];
    if constexpr (BYTES % 16 == 0) {
#pragma unroll
      for (int i = 0; i < BYTES / 16; ++i) {
        const uint4 v = __ldg(reinterpret_cast<const uint4*>(p) + i);
        u[4 * i] = v.x, u[4 * i + 1] = v.y, u[4 * i + 2] = v.z, u[4 * i + 3] = v.w;
      }
    } else if constexpr (BYTES % 8 == 0) {
#pragma unroll
      for (int i = 0; i < BYTES / 8; ++i) {
        const uint2 v = __ldg(reinterpret_cast<const uint2*>(p) + i);
        u[2 * i] = v.x, u[2 * i + 1] = v.y;
      }
    } else {
#pragma unroll
      for (int i = 0; i < BYTES / 4; ++i) u[i] = __ldg(reinterpret_cast<const uint32_t*>(p) + i);
    }
    if constexpr (sizeof(T) == 4) {
#pragma unroll
      for (int j = 0; j < BS; ++j) w[j] = __uint_as_float(u[j]);
    } else {
#pragma unroll
      for (int j = 0; j < BS; ++j) w[j] = __uint_as_float((j & 1) ? (u[j >> 1] & 0xffff0000u) : (u[j >> 1] << 16));
    }
  } else {
#pragma unroll
    for (int j = 0; j < BS; ++j) w[j] = __uint_as_float((uint32_t)__ldg(reinterpret_cast<const uint16_t*>(p) + j) << 16);
  }
}

}  // namespace skcq
