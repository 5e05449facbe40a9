// common.cuh — element types, conversions and the device-side error word.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>

#include "starkv.h"

namespace starkv {

// Error codes a kernel writes into the first word of the workspace (0 = none).
enum DeviceError : int {
  kDevOk = 0,
  kDevWaitCopy = 0x101,     // bulk copy never completed
  kDevWaitMma = 0x102,      // MMA commit never arrived
};

__device__ __forceinline__ void record_error(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

template <typename T>
__device__ __forceinline__ float to_f32(T x);
template <>
__device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ float to_f32<__half>(__half x) { return __half2float(x); }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <>
__device__ __forceinline__ float to_f32<int8_t>(int8_t x) { return (float)x; }

template <typename T>
__device__ __forceinline__ T from_f32(float x);
template <>
__device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

// Load element i of a dtype-tagged array as float.
__device__ __forceinline__ float load_as_f32(const void* p, int dtype, int64_t i) {
  switch (dtype) {
    case STARKV_F16: return __half2float(reinterpret_cast<const __half*>(p)[i]);
    case STARKV_BF16: return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
    default: return reinterpret_cast<const float*>(p)[i];
  }
}

__device__ __forceinline__ void store_from_f32(void* p, int dtype, int64_t i, float v) {
  switch (dtype) {
    case STARKV_F16: reinterpret_cast<__half*>(p)[i] = __float2half_rn(v); break;
    case STARKV_BF16: reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v); break;
    default: reinterpret_cast<float*>(p)[i] = v; break;
  }
}

__host__ __device__ __forceinline__ int dtype_bytes(int dtype) { return dtype == STARKV_F32 ? 4 : 2; }

// Element index of K latent / code (b, slot, c) of KV head kv (element size eb
// bytes).  Row-major: rows of r elements.  Tiled (lay.k_tiled): tiles of 128
// slots, each stored as r*eb/16 column chunks of 128 rows x 16 bytes, so that
// one 16-byte chunk of consecutive rows is contiguous.
__host__ __device__ __forceinline__ int64_t k_elem(const starkv_layout& l, int kv, int b, int64_t slot, int c,
                                                   int eb) {
  const int64_t base = l.k_offset[kv] + (int64_t)b * l.k_batch_stride[kv];
  const int r = l.k_rank[kv];
  if (!l.k_tiled) return base + slot * r + c;
  const int per = 16 / eb;
  return base + (slot >> 7) * 128 * r + (int64_t)(c / per) * 128 * per + (slot & 127) * per + (c % per);
}

// Combine two (max, sum-of-exp2) softmax partials in log2 domain.
__device__ __forceinline__ void softmax_merge(float& m, float& l, float m2, float l2) {
  const float mn = fmaxf(m, m2);
  l = l * exp2f(m - mn) + l2 * exp2f(m2 - mn);
  m = mn;
}

// Atomic maximum of a float in global memory (sign-split integer atomics on the
// IEEE bit pattern: non-negative floats order like signed ints, negative ones
// like reversed unsigned ints).
__device__ __forceinline__ void atomic_max_float(float* addr, float v) {
  if (v >= 0.f)
    atomicMax(reinterpret_cast<int*>(addr), __float_as_int(v));
  else
    atomicMin(reinterpret_cast<unsigned int*>(addr), __float_as_uint(v));
}

// Finite "minus infinity" so that (m - m) never produces NaN.
constexpr float kNegBig = -1.0e30f;

}  // namespace starkv
