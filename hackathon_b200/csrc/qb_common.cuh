// Shared definitions of the qlora_b200 kernel library: status codes, the dtype tags the C-ABI
// uses, the per-thread error message and small device helpers (conversions, warp/block sums).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "qlora_b200.h"

namespace qb {

// Records a message for qb_last_error() and returns the status, so call sites read
// `return fail(QB_ERR_INVALID, "...")`.
int fail(int status, const char* fmt, ...);

// Checks the launch that just happened on this thread; converts a CUDA error into a status.
int check_launch(const char* what);

inline int elem_size(int dtype) {
  return dtype == QB_F32 ? 4 : (dtype == QB_F16 || dtype == QB_BF16) ? 2 : 0;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---------------------------------------------------------------------------------------------
// element conversions (fp32 math, round-to-nearest-even on the way out)

template <typename T> struct Dt;
template <> struct Dt<float> {
  static __device__ __forceinline__ float to_f(float v) { return v; }
  static __device__ __forceinline__ float from_f(float v) { return v; }
};
template <> struct Dt<__half> {
  static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
};
template <> struct Dt<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
};

template <typename T> __device__ __forceinline__ float to_f(T v) { return Dt<T>::to_f(v); }
template <typename T> __device__ __forceinline__ T from_f(float v) { return Dt<T>::from_f(v); }

// A 16-byte vector of T: VEC elements.
template <typename T> struct Vec16 {
  static constexpr int N = 16 / sizeof(T);
  union { uint4 u; T v[16 / sizeof(T)]; };
};

template <typename T>
__device__ __forceinline__ void load16(const T* p, float* out) {
  Vec16<T> x;
  x.u = *reinterpret_cast<const uint4*>(p);
#pragma unroll
  for (int i = 0; i < Vec16<T>::N; ++i) out[i] = to_f(x.v[i]);
}

template <typename T>
__device__ __forceinline__ void store16(T* p, const float* in) {
  Vec16<T> x;
#pragma unroll
  for (int i = 0; i < Vec16<T>::N; ++i) x.v[i] = from_f<T>(in[i]);
  *reinterpret_cast<uint4*>(p) = x.u;
}

// Eight consecutive elements of T (one 16-byte access for 2-byte types, two for fp32); the
// pointer must be 16-byte aligned.
template <typename T>
__device__ __forceinline__ void load8(const T* p, float* out) {
  if constexpr (sizeof(T) == 4) {
    load16<T>(p, out);
    load16<T>(p + 4, out + 4);
  } else {
    load16<T>(p, out);
  }
}

template <typename T>
__device__ __forceinline__ void store8(T* p, const float* in) {
  if constexpr (sizeof(T) == 4) {
    store16<T>(p, in);
    store16<T>(p + 4, in + 4);
  } else {
    store16<T>(p, in);
  }
}

// Rotate-half RoPE on one (first half, second half) pair of a head, every product and sum
// rounded on its own (no contraction into a fused multiply-add), so the RoPE kernel and the
// projection epilogue that applies it produce the same bits:
//   forward  o1 = x1 c1 - x2 s1,  o2 = x2 c2 + x1 s2;   backward  o1 = x1 c1 + x2 s2,  o2 = x2 c2 - x1 s1
__device__ __forceinline__ void rope_rotate(float x1, float x2, float c1, float c2, float s1,
                                            float s2, float& o1, float& o2) {
  o1 = __fsub_rn(__fmul_rn(x1, c1), __fmul_rn(x2, s1));
  o2 = __fadd_rn(__fmul_rn(x2, c2), __fmul_rn(x1, s2));
}

__device__ __forceinline__ void rope_rotate_t(float x1, float x2, float c1, float c2, float s1,
                                              float s2, float& o1, float& o2) {
  o1 = __fadd_rn(__fmul_rn(x1, c1), __fmul_rn(x2, s2));
  o2 = __fsub_rn(__fmul_rn(x2, c2), __fmul_rn(x1, s1));
}

// Rounds v through T's precision and back (identity for fp32).
template <typename T>
__device__ __forceinline__ float round_through(float v) {
  if constexpr (sizeof(T) == 4) return v;
  else return to_f(from_f<T>(v));
}

// ---------------------------------------------------------------------------------------------
// reductions

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

// Sum over the whole block; every thread gets the result. `scratch` holds >= 32 floats.
__device__ __forceinline__ float block_sum(float v, float* scratch) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();  // scratch may still be read by a previous call
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float t = lane < nwarps ? scratch[lane] : 0.f;
  return warp_sum(t);
}

}  // namespace qb

// Dispatch over the three floating dtypes of the C-ABI.
#define QB_DISPATCH_FLOAT(dtype, T, ...)                                     \
  do {                                                                       \
    if ((dtype) == QB_F32) { using T = float; __VA_ARGS__; }                 \
    else if ((dtype) == QB_F16) { using T = __half; __VA_ARGS__; }           \
    else if ((dtype) == QB_BF16) { using T = __nv_bfloat16; __VA_ARGS__; }   \
    else return qb::fail(QB_ERR_INVALID, "unsupported dtype %d", (int)(dtype)); \
  } while (0)
