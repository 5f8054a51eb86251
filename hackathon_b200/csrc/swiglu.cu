// SwiGLU forward/backward over flat contiguous tensors (solution/swiglu.py:15-37), fp32 math.
// 8 elements per thread per step (16-byte accesses for 2-byte dtypes), grid-stride over a grid
// sized to the SM count; a scalar tail handles the last n % 8 elements.
#include "qb_common.cuh"

namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ float sigmoidf_(float g) { return 1.0f / (1.0f + __expf(-g)); }

template <typename T>
__global__ void __launch_bounds__(kThreads)
swiglu_fwd_kernel(const T* __restrict__ gate, const T* __restrict__ up, T* __restrict__ out,
                  int64_t n) {
  const int64_t nvec = n / 8;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kThreads;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; i < nvec;
       i += stride) {
    float g[8], u[8], o[8];
    qb::load8<T>(gate + i * 8, g);
    qb::load8<T>(up + i * 8, u);
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = g[e] * sigmoidf_(g[e]) * u[e];
    qb::store8<T>(out + i * 8, o);
  }
  for (int64_t i = nvec * 8 + static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; i < n;
       i += stride) {
    const float g = qb::to_f(gate[i]), u = qb::to_f(up[i]);
    out[i] = qb::from_f<T>(g * sigmoidf_(g) * u);
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads)
swiglu_bwd_kernel(const T* __restrict__ grad, const T* __restrict__ gate, const T* __restrict__ up,
                  T* __restrict__ dgate, T* __restrict__ dup, int64_t n) {
  const int64_t nvec = n / 8;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kThreads;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; i < nvec;
       i += stride) {
    float d[8], g[8], u[8], dg[8], du[8];
    qb::load8<T>(grad + i * 8, d);
    qb::load8<T>(gate + i * 8, g);
    qb::load8<T>(up + i * 8, u);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float sg = sigmoidf_(g[e]);
      du[e] = d[e] * g[e] * sg;
      dg[e] = d[e] * u[e] * sg * (1.0f + g[e] * (1.0f - sg));
    }
    qb::store8<T>(dgate + i * 8, dg);
    qb::store8<T>(dup + i * 8, du);
  }
  for (int64_t i = nvec * 8 + static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; i < n;
       i += stride) {
    const float d = qb::to_f(grad[i]), g = qb::to_f(gate[i]), u = qb::to_f(up[i]);
    const float sg = sigmoidf_(g);
    dup[i] = qb::from_f<T>(d * g * sg);
    dgate[i] = qb::from_f<T>(d * u * sg * (1.0f + g * (1.0f - sg)));
  }
}

unsigned grid_for(int64_t nvec) {
  int64_t g = (nvec + kThreads - 1) / kThreads;
  const int64_t cap = 148 * 16;  // 16 CTAs of 256 threads per SM: 4096 threads, full occupancy x2
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return static_cast<unsigned>(g);
}

}  // namespace

extern "C" int qb_swiglu_fwd(const void* gate, const void* up, void* out, int dtype, int64_t n,
                             cudaStream_t stream) {
  if (n < 0) return qb::fail(QB_ERR_INVALID, "swiglu_fwd: n < 0");
  if (n == 0) return QB_OK;
  if (!gate || !up || !out) return qb::fail(QB_ERR_INVALID, "swiglu_fwd: null pointer");
  if (!qb::aligned16(gate) || !qb::aligned16(up) || !qb::aligned16(out))
    return qb::fail(QB_ERR_INVALID, "swiglu_fwd: pointers must be 16-byte aligned");
  QB_DISPATCH_FLOAT(dtype, T, {
    swiglu_fwd_kernel<T><<<grid_for(n / 8 + 1), kThreads, 0, stream>>>(
        static_cast<const T*>(gate), static_cast<const T*>(up), static_cast<T*>(out), n);
  });
  return qb::check_launch("swiglu_fwd");
}

extern "C" int qb_swiglu_bwd(const void* grad, const void* gate, const void* up, void* dgate,
                             void* dup, int dtype, int64_t n, cudaStream_t stream) {
  if (n < 0) return qb::fail(QB_ERR_INVALID, "swiglu_bwd: n < 0");
  if (n == 0) return QB_OK;
  if (!grad || !gate || !up || !dgate || !dup) return qb::fail(QB_ERR_INVALID, "swiglu_bwd: null pointer");
  if (!qb::aligned16(grad) || !qb::aligned16(gate) || !qb::aligned16(up) ||
      !qb::aligned16(dgate) || !qb::aligned16(dup))
    return qb::fail(QB_ERR_INVALID, "swiglu_bwd: pointers must be 16-byte aligned");
  QB_DISPATCH_FLOAT(dtype, T, {
    swiglu_bwd_kernel<T><<<grid_for(n / 8 + 1), kThreads, 0, stream>>>(
        static_cast<const T*>(grad), static_cast<const T*>(gate), static_cast<const T*>(up),
        static_cast<T*>(dgate), static_cast<T*>(dup), n);
  });
  return qb::check_launch("swiglu_bwd");
}
