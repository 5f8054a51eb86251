// RMSNorm forward/backward (Qwen2RMSNorm with a frozen weight).
//
// Forward (solution/rmsnorm.py:25-39): rstd = 1/sqrt(sum(x^2)/N + eps); xn = x*rstd rounded
// through x's dtype; y = w*xn in the promoted output dtype. Backward (:43-55):
// g = dy*w, dx = rstd*(g - x*(rstd^2 * sum(g*x)/N)).
//
// Forward rows of up to 32 x 16 x 8 = 4096 elements whose rows allow 16-byte accesses take the
// warp-per-row kernel: a warp issues every 16-byte load of its row before it reduces, keeps the
// raw bytes in registers (not floats: half the registers for 2-byte dtypes), reduces with
// shuffles only (no block barrier), and writes the row from the registers - HBM is read once,
// with up to 16 loads in flight per lane. Longer rows, and the backward, take the CTA-per-row
// kernels (VPT 16-byte chunks per thread, a block reduction): in the backward, which holds dy and
// x, a warp-per-row form needs twice the registers and streams slower than the CTA-per-row one.
// Rows whose length or alignment rules out 16-byte chunks take the scalar kernel, which re-reads
// the row from L2 in its second loop.
#include "qb_common.cuh"

namespace {

constexpr int kMaxThreads = 512;

// Eight elements of T as raw bytes (one or two 16-byte words) and their float values.
template <typename T>
struct Chunk8 {
  static constexpr int W = sizeof(T) * 8 / 16;   // 16-byte words: 1 for 2-byte T, 2 for fp32
  uint4 u[W];
  __device__ __forceinline__ void load(const T* p) {
#pragma unroll
    for (int i = 0; i < W; ++i) u[i] = __ldg(reinterpret_cast<const uint4*>(p) + i);
  }
  __device__ __forceinline__ void to_float(float* f) const {
    const T* v = reinterpret_cast<const T*>(u);
#pragma unroll
    for (int e = 0; e < 8; ++e) f[e] = qb::to_f(v[e]);
  }
};

constexpr int kRowWarps = 8;      // rows (warps) per CTA of the warp-per-row kernels
constexpr int kWarpRowMax = 32 * 16 * 8;   // longest row the warp kernels take (CPL <= 16)

// One warp per row; CPL 8-element chunks per lane at most (chunk c of the row is lane c % 32's
// (c / 32)-th), row length a multiple of 8 and <= 256 * CPL.
template <typename XT, typename WT, typename YT, int CPL>
__global__ void __launch_bounds__(kRowWarps * 32)
rmsnorm_fwd_warp(const XT* __restrict__ x, int64_t xs, const WT* __restrict__ w,
                 YT* __restrict__ y, int64_t ys, float* __restrict__ rstd, int64_t rows,
                 int cols, float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kRowWarps + (threadIdx.x >> 5);
  if (row >= rows) return;                       // whole warps leave: no barrier follows
  const int nvec = cols / 8;
  const XT* xr = x + row * xs;
  Chunk8<XT> c[CPL];
#pragma unroll
  for (int j = 0; j < CPL; ++j)
    if (lane + 32 * j < nvec) c[j].load(xr + (lane + 32 * j) * 8);
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < CPL; ++j) {
    if (lane + 32 * j < nvec) {
      float f[8];
      c[j].to_float(f);
#pragma unroll
      for (int e = 0; e < 8; ++e) ss += f[e] * f[e];
    }
  }
  ss = qb::warp_sum(ss);
  const float r = 1.0f / sqrtf(ss / static_cast<float>(cols) + eps);
  if (lane == 0) rstd[row] = r;
  YT* yr = y + row * ys;
#pragma unroll
  for (int j = 0; j < CPL; ++j) {
    const int idx = lane + 32 * j;
    if (idx < nvec) {
      float f[8], wv[8], out[8];
      c[j].to_float(f);
      qb::load8<WT>(w + idx * 8, wv);
#pragma unroll
      for (int e = 0; e < 8; ++e) out[e] = wv[e] * qb::round_through<XT>(f[e] * r);
      qb::store8<YT>(yr + idx * 8, out);
    }
  }
}

template <typename XT, typename WT, typename YT, int VPT>
__global__ void __launch_bounds__(kMaxThreads)
rmsnorm_fwd_vec(const XT* __restrict__ x, int64_t xs, const WT* __restrict__ w,
                YT* __restrict__ y, int64_t ys, float* __restrict__ rstd, int cols, float eps) {
  __shared__ float scratch[32];
  const int64_t row = blockIdx.x;
  const int nvec = cols / 8;
  const XT* xr = x + row * xs;
  float v[VPT][8];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int idx = threadIdx.x + j * blockDim.x;
    if (idx < nvec) {
      qb::load8<XT>(xr + idx * 8, v[j]);
#pragma unroll
      for (int e = 0; e < 8; ++e) ss += v[j][e] * v[j][e];
    }
  }
  ss = qb::block_sum(ss, scratch);
  const float r = 1.0f / sqrtf(ss / static_cast<float>(cols) + eps);
  if (threadIdx.x == 0) rstd[row] = r;
  YT* yr = y + row * ys;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int idx = threadIdx.x + j * blockDim.x;
    if (idx < nvec) {
      float wv[8], out[8];
      qb::load8<WT>(w + idx * 8, wv);
#pragma unroll
      for (int e = 0; e < 8; ++e) out[e] = wv[e] * qb::round_through<XT>(v[j][e] * r);
      qb::store8<YT>(yr + idx * 8, out);
    }
  }
}

template <typename XT, typename WT, typename YT>
__global__ void rmsnorm_fwd_scalar(const XT* __restrict__ x, int64_t xs, const WT* __restrict__ w,
                                   YT* __restrict__ y, int64_t ys, float* __restrict__ rstd,
                                   int cols, float eps) {
  __shared__ float scratch[32];
  const int64_t row = blockIdx.x;
  const XT* xr = x + row * xs;
  float ss = 0.f;
  for (int c = threadIdx.x; c < cols; c += blockDim.x) {
    const float t = qb::to_f(xr[c]);
    ss += t * t;
  }
  ss = qb::block_sum(ss, scratch);
  const float r = 1.0f / sqrtf(ss / static_cast<float>(cols) + eps);
  if (threadIdx.x == 0) rstd[row] = r;
  YT* yr = y + row * ys;
  for (int c = threadIdx.x; c < cols; c += blockDim.x)
    yr[c] = qb::from_f<YT>(qb::to_f(w[c]) * qb::round_through<XT>(qb::to_f(xr[c]) * r));
}

template <typename DYT, typename XT, typename WT, int VPT>
__global__ void __launch_bounds__(kMaxThreads)
rmsnorm_bwd_vec(const DYT* __restrict__ dy, int64_t dys, const XT* __restrict__ x, int64_t xs,
                const WT* __restrict__ w, const float* __restrict__ rstd, XT* __restrict__ dx,
                int64_t dxs, int cols) {
  __shared__ float scratch[32];
  const int64_t row = blockIdx.x;
  const int nvec = cols / 8;
  float g[VPT][8], xv[VPT][8];
  float dot = 0.f;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int idx = threadIdx.x + j * blockDim.x;
    if (idx < nvec) {
      float dv[8], wv[8];
      qb::load8<DYT>(dy + row * dys + idx * 8, dv);
      qb::load8<XT>(x + row * xs + idx * 8, xv[j]);
      qb::load8<WT>(w + idx * 8, wv);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        g[j][e] = dv[e] * wv[e];
        dot += g[j][e] * xv[j][e];
      }
    }
  }
  dot = qb::block_sum(dot, scratch) / static_cast<float>(cols);
  const float r = rstd[row];
  const float c = r * r * dot;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int idx = threadIdx.x + j * blockDim.x;
    if (idx < nvec) {
      float out[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) out[e] = r * (g[j][e] - xv[j][e] * c);
      qb::store8<XT>(dx + row * dxs + idx * 8, out);
    }
  }
}

template <typename DYT, typename XT, typename WT>
__global__ void rmsnorm_bwd_scalar(const DYT* __restrict__ dy, int64_t dys,
                                   const XT* __restrict__ x, int64_t xs, const WT* __restrict__ w,
                                   const float* __restrict__ rstd, XT* __restrict__ dx,
                                   int64_t dxs, int cols) {
  __shared__ float scratch[32];
  const int64_t row = blockIdx.x;
  float dot = 0.f;
  for (int c = threadIdx.x; c < cols; c += blockDim.x)
    dot += qb::to_f(dy[row * dys + c]) * qb::to_f(w[c]) * qb::to_f(x[row * xs + c]);
  dot = qb::block_sum(dot, scratch) / static_cast<float>(cols);
  const float r = rstd[row];
  const float k = r * r * dot;
  for (int c = threadIdx.x; c < cols; c += blockDim.x) {
    const float g = qb::to_f(dy[row * dys + c]) * qb::to_f(w[c]);
    dx[row * dxs + c] = qb::from_f<XT>(r * (g - qb::to_f(x[row * xs + c]) * k));
  }
}

// Chooses VPT (chunks per thread) and the thread count for a row of `cols` elements.
struct RowPlan {
  int vpt = 0;      // 0 = scalar kernel
  int threads = 0;
};

RowPlan plan_row(int64_t cols, bool vec_ok) {
  RowPlan p;
  if (vec_ok && cols % 8 == 0) {
    const int64_t nvec = cols / 8;
    for (int vpt : {1, 2, 4, 8}) {
      if (nvec <= static_cast<int64_t>(vpt) * kMaxThreads) {
        p.vpt = vpt;
        int64_t t = (nvec + vpt - 1) / vpt;
        t = ((t + 31) / 32) * 32;
        p.threads = static_cast<int>(t);
        return p;
      }
    }
  }
  p.vpt = 0;
  p.threads = cols >= 1024 ? 512 : 256;
  return p;
}

bool rows_aligned(const void* p, int64_t row_stride, int esize) {
  return qb::aligned16(p) && (row_stride * esize) % 16 == 0;
}

template <typename XT, typename WT, typename YT>
int fwd_typed(const void* x, int64_t xs, const void* w, void* y, int64_t ys, float* rstd,
              int64_t rows, int64_t cols, float eps, cudaStream_t stream) {
  const bool vec_ok = rows_aligned(x, xs, sizeof(XT)) && rows_aligned(y, ys, sizeof(YT)) &&
                      qb::aligned16(w);
  const auto* xp = static_cast<const XT*>(x);
  const auto* wp = static_cast<const WT*>(w);
  auto* yp = static_cast<YT*>(y);
  const int c = static_cast<int>(cols);
  if constexpr (sizeof(XT) == 2) {
    if (vec_ok && cols % 8 == 0 && cols <= kWarpRowMax) {
      const dim3 wgrid(static_cast<unsigned>((rows + kRowWarps - 1) / kRowWarps));
      if (cols <= 1024)
        rmsnorm_fwd_warp<XT, WT, YT, 4><<<wgrid, kRowWarps * 32, 0, stream>>>(
            xp, xs, wp, yp, ys, rstd, rows, c, eps);
      else
        rmsnorm_fwd_warp<XT, WT, YT, 16><<<wgrid, kRowWarps * 32, 0, stream>>>(
            xp, xs, wp, yp, ys, rstd, rows, c, eps);
      return qb::check_launch("rmsnorm_fwd");
    }
  }
  const RowPlan p = plan_row(cols, vec_ok);
  const dim3 grid(static_cast<unsigned>(rows));
  switch (p.vpt) {
    case 1: rmsnorm_fwd_vec<XT, WT, YT, 1><<<grid, p.threads, 0, stream>>>(xp, xs, wp, yp, ys, rstd, c, eps); break;
    case 2: rmsnorm_fwd_vec<XT, WT, YT, 2><<<grid, p.threads, 0, stream>>>(xp, xs, wp, yp, ys, rstd, c, eps); break;
    case 4: rmsnorm_fwd_vec<XT, WT, YT, 4><<<grid, p.threads, 0, stream>>>(xp, xs, wp, yp, ys, rstd, c, eps); break;
    case 8: rmsnorm_fwd_vec<XT, WT, YT, 8><<<grid, p.threads, 0, stream>>>(xp, xs, wp, yp, ys, rstd, c, eps); break;
    default: rmsnorm_fwd_scalar<XT, WT, YT><<<grid, p.threads, 0, stream>>>(xp, xs, wp, yp, ys, rstd, c, eps);
  }
  return qb::check_launch("rmsnorm_fwd");
}

template <typename DYT, typename XT, typename WT>
int bwd_typed(const void* dy, int64_t dys, const void* x, int64_t xs, const void* w,
              const float* rstd, void* dx, int64_t dxs, int64_t rows, int64_t cols,
              cudaStream_t stream) {
  const bool vec_ok = rows_aligned(dy, dys, sizeof(DYT)) && rows_aligned(x, xs, sizeof(XT)) &&
                      rows_aligned(dx, dxs, sizeof(XT)) && qb::aligned16(w);
  const auto* dyp = static_cast<const DYT*>(dy);
  const auto* xp = static_cast<const XT*>(x);
  const auto* wp = static_cast<const WT*>(w);
  auto* dxp = static_cast<XT*>(dx);
  const int c = static_cast<int>(cols);
  const RowPlan p = plan_row(cols, vec_ok);
  const dim3 grid(static_cast<unsigned>(rows));
  switch (p.vpt) {
    case 1: rmsnorm_bwd_vec<DYT, XT, WT, 1><<<grid, p.threads, 0, stream>>>(dyp, dys, xp, xs, wp, rstd, dxp, dxs, c); break;
    case 2: rmsnorm_bwd_vec<DYT, XT, WT, 2><<<grid, p.threads, 0, stream>>>(dyp, dys, xp, xs, wp, rstd, dxp, dxs, c); break;
    case 4: rmsnorm_bwd_vec<DYT, XT, WT, 4><<<grid, p.threads, 0, stream>>>(dyp, dys, xp, xs, wp, rstd, dxp, dxs, c); break;
    case 8: rmsnorm_bwd_vec<DYT, XT, WT, 8><<<grid, p.threads, 0, stream>>>(dyp, dys, xp, xs, wp, rstd, dxp, dxs, c); break;
    default: rmsnorm_bwd_scalar<DYT, XT, WT><<<grid, p.threads, 0, stream>>>(dyp, dys, xp, xs, wp, rstd, dxp, dxs, c);
  }
  return qb::check_launch("rmsnorm_bwd");
}

int check_common(const void* a, const void* b, const void* c, const void* d, int64_t rows,
                 int64_t cols, const char* what) {
  if (rows < 0 || cols <= 0 || cols > (1 << 30) || rows > 0x7fffffff)
    return qb::fail(QB_ERR_INVALID, "%s: bad shape rows=%lld cols=%lld", what, (long long)rows, (long long)cols);
  if (rows > 0 && (!a || !b || !c || !d)) return qb::fail(QB_ERR_INVALID, "%s: null pointer", what);
  return QB_OK;
}

}  // namespace

extern "C" int qb_rmsnorm_fwd(const void* x, int x_dtype, int64_t x_row_stride, const void* w,
                              int w_dtype, void* y, int y_dtype, int64_t y_row_stride,
                              float* rstd, int64_t rows, int64_t cols, float eps,
                              cudaStream_t stream) {
  if (int s = check_common(x, w, y, rstd, rows, cols, "rmsnorm_fwd")) return s;
  if (rows == 0) return QB_OK;
  QB_DISPATCH_FLOAT(x_dtype, XT, {
    QB_DISPATCH_FLOAT(w_dtype, WT, {
      QB_DISPATCH_FLOAT(y_dtype, YT, {
        return fwd_typed<XT, WT, YT>(x, x_row_stride, w, y, y_row_stride, rstd, rows, cols, eps,
                                     stream);
      });
    });
  });
}

extern "C" int qb_rmsnorm_bwd(const void* dy, int dy_dtype, int64_t dy_row_stride,
                              const void* x, int x_dtype, int64_t x_row_stride, const void* w,
                              int w_dtype, const float* rstd, void* dx, int dx_dtype,
                              int64_t dx_row_stride, int64_t rows, int64_t cols,
                              cudaStream_t stream) {
  if (int s = check_common(dy, x, w, dx, rows, cols, "rmsnorm_bwd")) return s;
  if (!rstd && rows) return qb::fail(QB_ERR_INVALID, "rmsnorm_bwd: null rstd");
  if (dx_dtype != x_dtype) return qb::fail(QB_ERR_INVALID, "rmsnorm_bwd: dx must have x's dtype");
  if (rows == 0) return QB_OK;
  QB_DISPATCH_FLOAT(dy_dtype, DYT, {
    QB_DISPATCH_FLOAT(x_dtype, XT, {
      QB_DISPATCH_FLOAT(w_dtype, WT, {
        return bwd_typed<DYT, XT, WT>(dy, dy_row_stride, x, x_row_stride, w, rstd, dx,
                                      dx_row_stride, rows, cols, stream);
      });
    });
  });
}
