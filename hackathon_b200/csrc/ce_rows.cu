// Cross-entropy statistics (and the logits gradient, in place) over rows of materialised logits:
// the chunked path of solution/cross_entropy.py:48-90 and solution/fused_ce.py:42-96.
//
// One CTA per row. Pass 1 streams the row once with 16-byte loads; every thread keeps an online
// (max m, sum e = exp(z-m), sum e*z, first argmax) over its elements, rescaling once per chunk of
// 8, and the block merges the partial states. lse = m + log(s), entropy = lse - t/s,
// loss = lse - z[label] for labelled rows. Pass 2 (write_grad) rewrites the row with
// (exp(z - lse) - onehot) * scale, scale = grad_scale for labelled rows and 0 otherwise.
#include <cfloat>

#include "qb_common.cuh"

namespace {

constexpr int kThreads = 512;

struct RowStat {
  float m, s, t;    // running max, sum exp(z - m), sum exp(z - m) * z
  float best;       // argmax value
  int64_t idx;      // argmax index (first occurrence)
};

__device__ __forceinline__ void merge(RowStat& a, const RowStat& b) {
  if (b.best > a.best || (b.best == a.best && b.idx < a.idx)) {
    a.best = b.best;
    a.idx = b.idx;
  }
  const float m = fmaxf(a.m, b.m);
  if (m == -INFINITY) return;  // both empty
  const float fa = __expf(a.m - m), fb = __expf(b.m - m);
  a.s = a.s * fa + b.s * fb;
  a.t = a.t * fa + b.t * fb;
  a.m = m;
}

__device__ __forceinline__ void add_chunk(RowStat& st, const float* z, int n, int64_t first) {
  float cm = z[0];
  for (int e = 1; e < n; ++e) cm = fmaxf(cm, z[e]);
  for (int e = 0; e < n; ++e)
    if (z[e] > st.best) { st.best = z[e]; st.idx = first + e; }
  const float m = fmaxf(st.m, cm);
  const float f = __expf(st.m - m);  // 0 when st.m == -inf
  float s = 0.f, t = 0.f;
  for (int e = 0; e < n; ++e) {
    const float x = __expf(z[e] - m);
    s += x;
    t += x * z[e];
  }
  st.s = st.s * f + s;
  st.t = st.t * f + t;
  st.m = m;
}

__device__ RowStat block_merge(RowStat st) {
  __shared__ float sm[32], ss[32], stt[32], sb[32];
  __shared__ int64_t si[32];
  // warp level
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    RowStat other;
    other.m = __shfl_xor_sync(0xffffffffu, st.m, o);
    other.s = __shfl_xor_sync(0xffffffffu, st.s, o);
    other.t = __shfl_xor_sync(0xffffffffu, st.t, o);
    other.best = __shfl_xor_sync(0xffffffffu, st.best, o);
    other.idx = __shfl_xor_sync(0xffffffffu, st.idx, o);
    merge(st, other);
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) { sm[warp] = st.m; ss[warp] = st.s; stt[warp] = st.t; sb[warp] = st.best; si[warp] = st.idx; }
  __syncthreads();
  const int nw = blockDim.x >> 5;
  RowStat r{-INFINITY, 0.f, 0.f, -INFINITY, INT64_MAX};
  if (lane < nw) r = RowStat{sm[lane], ss[lane], stt[lane], sb[lane], si[lane]};
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    RowStat other;
    other.m = __shfl_xor_sync(0xffffffffu, r.m, o);
    other.s = __shfl_xor_sync(0xffffffffu, r.s, o);
    other.t = __shfl_xor_sync(0xffffffffu, r.t, o);
    other.best = __shfl_xor_sync(0xffffffffu, r.best, o);
    other.idx = __shfl_xor_sync(0xffffffffu, r.idx, o);
    merge(r, other);
  }
  return r;
}

template <typename T, int VEC>
__global__ void __launch_bounds__(kThreads)
ce_rows_kernel(T* __restrict__ logits, int64_t row_stride, const int64_t* __restrict__ target,
               int64_t vocab, float* __restrict__ loss, float* __restrict__ entropy,
               int64_t* __restrict__ pred, int32_t* __restrict__ correct, float grad_scale,
               int write_grad) {
  const int64_t row = blockIdx.x;
  T* z = logits + row * row_stride;
  const int64_t label = target[row];
  const bool labelled = label >= 0 && label < vocab;
  RowStat st{-INFINITY, 0.f, 0.f, -INFINITY, INT64_MAX};
  const int64_t nvec = vocab / VEC;
  for (int64_t v = threadIdx.x; v < nvec; v += kThreads) {
    float x[VEC];
    if constexpr (VEC == 8) qb::load8<T>(z + v * VEC, x);
    else x[0] = qb::to_f(z[v]);
    add_chunk(st, x, VEC, v * VEC);
  }
  for (int64_t c = nvec * VEC + threadIdx.x; c < vocab; c += kThreads) {
    float x = qb::to_f(z[c]);
    add_chunk(st, &x, 1, c);
  }
  const RowStat r = block_merge(st);
  const float lse = r.m + logf(r.s);
  if (threadIdx.x == 0) {
    const float zl = labelled ? qb::to_f(z[label]) : 0.f;
    loss[row] = labelled ? lse - zl : 0.f;
    entropy[row] = lse - r.t / r.s;
    if (pred) pred[row] = r.idx;
    if (correct) correct[row] = (labelled && r.idx == label) ? 1 : 0;
  }
  if (!write_grad) return;
  __syncthreads();  // z[label] is read above before it is overwritten below
  const float scale = labelled ? grad_scale : 0.f;
  for (int64_t v = threadIdx.x; v < nvec; v += kThreads) {
    float x[VEC];
    if constexpr (VEC == 8) qb::load8<T>(z + v * VEC, x);
    else x[0] = qb::to_f(z[v]);
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      const int64_t col = v * VEC + e;
      x[e] = (__expf(x[e] - lse) - (col == label ? 1.f : 0.f)) * scale;
    }
    if constexpr (VEC == 8) qb::store8<T>(z + v * VEC, x);
    else z[v] = qb::from_f<T>(x[0]);
  }
  for (int64_t c = nvec * VEC + threadIdx.x; c < vocab; c += kThreads) {
    const float x = qb::to_f(z[c]);
    z[c] = qb::from_f<T>((__expf(x - lse) - (c == label ? 1.f : 0.f)) * scale);
  }
}

}  // namespace

extern "C" int qb_ce_rows(void* logits, int logits_dtype, int64_t row_stride,
                          const int64_t* target, int64_t rows, int64_t vocab, float* loss,
                          float* entropy, int64_t* pred, int32_t* correct, float grad_scale,
                          int write_grad, cudaStream_t stream) {
  if (rows < 0 || vocab <= 0 || rows > 0x7fffffff) return qb::fail(QB_ERR_INVALID, "ce_rows: bad shape");
  if (rows == 0) return QB_OK;
  if (!logits || !target || !loss || !entropy) return qb::fail(QB_ERR_INVALID, "ce_rows: null pointer");
  QB_DISPATCH_FLOAT(logits_dtype, T, {
    const bool vec = qb::aligned16(logits) && (row_stride * (int64_t)sizeof(T)) % 16 == 0;
    auto* lp = static_cast<T*>(logits);
    const unsigned grid = static_cast<unsigned>(rows);
    if (vec)
      ce_rows_kernel<T, 8><<<grid, kThreads, 0, stream>>>(lp, row_stride, target, vocab, loss, entropy, pred, correct, grad_scale, write_grad);
    else
      ce_rows_kernel<T, 1><<<grid, kThreads, 0, stream>>>(lp, row_stride, target, vocab, loss, entropy, pred, correct, grad_scale, write_grad);
  });
  return qb::check_launch("ce_rows");
}
