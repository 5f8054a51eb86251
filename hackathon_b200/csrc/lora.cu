// LoRA helpers around the adapter GEMMs: dropout + scale + cast with a counter-based mask, and
// the scaled add of the adapter output onto the base projection (solution/lora.py:29-60).
//
// The dropout mask is Philox-4x32 with 10 rounds (Salmon et al., SC'11), keyed by the 64-bit
// seed (low word k0, high word k1) with counter (offset, 0, 0, 0), offset = int32(row*cols+col).
// The first output word w becomes a uniform in [0,1) as float(w >= 2^31 ? ~w : w) * 4.6566127342e-10
// (w read as int32) — the stream Triton's tl.rand(seed, offset) draws, so the masks equal the
// reference kernel's. Nothing is stored: the backward regenerates the mask from the seed.
#include "qb_common.cuh"

namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ uint32_t philox_first_word(uint32_t c0, uint32_t k0, uint32_t k1) {
  uint32_t c1 = 0, c2 = 0, c3 = 0;
  const uint32_t mA = 0xD2511F53u, mB = 0xCD9E8D57u;  // round multipliers
  const uint32_t wA = 0x9E3779B9u, wB = 0xBB67AE85u;  // key increments (Weyl sequence)
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t hiB = __umulhi(mB, c2), loB = mB * c2;
    const uint32_t hiA = __umulhi(mA, c0), loA = mA * c0;
    const uint32_t n0 = hiB ^ c1 ^ k0;
    const uint32_t n2 = hiA ^ c3 ^ k1;
    c0 = n0;
    c1 = loB;
    c2 = n2;
    c3 = loA;
    k0 += wA;
    k1 += wB;
  }
  return c0;
}

__device__ __forceinline__ float uniform_of(uint32_t w) {
  int32_t x = static_cast<int32_t>(w);
  if (x < 0) x = ~x;  // -x - 1 without overflow
  return __fmul_rn(__int2float_rn(x), 4.6566127342e-10f);
}

template <typename IT, typename OT, bool DROP, int VEC>
__global__ void __launch_bounds__(kThreads)
dropout_scale_kernel(const IT* __restrict__ in, int64_t ins, OT* __restrict__ out, int64_t outs,
                     int64_t cols, uint32_t k0, uint32_t k1, float p, float scale) {
  const int64_t row = blockIdx.x;
  const IT* src = in + row * ins;
  OT* dst = out + row * outs;
  for (int64_t c = static_cast<int64_t>(threadIdx.x) * VEC; c < cols; c += kThreads * VEC) {
    float v[VEC];
    if constexpr (VEC == 8) qb::load8<IT>(src + c, v);
    else v[0] = qb::to_f(src[c]);
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      if (DROP) {
        const uint32_t off = static_cast<uint32_t>(row * cols + c + e);  // int32 wrap, as the reference
        const bool keep = uniform_of(philox_first_word(off, k0, k1)) > p;
        v[e] = keep ? v[e] * scale : 0.0f;
      } else {
        v[e] = v[e] * scale;
      }
    }
    if constexpr (VEC == 8) qb::store8<OT>(dst + c, v);
    else dst[c] = qb::from_f<OT>(v[0]);
  }
}

template <typename BT, typename LT, typename OT, int VEC>
__global__ void __launch_bounds__(kThreads)
scaled_add_kernel(const BT* __restrict__ base, int64_t bs, const LT* __restrict__ lo, int64_t ls,
                  OT* __restrict__ out, int64_t os, int64_t cols, float scaling) {
  const int64_t row = blockIdx.x;
  for (int64_t c = static_cast<int64_t>(threadIdx.x) * VEC; c < cols; c += kThreads * VEC) {
    float b[VEC], l[VEC], o[VEC];
    if constexpr (VEC == 8) {
      qb::load8<BT>(base + row * bs + c, b);
      qb::load8<LT>(lo + row * ls + c, l);
    } else {
      b[0] = qb::to_f(base[row * bs + c]);
      l[0] = qb::to_f(lo[row * ls + c]);
    }
#pragma unroll
    for (int e = 0; e < VEC; ++e) o[e] = b[e] + l[e] * scaling;
    if constexpr (VEC == 8) qb::store8<OT>(out + row * os + c, o);
    else out[row * os + c] = qb::from_f<OT>(o[0]);
  }
}

bool rows_ok(const void* p, int64_t stride, int esize) {
  return qb::aligned16(p) && (stride * esize) % 16 == 0;
}

}  // namespace

extern "C" int qb_dropout_scale(const void* in, int in_dtype, int64_t in_row_stride, void* out,
                                int out_dtype, int64_t out_row_stride, int64_t rows, int64_t cols,
                                uint64_t seed, float p, float scale, cudaStream_t stream) {
  if (rows < 0 || cols < 0 || rows > 0x7fffffff) return qb::fail(QB_ERR_INVALID, "dropout_scale: bad shape");
  if (rows == 0 || cols == 0) return QB_OK;
  if (!in || !out) return qb::fail(QB_ERR_INVALID, "dropout_scale: null pointer");
  if (p >= 1.0f) return qb::fail(QB_ERR_INVALID, "dropout_scale: p must be < 1");
  const uint32_t k0 = static_cast<uint32_t>(seed & 0xffffffffu);
  const uint32_t k1 = static_cast<uint32_t>(seed >> 32);
  const bool drop = p > 0.0f;
  QB_DISPATCH_FLOAT(in_dtype, IT, {
    QB_DISPATCH_FLOAT(out_dtype, OT, {
      const bool vec = cols % 8 == 0 && rows_ok(in, in_row_stride, sizeof(IT)) &&
                       rows_ok(out, out_row_stride, sizeof(OT));
      const auto* ip = static_cast<const IT*>(in);
      auto* op = static_cast<OT*>(out);
      const unsigned grid = static_cast<unsigned>(rows);
      if (vec) {
        if (drop) dropout_scale_kernel<IT, OT, true, 8><<<grid, kThreads, 0, stream>>>(ip, in_row_stride, op, out_row_stride, cols, k0, k1, p, scale);
        else dropout_scale_kernel<IT, OT, false, 8><<<grid, kThreads, 0, stream>>>(ip, in_row_stride, op, out_row_stride, cols, k0, k1, p, scale);
      } else {
        if (drop) dropout_scale_kernel<IT, OT, true, 1><<<grid, kThreads, 0, stream>>>(ip, in_row_stride, op, out_row_stride, cols, k0, k1, p, scale);
        else dropout_scale_kernel<IT, OT, false, 1><<<grid, kThreads, 0, stream>>>(ip, in_row_stride, op, out_row_stride, cols, k0, k1, p, scale);
      }
    });
  });
  return qb::check_launch("dropout_scale");
}

extern "C" int qb_scaled_add(const void* base, int base_dtype, int64_t base_row_stride,
                             const void* lo, int lo_dtype, int64_t lo_row_stride, void* out,
                             int out_dtype, int64_t out_row_stride, int64_t rows, int64_t cols,
                             float scaling, cudaStream_t stream) {
  if (rows < 0 || cols < 0 || rows > 0x7fffffff) return qb::fail(QB_ERR_INVALID, "scaled_add: bad shape");
  if (rows == 0 || cols == 0) return QB_OK;
  if (!base || !lo || !out) return qb::fail(QB_ERR_INVALID, "scaled_add: null pointer");
  QB_DISPATCH_FLOAT(base_dtype, BT, {
    QB_DISPATCH_FLOAT(lo_dtype, LT, {
      QB_DISPATCH_FLOAT(out_dtype, OT, {
        const bool vec = cols % 8 == 0 && rows_ok(base, base_row_stride, sizeof(BT)) &&
                         rows_ok(lo, lo_row_stride, sizeof(LT)) &&
                         rows_ok(out, out_row_stride, sizeof(OT));
        const auto* bp = static_cast<const BT*>(base);
        const auto* lp = static_cast<const LT*>(lo);
        auto* op = static_cast<OT*>(out);
        const unsigned grid = static_cast<unsigned>(rows);
        if (vec) scaled_add_kernel<BT, LT, OT, 8><<<grid, kThreads, 0, stream>>>(bp, base_row_stride, lp, lo_row_stride, op, out_row_stride, cols, scaling);
        else scaled_add_kernel<BT, LT, OT, 1><<<grid, kThreads, 0, stream>>>(bp, base_row_stride, lp, lo_row_stride, op, out_row_stride, cols, scaling);
      });
    });
  });
  return qb::check_launch("scaled_add");
}
