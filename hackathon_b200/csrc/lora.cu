// LoRA helpers around the adapter GEMMs: dropout + scale + cast with a counter-based mask, and
// the scaled add of the adapter output onto the base projection (solution/lora.py:29-60).
//
// The dropout mask is Philox-4x32 with 10 rounds (Salmon et al., SC'11), keyed by the 64-bit
// seed (low word k0, high word k1) with counter (offset, 0, 0, 0), offset = int32(row*cols+col).
// The first output word w becomes a uniform in [0,1) as float(w >= 2^31 ? ~w : w) * 4.6566127342e-10
// (w read as int32) — the stream Triton's tl.rand(seed, offset) draws, so the masks equal the
// reference kernel's. The mask depends on (seed, offset) only, never on the data: it can be drawn
// ahead as bits (qb_dropout_bits) and applied later (qb_dropout_apply), or drawn and applied in
// one pass that also records the bits (qb_dropout_mask).
#include "qb_common.cuh"
#include "philox.cuh"

namespace tc_host {
int sm_count();   // tc_host.cu: SMs of the current device (cached)
}

namespace {

constexpr int kThreads = 256;

using qb::keep_of;
using qb::keep_threshold;
using qb::philox_first_word;

template <typename IT, typename OT, bool DROP, int VEC>
__global__ void __launch_bounds__(kThreads)
dropout_scale_kernel(const IT* __restrict__ in, int64_t ins, OT* __restrict__ out, int64_t outs,
                     int64_t cols, uint32_t k0, uint32_t k1, int32_t thresh, float scale) {
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
        const bool keep = keep_of(philox_first_word(off, k0, k1), thresh);
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

// Dropout that also records its mask: one warp walks a row 32 columns at a time, every lane
// draws its element's Philox number, and the warp's ballot is the 32-bit word of mask bits.
template <typename IT, typename OT>
__global__ void __launch_bounds__(kThreads)
dropout_mask_kernel(const IT* __restrict__ in, int64_t ins, OT* __restrict__ out, int64_t outs,
                    uint32_t* __restrict__ bits, int64_t words, int64_t rows, int64_t cols,
                    uint32_t k0, uint32_t k1, int32_t thresh, float scale) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * kThreads) >> 5;
  for (int64_t task = warp; task < rows * words; task += nwarps) {
    const int64_t row = task / words, w = task % words;
    const int64_t c = w * 32 + lane;
    bool keep = false;
    if (c < cols) {
      const uint32_t off = static_cast<uint32_t>(row * cols + c);  // int32 wrap, as the reference
      keep = keep_of(philox_first_word(off, k0, k1), thresh);
      const float v = qb::to_f(in[row * ins + c]);
      out[row * outs + c] = qb::from_f<OT>(keep ? v * scale : 0.0f);
    }
    const uint32_t word = __ballot_sync(0xffffffffu, keep);
    if (lane == 0) bits[row * words + w] = word;
  }
}

// The same for rows of a multiple of 32 columns with 16-byte-aligned rows: 8 elements per
// thread (16-byte accesses for 2-byte types), four consecutive threads combine their 8 bits
// into one mask word.
// (row, first column) of work item i of n8 items per row: 32-bit division when every index fits
// in 32 bits (a few instructions; the 64-bit one costs as much as several Philox rounds).
template <bool SMALL>
__device__ __forceinline__ void row_col8(int64_t i, int64_t n8, int64_t& row, int64_t& c) {
  if (SMALL) {
    const uint32_t ii = static_cast<uint32_t>(i), nn = static_cast<uint32_t>(n8);
    const uint32_t r = ii / nn;
    row = r;
    c = static_cast<int64_t>(ii - r * nn) * 8;
  } else {
    row = i / n8;
    c = (i - row * n8) * 8;
  }
}

template <typename IT, typename OT, bool SMALL>
__global__ void __launch_bounds__(kThreads)
dropout_mask8_kernel(const IT* __restrict__ in, int64_t ins, OT* __restrict__ out, int64_t outs,
                     uint32_t* __restrict__ bits, int64_t rows, int64_t cols, uint32_t k0,
                     uint32_t k1, int32_t thresh, float scale) {
  const int64_t n8 = cols / 8;
  const int64_t total = rows * n8;   // a multiple of 4: every group of four lanes is complete
  const int lane = threadIdx.x & 31;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
       i - lane < total; i += static_cast<int64_t>(gridDim.x) * kThreads) {
    uint32_t b = 0;
    int64_t row = 0, c = 0;
    if (i < total) {
      row_col8<SMALL>(i, n8, row, c);
      float v[8];
      qb::load8<IT>(in + row * ins + c, v);
      const uint32_t off0 = static_cast<uint32_t>(row * cols + c);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const bool keep = keep_of(philox_first_word(off0 + e, k0, k1), thresh);
        b |= static_cast<uint32_t>(keep) << e;
        v[e] = keep ? v[e] * scale : 0.0f;
      }
      qb::store8<OT>(out + row * outs + c, v);
    }
    uint32_t w = b << ((lane & 3) * 8);
    w |= __shfl_xor_sync(0xffffffffu, w, 1);
    w |= __shfl_xor_sync(0xffffffffu, w, 2);
    if (i < total && (lane & 3) == 0) bits[row * (cols / 32) + c / 32] = w;
  }
}

// out (+)= in * bit * scale from recorded mask bits: no random numbers, one HBM pass.
template <typename IT, typename OT, bool ACC, bool SMALL>
__global__ void __launch_bounds__(kThreads)
dropout_apply_kernel(const IT* __restrict__ in, int64_t ins, const uint32_t* __restrict__ bits,
                     int64_t words, OT* __restrict__ out, int64_t outs, int64_t rows,
                     int64_t cols, float scale) {
  const int64_t n8 = cols / 8;
  const int64_t total = rows * n8;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * kThreads) {
    int64_t row, c;
    row_col8<SMALL>(i, n8, row, c);
    const uint32_t b = (bits[row * words + c / 32] >> (c % 32)) & 0xffu;
    float v[8];
    qb::load8<IT>(in + row * ins + c, v);
    if (ACC) {
      float o[8];
      qb::load8<OT>(out + row * outs + c, o);
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = o[e] + (((b >> e) & 1u) ? v[e] * scale : 0.0f);
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = ((b >> e) & 1u) ? v[e] * scale : 0.0f;
    }
    qb::store8<OT>(out + row * outs + c, v);
  }
}

// Up to four dropouts of one input with their own recorded masks (the q / k / v projections'
// common input, the gate / up pair's): each 8-element piece of `in` is read once and written
// once per output, with dropout_apply_kernel's arithmetic (in * scale where the bit is set).
constexpr int kMaxApplyOuts = 4;
struct ApplyOuts {
  const uint32_t* bits[kMaxApplyOuts];   // [rows, words] each
  void* out[kMaxApplyOuts];
  int64_t outs[kMaxApplyOuts];           // row strides (elements)
  float scale[kMaxApplyOuts];
  int n;
};

template <typename IT, typename OT, bool SMALL>
__global__ void __launch_bounds__(kThreads)
dropout_apply_multi_kernel(const IT* __restrict__ in, int64_t ins,
                           const __grid_constant__ ApplyOuts o, int64_t words, int64_t rows,
                           int64_t cols) {
  const int64_t n8 = cols / 8;
  const int64_t total = rows * n8;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * kThreads) {
    int64_t row, c;
    row_col8<SMALL>(i, n8, row, c);
    float x[8];
    qb::load8<IT>(in + row * ins + c, x);
#pragma unroll
    for (int j = 0; j < kMaxApplyOuts; ++j) {
      if (j >= o.n) break;
      const uint32_t b = (__ldg(o.bits[j] + row * words + c / 32) >> (c % 32)) & 0xffu;
      float v[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = ((b >> e) & 1u) ? x[e] * o.scale[j] : 0.0f;
      qb::store8<OT>(static_cast<OT*>(o.out[j]) + row * o.outs[j] + c, v);
    }
  }
}

// Mask bits only, no data: one thread per 32-bit word (bit j = column 32w + j; bits past the
// row's end are 0, as the ballot of dropout_mask_kernel leaves them). A fixed grid of a few
// 256-thread blocks per SM with at most 32 registers a thread, so that the kernel can run on a
// side stream beside a persistent GEMM that holds one CTA per SM (the GEMM's CTAs still fit:
// its shared memory is untouched, and 2 x 256 x 32 registers leave 48K for it).
__global__ void __launch_bounds__(kThreads, 8)
dropout_bits_kernel(uint32_t* __restrict__ bits, int64_t words, int64_t rows, int64_t cols,
                    uint32_t k0, uint32_t k1, int32_t thresh) {
  const int64_t total = rows * words;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; t < total;
       t += static_cast<int64_t>(gridDim.x) * kThreads) {
    const int64_t row = t / words, w = t % words;
    const int64_t c0 = w * 32;
    const int n = cols - c0 < 32 ? static_cast<int>(cols - c0) : 32;
    const uint32_t word = qb::mask_word(row, cols, c0, n, k0, k1, thresh);
    bits[t] = word;
  }
}

unsigned grid_cap(int64_t work_items) {
  int64_t g = (work_items + kThreads - 1) / kThreads;
  if (g > 148 * 16) g = 148 * 16;
  if (g < 1) g = 1;
  return static_cast<unsigned>(g);
}

template <typename IT, typename OT>
void launch_apply(const IT* in, int64_t ins, const uint32_t* bits, int64_t words, OT* out,
                  int64_t outs, int64_t rows, int64_t cols, float scale, bool acc,
                  cudaStream_t stream) {
  const unsigned grid = grid_cap(rows * (cols / 8));
  const bool small = rows * (cols / 8) <= 0xffffffffll;
  if (acc && small)
    dropout_apply_kernel<IT, OT, true, true><<<grid, kThreads, 0, stream>>>(
        in, ins, bits, words, out, outs, rows, cols, scale);
  else if (acc)
    dropout_apply_kernel<IT, OT, true, false><<<grid, kThreads, 0, stream>>>(
        in, ins, bits, words, out, outs, rows, cols, scale);
  else if (small)
    dropout_apply_kernel<IT, OT, false, true><<<grid, kThreads, 0, stream>>>(
        in, ins, bits, words, out, outs, rows, cols, scale);
  else
    dropout_apply_kernel<IT, OT, false, false><<<grid, kThreads, 0, stream>>>(
        in, ins, bits, words, out, outs, rows, cols, scale);
}

}  // namespace

extern "C" int qb_dropout_mask(const void* in, int in_dtype, int64_t in_row_stride, void* out,
                               int out_dtype, int64_t out_row_stride, uint32_t* bits,
                               int64_t rows, int64_t cols, uint64_t seed, float p, float scale,
                               cudaStream_t stream) {
  if (rows < 0 || cols < 0) return qb::fail(QB_ERR_INVALID, "dropout_mask: bad shape");
  if (rows == 0 || cols == 0) return QB_OK;
  if (!in || !out || !bits) return qb::fail(QB_ERR_INVALID, "dropout_mask: null pointer");
  if (p >= 1.0f) return qb::fail(QB_ERR_INVALID, "dropout_mask: p must be < 1");
  const int32_t thresh = keep_threshold(p);
  const uint32_t k0 = static_cast<uint32_t>(seed & 0xffffffffu);
  const uint32_t k1 = static_cast<uint32_t>(seed >> 32);
  const int64_t words = (cols + 31) / 32;
  QB_DISPATCH_FLOAT(in_dtype, IT, {
    QB_DISPATCH_FLOAT(out_dtype, OT, {
      if (cols % 32 == 0 && rows_ok(in, in_row_stride, sizeof(IT)) &&
          rows_ok(out, out_row_stride, sizeof(OT))) {
        const unsigned grid = grid_cap(rows * (cols / 8));
        if (rows * (cols / 8) <= 0xffffffffll)
          dropout_mask8_kernel<IT, OT, true><<<grid, kThreads, 0, stream>>>(
              static_cast<const IT*>(in), in_row_stride, static_cast<OT*>(out),
              out_row_stride, bits, rows, cols, k0, k1, thresh, scale);
        else
          dropout_mask8_kernel<IT, OT, false><<<grid, kThreads, 0, stream>>>(
              static_cast<const IT*>(in), in_row_stride, static_cast<OT*>(out),
              out_row_stride, bits, rows, cols, k0, k1, thresh, scale);
      } else {
        dropout_mask_kernel<IT, OT><<<grid_cap(rows * words * 32), kThreads, 0, stream>>>(
            static_cast<const IT*>(in), in_row_stride, static_cast<OT*>(out), out_row_stride,
            bits, words, rows, cols, k0, k1, thresh, scale);
      }
    });
  });
  return qb::check_launch("dropout_mask");
}

extern "C" int qb_dropout_bits(uint32_t* bits, int64_t rows, int64_t cols, uint64_t seed,
                               float p, int ctas_per_sm, cudaStream_t stream) {
  if (rows < 0 || cols < 0) return qb::fail(QB_ERR_INVALID, "dropout_bits: bad shape");
  if (ctas_per_sm < 0 || ctas_per_sm > 8)
    return qb::fail(QB_ERR_INVALID, "dropout_bits: ctas_per_sm must be 0..8");
  if (p >= 1.0f) return qb::fail(QB_ERR_INVALID, "dropout_bits: p must be < 1");
  if (rows == 0 || cols == 0) return QB_OK;
  if (!bits) return qb::fail(QB_ERR_INVALID, "dropout_bits: null pointer");
  const int32_t thresh = keep_threshold(p);
  const int64_t words = (cols + 31) / 32;
  int64_t grid = (rows * words + kThreads - 1) / kThreads;
  const int64_t cap = static_cast<int64_t>(tc_host::sm_count()) * (ctas_per_sm ? ctas_per_sm : 8);
  if (grid > cap) grid = cap;
  dropout_bits_kernel<<<static_cast<unsigned>(grid), kThreads, 0, stream>>>(
      bits, words, rows, cols, static_cast<uint32_t>(seed & 0xffffffffu),
      static_cast<uint32_t>(seed >> 32), thresh);
  return qb::check_launch("dropout_bits");
}

extern "C" int qb_dropout_apply(const void* in, int in_dtype, int64_t in_row_stride,
                                const uint32_t* bits, void* out, int out_dtype,
                                int64_t out_row_stride, int64_t rows, int64_t cols, float scale,
                                int accumulate, cudaStream_t stream) {
  if (rows < 0 || cols < 0) return qb::fail(QB_ERR_INVALID, "dropout_apply: bad shape");
  if (rows == 0 || cols == 0) return QB_OK;
  if (!in || !out || !bits) return qb::fail(QB_ERR_INVALID, "dropout_apply: null pointer");
  if (cols % 8) return qb::fail(QB_ERR_UNSUPPORTED, "dropout_apply: cols must be a multiple of 8");
  const int64_t words = (cols + 31) / 32;
  QB_DISPATCH_FLOAT(in_dtype, IT, {
    QB_DISPATCH_FLOAT(out_dtype, OT, {
      if (!rows_ok(in, in_row_stride, sizeof(IT)) || !rows_ok(out, out_row_stride, sizeof(OT)))
        return qb::fail(QB_ERR_INVALID, "dropout_apply: rows must be 16-byte aligned");
      launch_apply<IT, OT>(static_cast<const IT*>(in), in_row_stride, bits, words,
                           static_cast<OT*>(out), out_row_stride, rows, cols, scale,
                           accumulate != 0, stream);
    });
  });
  return qb::check_launch("dropout_apply");
}

extern "C" int qb_dropout_apply_multi(const void* in, int in_dtype, int64_t in_row_stride, int n,
                                      const uint32_t* const* bits, void* const* outs,
                                      int out_dtype, const int64_t* out_row_strides,
                                      const float* scales, int64_t rows, int64_t cols,
                                      cudaStream_t stream) {
  const char* what = "dropout_apply_multi";
  if (n < 1 || n > kMaxApplyOuts)
    return qb::fail(QB_ERR_INVALID, "%s: 1..%d outputs", what, kMaxApplyOuts);
  if (!bits || !outs || !out_row_strides || !scales)
    return qb::fail(QB_ERR_INVALID, "%s: null output table", what);
  if (rows < 0 || cols < 0) return qb::fail(QB_ERR_INVALID, "%s: bad shape", what);
  if (rows == 0 || cols == 0) return QB_OK;
  if (cols % 8) return qb::fail(QB_ERR_UNSUPPORTED, "%s: cols must be a multiple of 8", what);
  if (!in) return qb::fail(QB_ERR_INVALID, "%s: null pointer", what);
  ApplyOuts o{};
  o.n = n;
  for (int j = 0; j < n; ++j) {
    if (!bits[j] || !outs[j]) return qb::fail(QB_ERR_INVALID, "%s: null pointer", what);
    if (reinterpret_cast<uintptr_t>(bits[j]) % 4)
      return qb::fail(QB_ERR_INVALID, "%s: mask bits must be 4-byte aligned", what);
    o.bits[j] = bits[j];
    o.out[j] = outs[j];
    o.outs[j] = out_row_strides[j];
    o.scale[j] = scales[j];
  }
  const int64_t words = (cols + 31) / 32;
  QB_DISPATCH_FLOAT(in_dtype, IT, {
    QB_DISPATCH_FLOAT(out_dtype, OT, {
      if (!rows_ok(in, in_row_stride, sizeof(IT)))
        return qb::fail(QB_ERR_INVALID, "%s: rows must be 16-byte aligned", what);
      for (int j = 0; j < n; ++j)
        if (!rows_ok(outs[j], out_row_strides[j], sizeof(OT)))
          return qb::fail(QB_ERR_INVALID, "%s: rows must be 16-byte aligned", what);
      const unsigned grid = grid_cap(rows * (cols / 8));
      if (rows * (cols / 8) <= 0xffffffffll)
        dropout_apply_multi_kernel<IT, OT, true><<<grid, kThreads, 0, stream>>>(
            static_cast<const IT*>(in), in_row_stride, o, words, rows, cols);
      else
        dropout_apply_multi_kernel<IT, OT, false><<<grid, kThreads, 0, stream>>>(
            static_cast<const IT*>(in), in_row_stride, o, words, rows, cols);
    });
  });
  return qb::check_launch(what);
}

extern "C" int qb_dropout_scale(const void* in, int in_dtype, int64_t in_row_stride, void* out,
                                int out_dtype, int64_t out_row_stride, int64_t rows, int64_t cols,
                                uint64_t seed, float p, float scale, cudaStream_t stream) {
  if (rows < 0 || cols < 0 || rows > 0x7fffffff) return qb::fail(QB_ERR_INVALID, "dropout_scale: bad shape");
  if (rows == 0 || cols == 0) return QB_OK;
  if (!in || !out) return qb::fail(QB_ERR_INVALID, "dropout_scale: null pointer");
  if (p >= 1.0f) return qb::fail(QB_ERR_INVALID, "dropout_scale: p must be < 1");
  const int32_t thresh = keep_threshold(p);
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
        if (drop) dropout_scale_kernel<IT, OT, true, 8><<<grid, kThreads, 0, stream>>>(ip, in_row_stride, op, out_row_stride, cols, k0, k1, thresh, scale);
        else dropout_scale_kernel<IT, OT, false, 8><<<grid, kThreads, 0, stream>>>(ip, in_row_stride, op, out_row_stride, cols, k0, k1, thresh, scale);
      } else {
        if (drop) dropout_scale_kernel<IT, OT, true, 1><<<grid, kThreads, 0, stream>>>(ip, in_row_stride, op, out_row_stride, cols, k0, k1, thresh, scale);
        else dropout_scale_kernel<IT, OT, false, 1><<<grid, kThreads, 0, stream>>>(ip, in_row_stride, op, out_row_stride, cols, k0, k1, thresh, scale);
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

// ------------------------------------------------------------------------------ adapter pack

namespace {

constexpr int kPackChunk = 2048;   // elements per CTA: 256 threads x 8

__global__ void __launch_bounds__(kThreads)
adapter_pack_kernel(const qb_pack_segment* __restrict__ segs, int nseg) {
  __shared__ int s_seg;
  if (threadIdx.x == 0) {   // the last segment whose first chunk is <= this CTA's chunk
    int lo = 0, hi = nseg - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) / 2;
      if (segs[mid].first_chunk <= static_cast<int64_t>(blockIdx.x)) lo = mid;
      else hi = mid - 1;
    }
    s_seg = lo;
  }
  __syncthreads();
  const qb_pack_segment sg = segs[s_seg];
  const int64_t n = static_cast<int64_t>(sg.rows) * sg.cols;
  const int64_t e0 = (static_cast<int64_t>(blockIdx.x) - sg.first_chunk) * kPackChunk +
                     threadIdx.x * 8;
  auto* dst = static_cast<__nv_bfloat16*>(sg.dst);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int64_t e = e0 + j;
    if (e >= n) break;
    const int64_t row = e / sg.cols, col = e - row * sg.cols;
    dst[row * sg.dst_ld + col] = __float2bfloat16_rn(__fmul_rn(sg.src[row * sg.src_ld + col],
                                                               sg.scale));
  }
}

}  // namespace

extern "C" int64_t qb_pack_segment_size(void) { return sizeof(qb_pack_segment); }

extern "C" int qb_adapter_pack(const qb_pack_segment* segs, int nseg, int64_t total_chunks,
                               cudaStream_t stream) {
  if (nseg < 0 || total_chunks < 0 || total_chunks > 0x7fffffff)
    return qb::fail(QB_ERR_INVALID, "adapter_pack: bad sizes");
  if (nseg == 0 || total_chunks == 0) return QB_OK;
  if (!segs) return qb::fail(QB_ERR_INVALID, "adapter_pack: null segment table");
  adapter_pack_kernel<<<static_cast<unsigned>(total_chunks), kThreads, 0, stream>>>(segs, nseg);
  return qb::check_launch("adapter_pack");
}
