// The dropout mask stream shared by the dropout kernels (lora.cu) and the GEMM whose spare warps
// draw the next layer's masks (tc_gemm.cuh).
//
// The mask is Philox-4x32 with 10 rounds (Salmon et al., SC'11), keyed by the 64-bit seed (low
// word k0, high word k1) with counter (offset, 0, 0, 0), offset = int32(row*cols+col). The first
// output word w becomes a uniform in [0,1) as float(w >= 2^31 ? ~w : w) * 4.6566127342e-10 (w
// read as int32) - the stream Triton's tl.rand(seed, offset) draws, so the masks equal the
// reference kernel's. An element is kept when its uniform is above p.
#pragma once

#include <stdint.h>

namespace qb {

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

// The reference keeps an element when uniform(w) > p, with uniform(w) = fl(fl(x) * 2^-31-ish),
// x = w as int32 folded onto [0, 2^31) (x < 0 -> -x - 1). uniform is non-decreasing in x, so the
// test is x > T for one integer T per call (keep_threshold, host side, same IEEE single
// operations): the kernels compare integers and never convert to float.
constexpr float kUniformScale = 4.6566127342e-10f;

__device__ __forceinline__ bool keep_of(uint32_t w, int32_t thresh) {
  const int32_t x = static_cast<int32_t>(w ^ static_cast<uint32_t>(static_cast<int32_t>(w) >> 31));
  return x > thresh;
}

// Largest x in [0, 2^31) with fl(fl(x) * kUniformScale) <= p, or -1 when there is none
// (p below every uniform: everything kept). Bisection over a non-decreasing function.
inline int32_t keep_threshold(float p) {
  auto u = [](int32_t x) {
    volatile float f = static_cast<float>(x);   // round to nearest, as __int2float_rn
    volatile float r = f * kUniformScale;       // round to nearest, as __fmul_rn
    return static_cast<float>(r);
  };
  if (!(u(0) <= p)) return -1;
  int32_t lo = 0, hi = 0x7fffffff;              // u(lo) <= p
  if (u(hi) <= p) return hi;                    // nothing kept
  while (hi - lo > 1) {                         // u(hi) > p
    const int32_t mid = lo + (hi - lo) / 2;
    if (u(mid) <= p) lo = mid;
    else hi = mid;
  }
  return lo;
}

// One 32-bit word of mask bits: bit j for column c0 + j of `row` (n <= 32 columns; the bits past
// the row's end stay 0).
__device__ __forceinline__ uint32_t mask_word(int64_t row, int64_t cols, int64_t c0, int n,
                                              uint32_t k0, uint32_t k1, int32_t thresh) {
  const uint32_t off0 = static_cast<uint32_t>(row * cols + c0);  // int32 wrap, as the reference
  uint32_t word = 0;
  if (n == 32) {
#pragma unroll 8
    for (int j = 0; j < 32; ++j)
      word |= static_cast<uint32_t>(keep_of(philox_first_word(off0 + j, k0, k1), thresh)) << j;
  } else {
    for (int j = 0; j < n; ++j)
      word |= static_cast<uint32_t>(keep_of(philox_first_word(off0 + j, k0, k1), thresh)) << j;
  }
  return word;
}

}  // namespace qb
