// Rotate-half RoPE on q and k in one launch, forward and backward (solution/rope.py:25-62).
//
// One CTA per (batch, position) - or per a few consecutive positions when a position has few
// heads - handles every q head and every k head of that position. A work item is one chunk of 8
// dims in the first half and the matching 8 dims of the second half of one head: it reads x1,
// x2 (16-byte loads for 2-byte dtypes) and the cos/sin chunks, and writes o1, o2. With (B,S,H,D) buffers seen as (B,H,S,D) — how the attention builds q and k — the
// heads of one position are contiguous, so a CTA's loads and stores cover whole cache lines.
#include "qb_common.cuh"

namespace {

struct Strides3 {
  int64_t b, h, s;
};

template <typename T, int VEC>
__device__ __forceinline__ void ld(const T* p, float* out) {
  if constexpr (VEC == 8) qb::load8<T>(p, out);
  else out[0] = qb::to_f(p[0]);
}

template <typename T, int VEC>
__device__ __forceinline__ void st(T* p, const float* in) {
  if constexpr (VEC == 8) qb::store8<T>(p, in);
  else p[0] = qb::from_f<T>(in[0]);
}

// A CTA takes `ppc` consecutive (batch, position) pairs, `span` threads each (ppc > 1 when a
// position has few items, e.g. the 4 k heads: one CTA per position would leave 32-thread CTAs).
template <typename QT, typename OT, typename CT, int VEC, bool BACKWARD, bool MULTI>
__global__ void rope_qk_kernel(const QT* __restrict__ q, const QT* __restrict__ k,
                               OT* __restrict__ qo, OT* __restrict__ ko,
                               const CT* __restrict__ cosp, const CT* __restrict__ sinp, int S,
                               int HQ, int HK, int half, Strides3 sq, Strides3 sk, Strides3 sqo,
                               Strides3 sko, int64_t csb, int64_t css, int64_t npos, int ppc,
                               int span) {
  // MULTI: ppc positions of span threads each; else one position of blockDim.x threads
  const int local = MULTI ? static_cast<int>(threadIdx.x) / span : 0;
  const int64_t pid = MULTI ? static_cast<int64_t>(blockIdx.x) * ppc + local : blockIdx.x;
  if (MULTI && pid >= npos) return;    // no barrier below
  const int stride = MULTI ? span : static_cast<int>(blockDim.x);
  const int64_t b = pid / S, s = pid % S;
  const int chunks = half / VEC;
  const int items = (HQ + HK) * chunks;
  const CT* cb = cosp + b * csb + s * css;
  const CT* sb = sinp + b * csb + s * css;
  for (int it = static_cast<int>(threadIdx.x) - local * span; it < items; it += stride) {
    const int head = it / chunks;
    const int d = (it % chunks) * VEC;
    float c1[VEC], c2[VEC], s1[VEC], s2[VEC];
    ld<CT, VEC>(cb + d, c1);
    ld<CT, VEC>(cb + half + d, c2);
    ld<CT, VEC>(sb + d, s1);
    ld<CT, VEC>(sb + half + d, s2);
    const QT* src;
    OT* dst;
    if (head < HQ) {
      src = q + b * sq.b + head * sq.h + s * sq.s;
      dst = qo + b * sqo.b + head * sqo.h + s * sqo.s;
    } else {
      const int h = head - HQ;
      src = k + b * sk.b + h * sk.h + s * sk.s;
      dst = ko + b * sko.b + h * sko.h + s * sko.s;
    }
    float x1[VEC], x2[VEC], o1[VEC], o2[VEC];
    ld<QT, VEC>(src + d, x1);
    ld<QT, VEC>(src + half + d, x2);
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      if (BACKWARD)  // transpose of the rotation
        qb::rope_rotate_t(x1[e], x2[e], c1[e], c2[e], s1[e], s2[e], o1[e], o2[e]);
      else
        qb::rope_rotate(x1[e], x2[e], c1[e], c2[e], s1[e], s2[e], o1[e], o2[e]);
    }
    st<OT, VEC>(dst + d, o1);
    st<OT, VEC>(dst + half + d, o2);
  }
}

bool al(const void* p, int64_t stride, int esize) {
  return qb::aligned16(p) && (stride * esize) % 16 == 0;
}

template <typename QT, typename OT, typename CT>
int rope_typed(const void* q, const void* k, void* qo, void* ko, const void* c, const void* s,
               int64_t B, int64_t HQ, int64_t HK, int64_t S, int64_t D, Strides3 sq, Strides3 sk,
               Strides3 sqo, Strides3 sko, int64_t csb, int64_t css, bool backward,
               cudaStream_t stream) {
  const int half = static_cast<int>(D / 2);
  const int qs = sizeof(QT), os = sizeof(OT), cs = sizeof(CT);
  const bool vec = half % 8 == 0 && al(q, sq.b, qs) && al(q, sq.h, qs) && al(q, sq.s, qs) &&
                   al(k, sk.b, qs) && al(k, sk.h, qs) && al(k, sk.s, qs) &&
                   al(qo, sqo.b, os) && al(qo, sqo.h, os) && al(qo, sqo.s, os) &&
                   al(ko, sko.b, os) && al(ko, sko.h, os) && al(ko, sko.s, os) &&
                   al(c, csb, cs) && al(c, css, cs) && al(s, csb, cs) && al(s, css, cs) &&
                   (half * qs) % 16 == 0 && (half * os) % 16 == 0 && (half * cs) % 16 == 0;
  const int vecw = vec ? 8 : 1;
  const int64_t items = (HQ + HK) * (half / vecw);
  int span = static_cast<int>(((items + 31) / 32) * 32);
  if (span > 512) span = 512;
  if (span < 32) span = 32;
  const int ppc = span >= 256 ? 1 : 256 / span;     // positions per CTA
  const int threads = span * ppc;
  const int64_t npos = B * S;
  const dim3 grid(static_cast<unsigned>((npos + ppc - 1) / ppc));
  auto* qp = static_cast<const QT*>(q);
  auto* kp = static_cast<const QT*>(k);
  auto* qop = static_cast<OT*>(qo);
  auto* kop = static_cast<OT*>(ko);
  auto* cp = static_cast<const CT*>(c);
  auto* sp = static_cast<const CT*>(s);
  const int Si = static_cast<int>(S), HQi = static_cast<int>(HQ), HKi = static_cast<int>(HK);
#define QB_ROPE_LAUNCH(V, BW, M)                                                                  \
  rope_qk_kernel<QT, OT, CT, V, BW, M><<<grid, threads, 0, stream>>>(                             \
      qp, kp, qop, kop, cp, sp, Si, HQi, HKi, half, sq, sk, sqo, sko, csb, css, npos, ppc, span)
  const bool multi = ppc > 1;
  if (vec) {
    if (backward) {
      if (multi) QB_ROPE_LAUNCH(8, true, true); else QB_ROPE_LAUNCH(8, true, false);
    } else {
      if (multi) QB_ROPE_LAUNCH(8, false, true); else QB_ROPE_LAUNCH(8, false, false);
    }
  } else {
    if (backward) {
      if (multi) QB_ROPE_LAUNCH(1, true, true); else QB_ROPE_LAUNCH(1, true, false);
    } else {
      if (multi) QB_ROPE_LAUNCH(1, false, true); else QB_ROPE_LAUNCH(1, false, false);
    }
  }
#undef QB_ROPE_LAUNCH
  return qb::check_launch("rope_qk");
}

}  // namespace

extern "C" int qb_rope_qk(const void* q, const void* k, void* q_out, void* k_out,
                          const void* cos_, const void* sin_, int in_dtype, int out_dtype,
                          int cs_dtype, int64_t B, int64_t HQ, int64_t HK, int64_t S, int64_t D,
                          const int64_t* q_strides, const int64_t* k_strides,
                          const int64_t* qo_strides, const int64_t* ko_strides,
                          int64_t cs_stride_b, int64_t cs_stride_s, int backward,
                          cudaStream_t stream) {
  if (B < 0 || HQ < 0 || HK < 0 || S < 0 || D <= 0 || D % 2)
    return qb::fail(QB_ERR_INVALID, "rope_qk: bad shape (D must be even)");
  if (B * S > 0x7fffffff || HQ + HK > (1 << 20)) return qb::fail(QB_ERR_INVALID, "rope_qk: too large");
  if (B == 0 || S == 0 || HQ + HK == 0) return QB_OK;
  if (!q_strides || !k_strides || !qo_strides || !ko_strides)
    return qb::fail(QB_ERR_INVALID, "rope_qk: null strides");
  if ((HQ && (!q || !q_out)) || (HK && (!k || !k_out)) || !cos_ || !sin_)
    return qb::fail(QB_ERR_INVALID, "rope_qk: null pointer");
  const Strides3 sq{q_strides[0], q_strides[1], q_strides[2]};
  const Strides3 sk{k_strides[0], k_strides[1], k_strides[2]};
  const Strides3 sqo{qo_strides[0], qo_strides[1], qo_strides[2]};
  const Strides3 sko{ko_strides[0], ko_strides[1], ko_strides[2]};
  QB_DISPATCH_FLOAT(in_dtype, QT, {
    QB_DISPATCH_FLOAT(out_dtype, OT, {
      QB_DISPATCH_FLOAT(cs_dtype, CT, {
        return rope_typed<QT, OT, CT>(q, k, q_out, k_out, cos_, sin_, B, HQ, HK, S, D, sq, sk,
                                      sqo, sko, cs_stride_b, cs_stride_s, backward != 0, stream);
      });
    });
  });
}
