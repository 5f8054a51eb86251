// Fused linear cross-entropy on the tcgen05 GEMM: the [rows x vocab] logits live only in TMEM.
//
// (solution/cross_entropy.py:48-138 and fused_ce.py:42-158 compute the same quantities from a
// materialised logits chunk.) Here, per chunk of rows:
//   pass 1  qb_linear_ce_stats: logits tile = H W^T (128 rows x 256 vocab) in TMEM; the
//           epilogue reduces each row of the tile to (max m, sum e^(z-m), sum e^(z-m) z, first
//           argmax) — one float4 per (vocab tile, row) — and picks z[label] from the tile that
//           holds it. Logits never reach HBM.
//   reduce  qb_ce_reduce: merges the per-tile partials of every row into lse, loss =
//           lse - z[label], entropy = lse - t/s, argmax, correct.
//   pass 2  qb_linear_ce_grad: the logits tile again, epilogue dZ = (e^(z - lse) - onehot) *
//           scale in bf16 (scale a device scalar, the caller's gradient factor; 0 for unlabelled
//           rows) — the gradient, not the logits.
//   then    dH = dZ W (qb_gemm_bf16 with W read MN-major), fp32.
// Executed flops: 3 x 2 N H V against the algorithmic 4 N H V (logits + dH).
#include <cfloat>

#include "tc_gemm.cuh"

namespace {

constexpr int kBN = 256;

//
// With a tensor map of dz (`tma`), each epilogue warp stages its 32 rows of a 32-column chunk in
// shared memory (two alternating boxes, 64-byte swizzle) and one lane stores the box with a TMA
// store: whole lines to L2 for the [rows, vocab] gradient, the pass's only large output.
struct EpiGrad {
  __nv_bfloat16* dz;       // [rows, ldz]
  int64_t ldz;
  const int64_t* target;
  const float* lse;        // [rows]
  const float* scale_dev;  // device scalar: the factor dZ carries
  int rows, vocab;
  bool vec;
  bool tma = false;        // dmap holds dz: [rows, vocab], box 32 x 32, 64-byte swizzle
  CUtensorMap dmap;

  static constexpr int kBoxBytes = 32 * 64;
  static constexpr int kStageBytes = 2 * kBoxBytes;

  template <int BN>
  __device__ __forceinline__ void tile(int m0, int n0, int row, uint32_t taddr,
                                       uint8_t* stage) const {
    if (!tma) {
      tile<BN>(m0, n0, row, taddr);
      return;
    }
    const int lane = row & 31;
    const int r = m0 + row;
    const int rw = r - lane;   // the warp's first row
    const bool live = r < rows;
    const int64_t label = live ? __ldg(target + r) : -1;
    const float l = live ? __ldg(lse + r) : 0.f;
    const float sc = (live && label >= 0) ? __ldg(scale_dev) : 0.f;
    if (lane == 0) tc::bulk_wait_read_all();   // the previous tile's boxes are free
    __syncwarp();
#pragma unroll 1
    for (int ch = 0; ch < BN / 32; ++ch) {
      float v[32];
      tc::tmem_ld32(taddr + ch * 32, v);
      const int n = n0 + ch * 32;
      if (n >= vocab) continue;   // warp-uniform
#pragma unroll
      for (int i = 0; i < 32; ++i)
        v[i] = live ? (__expf(v[i] - l) - (n + i == label ? 1.f : 0.f)) * sc : 0.f;
      uint8_t* box = stage + (ch & 1) * kBoxBytes;
      if (ch >= 2) {   // the store of chunk ch - 2 read this box
        if (lane == 0) tc::bulk_wait_read_newest_pending();
        __syncwarp();
      }
      tcg::stage_row_bf16(box, lane, v);
      tc::fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0 && rw < rows) {   // rows past `rows` and columns past vocab are clipped
        tc::tma_store_2d(&dmap, box, n, rw);
        tc::bulk_commit();
      }
    }
  }

  template <int BN>
  __device__ __forceinline__ void tile(int m0, int n0, int row, uint32_t taddr) const {
    const int r = m0 + row;
    const bool live = r < rows;
    const int64_t label = live ? __ldg(target + r) : -1;
    const float l = live ? __ldg(lse + r) : 0.f;
    const float sc = (live && label >= 0) ? __ldg(scale_dev) : 0.f;
#pragma unroll 1
    for (int ch = 0; ch < BN / 32; ++ch) {
      float v[32];
      tc::tmem_ld32(taddr + ch * 32, v);
      const int n = n0 + ch * 32;
      if (!live || n >= vocab) continue;
#pragma unroll
      for (int i = 0; i < 32; ++i)
        v[i] = (__expf(v[i] - l) - (n + i == label ? 1.f : 0.f)) * sc;
      __nv_bfloat16* dst = dz + static_cast<int64_t>(r) * ldz + n;
      if (vec && n + 32 <= vocab) {
#pragma unroll
        for (int i = 0; i < 32; i += 8) qb::store8<__nv_bfloat16>(dst + i, v + i);
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (n + i < vocab) dst[i] = __float2bfloat16_rn(v[i]);
      }
    }
  }
};

// Per row of the tile: (max m, sum e^(z-m), sum e^(z-m) z, first argmax) over the tile's
// columns; z[label] when the label falls in this tile. One running max per 32-column chunk: when
// a chunk raises it, the sums so far are rescaled once.
// With `logits` set, the tile's fp32 logits are also stored ([rows, ldl]), so the gradient pass
// can read them back (qb_ce_grad_from_logits) instead of recomputing the GEMM.
struct EpiStats {
  float4* partials;
  float* z_label;
  const int64_t* target;
  int rows, vocab;
  float* logits;   // or null
  int64_t ldl;
  bool lvec;       // 16-byte aligned logits rows

  template <int BN>
  __device__ __forceinline__ void tile(int m0, int n0, int row, uint32_t taddr) const {
    const int r = m0 + row;
    const int64_t label = r < rows ? __ldg(target + r) : -1;
    float m = -INFINITY, s = 0.f, t = 0.f;
    int idx = 0x7fffffff;
#pragma unroll 1
    for (int ch = 0; ch < BN / 32; ++ch) {
      float v[32];
      tc::tmem_ld32(taddr + ch * 32, v);
      const int n = n0 + ch * 32;
      if (logits && r < rows && n < vocab) {
        float* dst = logits + static_cast<int64_t>(r) * ldl + n;
        if (lvec && n + 32 <= vocab) {
#pragma unroll
          for (int i = 0; i < 32; i += 4)
            *reinterpret_cast<float4*>(dst + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (n + i < vocab) dst[i] = v[i];
        }
      }
      float cm = -INFINITY;
      int cidx = 0x7fffffff;
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        if (n + i >= vocab) v[i] = -INFINITY;
        if (v[i] > cm) { cm = v[i]; cidx = n + i; }
        if (n + i == label && r < rows) z_label[r] = v[i];
      }
      if (cm == -INFINITY) continue;
      if (cm > m) {                     // new running max: rescale what was summed so far
        const float f = __expf(m - cm); // 0 when m == -inf
        s *= f;
        t *= f;
        m = cm;
        idx = cidx;
      }
      float cs = 0.f, ct = 0.f;
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float e = __expf(v[i] - m);
        cs += e;
        ct += (v[i] == -INFINITY) ? 0.f : e * v[i];
      }
      s += cs;
      t += ct;
    }
    if (r < rows)
      partials[static_cast<int64_t>(n0 / BN) * rows + r] = make_float4(m, s, t, __int_as_float(idx));
  }
};

// dz = (e^(z - lse) - onehot) * scale from stored fp32 logits: the same arithmetic as EpiGrad
// on the same z, so dz is identical to the recomputing pass. One CTA per row, 16-byte loads.
__global__ void __launch_bounds__(256)
ce_grad_from_logits_kernel(const float* __restrict__ logits, int64_t ldl,
                           const int64_t* __restrict__ target, const float* __restrict__ lse,
                           const float* __restrict__ scale_dev, __nv_bfloat16* __restrict__ dz,
                           int64_t ldz, int vocab, bool vec) {
  const int64_t r = blockIdx.x;
  const int64_t label = __ldg(target + r);
  const float l = __ldg(lse + r);
  const float sc = label >= 0 ? __ldg(scale_dev) : 0.f;
  const float* z = logits + r * ldl;
  __nv_bfloat16* d = dz + r * ldz;
  if (vec) {
    for (int n = threadIdx.x * 8; n < vocab; n += blockDim.x * 8) {
      if (n + 8 <= vocab) {
        const float4 a = __ldg(reinterpret_cast<const float4*>(z + n));
        const float4 b = __ldg(reinterpret_cast<const float4*>(z + n + 4));
        float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = (__expf(v[i] - l) - (n + i == label ? 1.f : 0.f)) * sc;
        qb::store8<__nv_bfloat16>(d + n, v);
      } else {
        for (int i = n; i < vocab; ++i)
          d[i] = __float2bfloat16_rn((__expf(z[i] - l) - (i == label ? 1.f : 0.f)) * sc);
      }
    }
  } else {
    for (int i = threadIdx.x; i < vocab; i += blockDim.x)
      d[i] = __float2bfloat16_rn((__expf(z[i] - l) - (i == label ? 1.f : 0.f)) * sc);
  }
}

// One warp per row: merge the row's partials, finish the statistics.
__global__ void ce_reduce_kernel(const float4* __restrict__ partials, int n_vt, int rows,
                                 const int64_t* __restrict__ target,
                                 const float* __restrict__ z_label, float* __restrict__ loss,
                                 float* __restrict__ entropy, int64_t* __restrict__ pred,
                                 int32_t* __restrict__ correct, float* __restrict__ lse_out,
                                 int vocab) {
  const int r = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  float m = -INFINITY, s = 0.f, t = 0.f;
  int idx = 0x7fffffff;
  for (int j = lane; j < n_vt; j += 32) {
    const float4 p = partials[static_cast<int64_t>(j) * rows + r];
    const int pidx = __float_as_int(p.w);
    if (p.x == -INFINITY) continue;
    if (p.x > m || (p.x == m && pidx < idx)) idx = pidx;
    const float mm = fmaxf(m, p.x);
    const float fa = __expf(m - mm), fb = __expf(p.x - mm);
    s = s * fa + p.y * fb;
    t = t * fa + p.z * fb;
    m = mm;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, m, o);
    const float os = __shfl_xor_sync(0xffffffffu, s, o);
    const float ot = __shfl_xor_sync(0xffffffffu, t, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (om == -INFINITY) continue;
    if (om > m || (om == m && oi < idx)) idx = oi;
    const float mm = fmaxf(m, om);
    const float fa = __expf(m - mm), fb = __expf(om - mm);
    s = s * fa + os * fb;
    t = t * fa + ot * fb;
    m = mm;
  }
  if (lane == 0) {
    const float lse = m + logf(s);
    const int64_t label = target[r];
    const bool labelled = label >= 0 && label < vocab;
    loss[r] = labelled ? lse - z_label[r] : 0.f;
    entropy[r] = lse - t / s;
    if (pred) pred[r] = idx;
    if (correct) correct[r] = (labelled && idx == label) ? 1 : 0;
    if (lse_out) lse_out[r] = lse;
  }
}

int maps(CUtensorMap* mh, CUtensorMap* mw, const void* hidden, int64_t ldh, const void* weight,
         int64_t ldw, int64_t rows, int64_t vocab, int64_t hdim) {
  if (int s = tc_host::encode_2d(mh, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, hidden, hdim, rows,
                                 ldh * 2, 64, tcg::BM, CU_TENSOR_MAP_SWIZZLE_128B))
    return s;
  return tc_host::encode_2d(mw, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, weight, hdim, vocab, ldw * 2, 64,
                            kBN, CU_TENSOR_MAP_SWIZZLE_128B);
}

int check(int64_t rows, int64_t vocab, int64_t hdim, const void* a, const void* b,
          const char* what) {
  if (rows < 0 || vocab <= 0 || hdim <= 0 || rows > (1 << 30) || vocab > (1 << 30) || hdim > (1 << 30))
    return qb::fail(QB_ERR_INVALID, "%s: bad shape", what);
  if (rows > 0 && (!a || !b)) return qb::fail(QB_ERR_INVALID, "%s: null pointer", what);
  return QB_OK;
}


int stats(const void* hidden, int64_t ldh, const void* weight, int64_t ldw,
          const int64_t* target, int64_t rows, int64_t vocab, int64_t hdim, void* partials,
          float* z_label, float* logits, int64_t ldl, cudaStream_t stream, const char* what) {
  if (int s = check(rows, vocab, hdim, hidden, weight, what)) return s;
  if (rows == 0) return QB_OK;
  if (!target || !partials || !z_label) return qb::fail(QB_ERR_INVALID, "%s: null pointer", what);
  if (logits && ldl < vocab) return qb::fail(QB_ERR_INVALID, "%s: logits row stride", what);
  CUtensorMap mh, mw;
  if (int s = maps(&mh, &mw, hidden, ldh, weight, ldw, rows, vocab, hdim)) return s;
  tcg::Problem pb{static_cast<int>(rows), static_cast<int>(vocab), static_cast<int>((hdim + 63) / 64),
                  0, static_cast<int>((rows + 127) / 128), static_cast<int>((vocab + kBN - 1) / kBN)};
  EpiStats epi{static_cast<float4*>(partials), z_label, target, static_cast<int>(rows),
                static_cast<int>(vocab), logits, ldl,
                logits && qb::aligned16(logits) && (ldl * 4) % 16 == 0};
  return tcg::launch<tcg::kTmaK, tcg::kTmaK, tcg::kTmaK, tcg::kTmaK, kBN>(
      mh, mw, mh, mw, pb, epi, stream, what);
}

}  // namespace

extern "C" int64_t qb_linear_ce_vocab_tiles(int64_t vocab) { return (vocab + kBN - 1) / kBN; }

extern "C" int qb_linear_ce_stats(const void* hidden, int64_t ldh, const void* weight,
                                  int64_t ldw, const int64_t* target, int64_t rows,
                                  int64_t vocab, int64_t hdim, void* partials, float* z_label,
                                  cudaStream_t stream) {
  return stats(hidden, ldh, weight, ldw, target, rows, vocab, hdim, partials, z_label, nullptr, 0,
               stream, "linear_ce_stats");
}

extern "C" int qb_linear_ce_stats_logits(const void* hidden, int64_t ldh, const void* weight,
                                         int64_t ldw, const int64_t* target, int64_t rows,
                                         int64_t vocab, int64_t hdim, void* partials,
                                         float* z_label, float* logits, int64_t ldl,
                                         cudaStream_t stream) {
  if (!logits) return qb::fail(QB_ERR_INVALID, "linear_ce_stats_logits: null logits");
  return stats(hidden, ldh, weight, ldw, target, rows, vocab, hdim, partials, z_label, logits,
               ldl, stream, "linear_ce_stats_logits");
}

extern "C" int qb_ce_grad_from_logits(const float* logits, int64_t ldl, const int64_t* target,
                                      int64_t rows, int64_t vocab, const float* lse,
                                      const float* scale_dev, void* dz, int64_t ldz,
                                      cudaStream_t stream) {
  if (rows < 0 || vocab <= 0 || rows > 0x7fffffff || vocab > (1 << 30) || ldl < vocab || ldz < vocab)
    return qb::fail(QB_ERR_INVALID, "ce_grad_from_logits: bad shape");
  if (rows == 0) return QB_OK;
  if (!logits || !target || !lse || !scale_dev || !dz)
    return qb::fail(QB_ERR_INVALID, "ce_grad_from_logits: null pointer");
  const bool vec = qb::aligned16(logits) && (ldl * 4) % 16 == 0 && qb::aligned16(dz) &&
                   (ldz * 2) % 16 == 0;
  ce_grad_from_logits_kernel<<<static_cast<unsigned>(rows), 256, 0, stream>>>(
      logits, ldl, target, lse, scale_dev, static_cast<__nv_bfloat16*>(dz), ldz,
      static_cast<int>(vocab), vec);
  return qb::check_launch("ce_grad_from_logits");
}

extern "C" int qb_ce_reduce(const void* partials, int64_t n_vtiles, int64_t rows, int64_t vocab,
                            const int64_t* target, const float* z_label, float* loss,
                            float* entropy, int64_t* pred, int32_t* correct, float* lse,
                            cudaStream_t stream) {
  if (rows < 0 || n_vtiles <= 0 || rows > (1 << 30)) return qb::fail(QB_ERR_INVALID, "ce_reduce: bad shape");
  if (rows == 0) return QB_OK;
  if (!partials || !target || !z_label || !loss || !entropy)
    return qb::fail(QB_ERR_INVALID, "ce_reduce: null pointer");
  const int warps = 8;
  const unsigned grid = static_cast<unsigned>((rows + warps - 1) / warps);
  ce_reduce_kernel<<<grid, warps * 32, 0, stream>>>(
      static_cast<const float4*>(partials), static_cast<int>(n_vtiles), static_cast<int>(rows),
      target, z_label, loss, entropy, pred, correct, lse, static_cast<int>(vocab));
  return qb::check_launch("ce_reduce");
}

extern "C" int qb_linear_ce_grad(const void* hidden, int64_t ldh, const void* weight,
                                 int64_t ldw, const int64_t* target, int64_t rows, int64_t vocab,
                                 int64_t hdim, const float* lse, const float* scale_dev,
                                 void* dz, int64_t ldz, cudaStream_t stream) {
  if (int s = check(rows, vocab, hdim, hidden, weight, "linear_ce_grad")) return s;
  if (rows == 0) return QB_OK;
  if (!target || !lse || !scale_dev || !dz) return qb::fail(QB_ERR_INVALID, "linear_ce_grad: null pointer");
  CUtensorMap mh, mw;
  if (int s = maps(&mh, &mw, hidden, ldh, weight, ldw, rows, vocab, hdim)) return s;
  tcg::Problem pb{static_cast<int>(rows), static_cast<int>(vocab), static_cast<int>((hdim + 63) / 64),
                  0, static_cast<int>((rows + 127) / 128), static_cast<int>((vocab + kBN - 1) / kBN)};
  const bool vec = qb::aligned16(dz) && (ldz * 2) % 16 == 0;
  EpiGrad epi{static_cast<__nv_bfloat16*>(dz), ldz, target, lse, scale_dev,
              static_cast<int>(rows), static_cast<int>(vocab), vec};
  if (vec) {   // dz as TMA stores it from the epilogue's staging boxes
    if (int s = tc_host::encode_2d(&epi.dmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, dz, vocab, rows,
                                   ldz * 2, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B))
      return s;
    epi.tma = true;
  }
  return tcg::launch<tcg::kTmaK, tcg::kTmaK, tcg::kTmaK, tcg::kTmaK, kBN>(
      mh, mw, mh, mw, pb, epi, stream, "linear_ce_grad");
}
