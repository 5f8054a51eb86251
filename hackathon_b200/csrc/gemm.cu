// Plain bf16 GEMMs on the tcgen05 kernel, fp32 accumulation, fp32 or bf16 output:
//   qb_gemm_bf16    C[M,N] = A[M,K] * B[N,K]^T (+ bias[N])
//   qb_gemm2_bf16   C[M,N] = A0[M,K0] * B0[N,K0]^T + A1[M,K1] * B1[N,K1]^T (+ bias[N])
//   qb_gemm_bf16_acc_f32   C[M,N] (fp32) = beta * C + alpha * A[M,K] * B[N,K]^T (beta 0 or 1),
//                          K split over the SMs
//                          (partials in a workspace, summed in a fixed order: deterministic)
// Each operand may be K-major or MN-major in HBM (qb_gemm_bf16: every orientation the suite
// needs — logits = H W^T, dH = dZ W, LoRA products; qb_gemm2_bf16: the two layouts of a
// projection with its LoRA term as extra K, forward and input gradient).
#include <cstdlib>

#include "tc_gemm_pair.cuh"

namespace {

constexpr int kBN = 256;

// Row-major store: each epilogue thread owns one output row of the tile and writes its 32
// consecutive columns per TMEM chunk with 16-byte stores; optionally adds a bias row and a
// residual matrix of the output's type first (one rounding of acc + bias + residual).
//
// With a tensor map of C (`tma`), the one-CTA kernel gives each epilogue warp two [32 x 32]
// staging boxes in shared memory: each thread writes its row of the box (16-byte pieces, in the
// 64-byte / 128-byte swizzle of the map, so a warp's writes hit every bank once), and one lane
// stores the box with a TMA store — whole lines to L2 instead of 32 rows of 16 bytes per store
// instruction. The two boxes alternate; a box is rewritten only after its previous store has
// read it.
template <typename OutT>
struct EpiStoreRow {
  OutT* c;
  int64_t ldc;
  int M, N;
  const float* bias;  // [N] or null
  const OutT* resid;  // [M, N] (row stride ldr) or null
  int64_t ldr;
  bool vec;           // 16-byte aligned rows (output and residual)
  bool tma = false;   // cmap holds C: [M, N], box 32 x 32, 64-byte (bf16) / 128-byte (fp32) swizzle
  CUtensorMap cmap;

  static constexpr int kRowBytes = 32 * static_cast<int>(sizeof(OutT));   // one box row
  static constexpr int kBoxBytes = 32 * kRowBytes;
  static constexpr int kStageBytes = 2 * kBoxBytes;

  // acc (+ bias) (+ residual) of 32 columns n.. of row m
  __device__ __forceinline__ void finish(float (&v)[32], int m, int n) const {
    if (bias) {
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] += (n + i < N) ? __ldg(bias + n + i) : 0.f;
    }
    if (resid && m < M) {
      const OutT* res = resid + static_cast<int64_t>(m) * ldr + n;
      if (vec && n + 32 <= N) {
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          float r[8];
          qb::load8(res + i, r);
#pragma unroll
          for (int j = 0; j < 8; ++j) v[i + j] += r[j];
        }
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (n + i < N) v[i] += qb::to_f(res[i]);
      }
    }
  }

  template <int BN>
  __device__ __forceinline__ void tile(int m0, int n0, int row, uint32_t taddr,
                                       uint8_t* stage) const {
    if (!tma) {
      tile<BN>(m0, n0, row, taddr);
      return;
    }
    const int lane = row & 31;
    const int m = m0 + row;
    const int mw = m - lane;   // the warp's first row
    if (lane == 0) tc::bulk_wait_read_all();   // the previous tile's boxes are free
    __syncwarp();
#pragma unroll 1
    for (int ch = 0; ch < BN / 32; ++ch) {
      float v[32];
      tc::tmem_ld32(taddr + ch * 32, v);
      const int n = n0 + ch * 32;
      if (n >= N) continue;   // warp-uniform
      finish(v, m, n);
      uint8_t* box = stage + (ch & 1) * kBoxBytes;
      if (ch >= 2) {   // the store of chunk ch - 2 read this box
        if (lane == 0) tc::bulk_wait_read_newest_pending();
        __syncwarp();
      }
      uint8_t* dst = box + lane * kRowBytes;
#pragma unroll
      for (int p = 0; p < kRowBytes / 16; ++p) {
        const int sp = sizeof(OutT) == 2 ? (p ^ ((lane >> 1) & 3)) : (p ^ (lane & 7));
        constexpr int kPer = qb::Vec16<OutT>::N;   // elements per 16 bytes
        qb::Vec16<OutT> w;
#pragma unroll
        for (int i = 0; i < kPer; ++i) w.v[i] = qb::from_f<OutT>(v[p * kPer + i]);
        *reinterpret_cast<uint4*>(dst + sp * 16) = w.u;
      }
      tc::fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0 && mw < M) {   // rows past M and columns past N are clipped by the store
        tc::tma_store_2d(&cmap, box, n, mw);
        tc::bulk_commit();
      }
    }
  }

  template <int BN>
  __device__ __forceinline__ void tile(int m0, int n0, int row, uint32_t taddr) const {
    const int m = m0 + row;
#pragma unroll 1
    for (int ch = 0; ch < BN / 32; ++ch) {
      float v[32];
      tc::tmem_ld32(taddr + ch * 32, v);
      const int n = n0 + ch * 32;
      if (m >= M || n >= N) continue;
      if (bias) {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] += (n + i < N) ? __ldg(bias + n + i) : 0.f;
      }
      OutT* dst = c + static_cast<int64_t>(m) * ldc + n;
      const OutT* res = resid ? resid + static_cast<int64_t>(m) * ldr + n : nullptr;
      if (vec && n + 32 <= N) {
        if (res) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            float r[8];
            qb::load8(res + i, r);
#pragma unroll
            for (int j = 0; j < 8; ++j) v[i + j] += r[j];
          }
        }
#pragma unroll
        for (int i = 0; i < 32; i += 8) qb::store8<OutT>(dst + i, v + i);
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (n + i < N) dst[i] = qb::from_f<OutT>(v[i] + (res ? qb::to_f(res[i]) : 0.f));
      }
    }
  }
};

// C = (accumulate ? C : 0) + alpha * the tile, fp32 (one work item per tile): each element is
// read and written by the one thread that owns its row.
struct EpiAccF32 {
  float* c;
  int64_t ldc;
  int M, N;
  float alpha;
  bool vec;          // 16-byte aligned rows
  bool accumulate;   // false: C is written without being read

  template <int BN>
  __device__ __forceinline__ void tile(int m0, int n0, int row, uint32_t taddr) const {
    const int m = m0 + row;
#pragma unroll 1
    for (int ch = 0; ch < BN / 32; ++ch) {
      float v[32];
      tc::tmem_ld32(taddr + ch * 32, v);
      const int n = n0 + ch * 32;
      if (m >= M || n >= N) continue;
      float* dst = c + static_cast<int64_t>(m) * ldc + n;
      if (vec && n + 32 <= N) {
#pragma unroll
        for (int i = 0; i < 32; i += 4) {
          float4 o = accumulate ? *reinterpret_cast<const float4*>(dst + i)
                                : make_float4(0.f, 0.f, 0.f, 0.f);
          o.x += alpha * v[i];
          o.y += alpha * v[i + 1];
          o.z += alpha * v[i + 2];
          o.w += alpha * v[i + 3];
          *reinterpret_cast<float4*>(dst + i) = o;
        }
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (n + i < N) dst[i] = (accumulate ? dst[i] : 0.f) + alpha * v[i];
      }
    }
  }
};

// The raw fp32 partial product of one split-K work item into the workspace: row m0 + row of
// [splits x Mp, ldw] (the kernel passes m0 already offset by split x Mp; Mp = M padded to whole
// tiles), columns below N. split_reduce_kernel then sums the splits in order.
struct EpiPartialF32 {
  float* ws;
  int64_t ldw;   // a multiple of 4: 16-byte rows
  int N;

  template <int BN>
  __device__ __forceinline__ void tile(int m0, int n0, int row, uint32_t taddr) const {
    const int64_t m = static_cast<int64_t>(m0) + row;
#pragma unroll 1
    for (int ch = 0; ch < BN / 32; ++ch) {
      float v[32];
      tc::tmem_ld32(taddr + ch * 32, v);
      const int n = n0 + ch * 32;
      if (n >= N) continue;
      float* dst = ws + m * ldw + n;
      if (n + 32 <= N) {
#pragma unroll
        for (int i = 0; i < 32; i += 4)
          *reinterpret_cast<float4*>(dst + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (n + i < N) dst[i] = v[i];
      }
    }
  }
};

// C[m, n] = (ACC ? C[m, n] : 0) + alpha * (((P_0 + P_1) + P_2) + ...) over the splits'
// partials P_s (rows s x Mp of the workspace): a fixed summation order, so a split launch gives
// the same bits every time. VEC: four columns per thread (N, ldc and ldw multiples of 4, C
// 16-byte aligned).
template <bool VEC, bool ACC>
__global__ void __launch_bounds__(256)
split_reduce_kernel(const float* __restrict__ ws, int64_t ldw, int64_t split_stride, int splits,
                    float alpha, float* __restrict__ c, int64_t ldc, int M, int N) {
  const int per_row = VEC ? N / 4 : N;
  const int64_t total = static_cast<int64_t>(M) * per_row;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t m = i / per_row;
    const int n = static_cast<int>(i - m * per_row) * (VEC ? 4 : 1);
    const float* p = ws + m * ldw + n;
    float* dst = c + m * ldc + n;
    if (VEC) {
      float4 acc = __ldg(reinterpret_cast<const float4*>(p));
      for (int sp = 1; sp < splits; ++sp) {
        const float4 q = __ldg(reinterpret_cast<const float4*>(p + sp * split_stride));
        acc.x += q.x;
        acc.y += q.y;
        acc.z += q.z;
        acc.w += q.w;
      }
      float4 o = ACC ? *reinterpret_cast<const float4*>(dst) : make_float4(0.f, 0.f, 0.f, 0.f);
      o.x += alpha * acc.x;
      o.y += alpha * acc.y;
      o.z += alpha * acc.z;
      o.w += alpha * acc.w;
      *reinterpret_cast<float4*>(dst) = o;
    } else {
      float acc = __ldg(p);
      for (int sp = 1; sp < splits; ++sp) acc += __ldg(p + sp * split_stride);
      *dst = (ACC ? *dst : 0.f) + alpha * acc;
    }
  }
}

// Gate / up pair with SwiGLU: the tile's first BN/2 accumulator columns are gate features
// j0..j0+BN/2-1 (j0 = n0 / 2), the last BN/2 the same up features. Each is rounded to bf16 — the
// value the separate projections would store — and h = g * sigmoid(g) * u in fp32 (the
// arithmetic of the SwiGLU kernel) is stored as bf16; g and u themselves only when asked for
// (the backward's inputs).
__device__ __forceinline__ float swiglu_sigmoid(float g) { return 1.0f / (1.0f + __expf(-g)); }

//
// With tensor maps of h (and g, u) (`tma`), the one-CTA kernel stages each 32-column chunk of the
// warp's 32 rows in shared memory (64-byte swizzle: a warp's 16-byte writes hit every bank once)
// and one lane stores h (and g, u) with TMA stores.
struct EpiSwiGLU {
  __nv_bfloat16* h;
  int64_t ldh;
  __nv_bfloat16* g;   // or null
  __nv_bfloat16* u;   // or null
  int64_t ldgu;
  int M, I;
  bool vec;
  bool tma = false;   // hmap (and gmap, umap when g is stored): [M, I], box 32 x 32, 64-byte swizzle
  CUtensorMap hmap, gmap, umap;

  static constexpr int kBoxBytes = 32 * 64;
  static constexpr int kStageBytes = 3 * kBoxBytes;   // h, g, u boxes of one chunk

  template <int BN>
  __device__ __forceinline__ void tile(int m0, int n0, int row, uint32_t taddr,
                                       uint8_t* stage) const {
    if (!tma) {
      tile<BN>(m0, n0, row, taddr);
      return;
    }
    const int lane = row & 31;
    const int mw = m0 + row - lane;   // the warp's first row
    const int j0 = n0 / 2;
#pragma unroll 1
    for (int c = 0; c < BN / 64; ++c) {
      float gv[32], uv[32];
      tc::tmem_ld32(taddr + c * 32, gv);
      tc::tmem_ld32(taddr + BN / 2 + c * 32, uv);
      const int j = j0 + c * 32;
      if (j >= I) continue;   // warp-uniform
      float hv[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        gv[i] = __bfloat162float(__float2bfloat16_rn(gv[i]));
        uv[i] = __bfloat162float(__float2bfloat16_rn(uv[i]));
        hv[i] = gv[i] * swiglu_sigmoid(gv[i]) * uv[i];
      }
      if (lane == 0) tc::bulk_wait_read_all();   // the previous chunk's boxes are free
      __syncwarp();
      tcg::stage_row_bf16(stage, lane, hv);
      if (g) {
        tcg::stage_row_bf16(stage + kBoxBytes, lane, gv);
        tcg::stage_row_bf16(stage + 2 * kBoxBytes, lane, uv);
      }
      tc::fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0 && mw < M) {   // rows past M and columns past I are clipped by the stores
        tc::tma_store_2d(&hmap, stage, j, mw);
        if (g) {
          tc::tma_store_2d(&gmap, stage + kBoxBytes, j, mw);
          tc::tma_store_2d(&umap, stage + 2 * kBoxBytes, j, mw);
        }
        tc::bulk_commit();
      }
    }
  }

  template <int BN>
  __device__ __forceinline__ void tile(int m0, int n0, int row, uint32_t taddr) const {
    const int m = m0 + row;
    const int j0 = n0 / 2;
#pragma unroll 1
    for (int c = 0; c < BN / 64; ++c) {
      float gv[32], uv[32];
      tc::tmem_ld32(taddr + c * 32, gv);
      tc::tmem_ld32(taddr + BN / 2 + c * 32, uv);
      const int j = j0 + c * 32;
      if (m >= M || j >= I) continue;
      float hv[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        gv[i] = __bfloat162float(__float2bfloat16_rn(gv[i]));
        uv[i] = __bfloat162float(__float2bfloat16_rn(uv[i]));
        hv[i] = gv[i] * swiglu_sigmoid(gv[i]) * uv[i];
      }
      const int64_t oh = static_cast<int64_t>(m) * ldh + j;
      const int64_t og = static_cast<int64_t>(m) * ldgu + j;
      if (vec && j + 32 <= I) {
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          qb::store8<__nv_bfloat16>(h + oh + i, hv + i);
          if (g) {
            qb::store8<__nv_bfloat16>(g + og + i, gv + i);
            qb::store8<__nv_bfloat16>(u + og + i, uv + i);
          }
        }
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          if (j + i >= I) break;
          h[oh + i] = __float2bfloat16_rn(hv[i]);
          if (g) {
            g[og + i] = __float2bfloat16_rn(gv[i]);
            u[og + i] = __float2bfloat16_rn(uv[i]);
          }
        }
      }
    }
  }
};

// Projection output with the rotate-half RoPE of its heads applied (q / k, head_dim 128): each
// row is a token at position m % S; acc + bias is rounded to bf16 — the projection's output —
// then rotated in fp32 with that position's cos/sin (qb::rope_rotate, the RoPE kernel's
// arithmetic) and rounded again. A 256-wide tile holds two whole heads; chunk c (32 columns)
// pairs with chunk c + 2 (dims d and d + 64 of the same head).
//
// With a tensor map of C (`tma`), the one-CTA kernel stages the two 32-column pieces of each
// (first half, second half) pair in shared memory and one lane stores them with TMA stores; the
// two pair buffers alternate.
struct EpiStoreRope {
  __nv_bfloat16* c;
  int64_t ldc;
  int M, N, S;
  const float* bias;            // [N] or null
  const __nv_bfloat16* cosp;    // [S, 128], row stride css
  const __nv_bfloat16* sinp;
  int64_t css;
  bool vec;
  bool tma = false;   // cmap holds C: [M, N], box 32 x 32, 64-byte swizzle
  CUtensorMap cmap;

  static constexpr int kBoxBytes = 32 * 64;
  static constexpr int kStageBytes = 4 * kBoxBytes;

  // the rotated pair (x1 at column n1 = n0 + ch * 32, x2 at n1 + 64) of one row
  __device__ __forceinline__ void rotate(float (&x1)[32], float (&x2)[32], int ch, int n1,
                                         const __nv_bfloat16* cr,
                                         const __nv_bfloat16* sr) const {
    const int d = (ch & 1) * 32;             // dim of x1[0] within its head
    float c1[32], c2[32], s1[32], s2[32];
#pragma unroll
    for (int i = 0; i < 32; i += 8) {
      qb::load8(cr + d + i, c1 + i);
      qb::load8(cr + 64 + d + i, c2 + i);
      qb::load8(sr + d + i, s1 + i);
      qb::load8(sr + 64 + d + i, s2 + i);
    }
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const float a = x1[i] + (bias ? __ldg(bias + n1 + i) : 0.f);
      const float b = x2[i] + (bias ? __ldg(bias + n1 + 64 + i) : 0.f);
      qb::rope_rotate(__bfloat162float(__float2bfloat16_rn(a)),
                      __bfloat162float(__float2bfloat16_rn(b)), c1[i], c2[i], s1[i], s2[i],
                      x1[i], x2[i]);
    }
  }

  template <int BN>
  __device__ __forceinline__ void tile(int m0, int n0, int row, uint32_t taddr,
                                       uint8_t* stage) const {
    static_assert(BN % 128 == 0, "whole heads of 128 per tile");
    if (!tma) {
      tile<BN>(m0, n0, row, taddr);
      return;
    }
    const int lane = row & 31;
    const int m = m0 + row;
    const int mw = m - lane;   // the warp's first row
    const bool live = m < M;
    const __nv_bfloat16* cr = cosp + static_cast<int64_t>(live ? m % S : 0) * css;
    const __nv_bfloat16* sr = sinp + static_cast<int64_t>(live ? m % S : 0) * css;
    if (lane == 0) tc::bulk_wait_read_all();   // the previous tile's buffers are free
    __syncwarp();
#pragma unroll 1
    for (int p = 0; p < BN / 64; ++p) {
      const int ch = (p & 1) + (p >> 1) * 4;   // 0, 1, 4, 5: first halves of the two heads
      float x1[32], x2[32];
      tc::tmem_ld32(taddr + ch * 32, x1);
      tc::tmem_ld32(taddr + (ch + 2) * 32, x2);
      const int n1 = n0 + ch * 32;
      if (n1 >= N) continue;   // warp-uniform; N is whole heads, so n1 + 64 < N too
      rotate(x1, x2, ch, n1, cr, sr);
      uint8_t* pair = stage + (p & 1) * 2 * kBoxBytes;
      if (p >= 2) {   // the stores of pair p - 2 read this buffer
        if (lane == 0) tc::bulk_wait_read_newest_pending();
        __syncwarp();
      }
      tcg::stage_row_bf16(pair, lane, x1);
      tcg::stage_row_bf16(pair + kBoxBytes, lane, x2);
      tc::fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0 && mw < M) {   // rows past M are clipped by the stores
        tc::tma_store_2d(&cmap, pair, n1, mw);
        tc::tma_store_2d(&cmap, pair + kBoxBytes, n1 + 64, mw);
        tc::bulk_commit();
      }
    }
  }

  template <int BN>
  __device__ __forceinline__ void tile(int m0, int n0, int row, uint32_t taddr) const {
    static_assert(BN % 128 == 0, "whole heads of 128 per tile");
    const int m = m0 + row;
    const bool live = m < M;
    const __nv_bfloat16* cr = cosp + static_cast<int64_t>(live ? m % S : 0) * css;
    const __nv_bfloat16* sr = sinp + static_cast<int64_t>(live ? m % S : 0) * css;
#pragma unroll 1
    for (int p = 0; p < BN / 64; ++p) {
      const int ch = (p & 1) + (p >> 1) * 4;   // 0, 1, 4, 5: first halves of the two heads
      float x1[32], x2[32];
      tc::tmem_ld32(taddr + ch * 32, x1);
      tc::tmem_ld32(taddr + (ch + 2) * 32, x2);
      const int n1 = n0 + ch * 32, n2 = n1 + 64;
      if (!live || n1 >= N) continue;
      rotate(x1, x2, ch, n1, cr, sr);
      __nv_bfloat16* dst = c + static_cast<int64_t>(m) * ldc;
      if (vec) {
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          qb::store8<__nv_bfloat16>(dst + n1 + i, x1 + i);
          qb::store8<__nv_bfloat16>(dst + n2 + i, x2 + i);
        }
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          dst[n1 + i] = __float2bfloat16_rn(x1[i]);
          dst[n2 + i] = __float2bfloat16_rn(x2[i]);
        }
      }
    }
  }
};

int map_operand(CUtensorMap* map, const void* p, int64_t ld, bool mn_major, int64_t rows,
                int64_t k, int box_rows) {
  // K-major: [rows, k] with row stride ld; MN-major: stored [k, rows] with row stride ld
  if (!mn_major)
    return tc_host::encode_2d(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, p, k, rows, ld * 2, 64,
                              box_rows, CU_TENSOR_MAP_SWIZZLE_128B);
  return tc_host::encode_2d(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, p, rows, k, ld * 2, 64, 64,
                            CU_TENSOR_MAP_SWIZZLE_128B);
}

template <int A0, int B0, int A1, int B1, int BN, typename OutT>
int run(const CUtensorMap (&m)[4], const tcg::Problem& pb, void* c, int64_t ldc,
        const float* bias, const void* resid, int64_t ldr, bool vec, cudaStream_t s,
        const char* what) {
  EpiStoreRow<OutT> epi{static_cast<OutT*>(c), ldc, pb.M, pb.N, bias,
                        static_cast<const OutT*>(resid), ldr, vec};
  if (qb::aligned16(c) && (ldc * static_cast<int64_t>(sizeof(OutT))) % 16 == 0) {
    // C as TMA stores it from the epilogue's staging boxes (EpiStoreRow)
    const bool f32 = sizeof(OutT) == 4;
    if (int e = tc_host::encode_2d(&epi.cmap,
                                   f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                       : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                                   c, pb.N, pb.M, ldc * sizeof(OutT), 32, 32,
                                   f32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B))
      return e;
    epi.tma = true;
  }
  return tcg::launch<A0, B0, A1, B1, BN>(m[0], m[1], m[2], m[3], pb, epi, s, what);
}

// Which launches take the 2-SM kernel (K-major A operands). By default none: the one-CTA kernel
// runs every GEMM (1.32-1.38 PFLOP/s at the 7B projection shapes; the 2-SM kernel measured
// 1.47-1.50). The 2-SM kernel was the default for large launches when runs of the 7B step began
// to stall, and it stays opt-in until that is explained. QB_GEMM_PAIR=2 takes it for launches
// with enough 256 x 256 pair tiles to give every SM pair one; QB_GEMM_PAIR=1 for every K-major-A
// launch (the tests' small and ragged shapes).
bool use_pair(bool a_k_major, int64_t M, int64_t N) {
  static const int mode = [] {
    const char* e = std::getenv("QB_GEMM_PAIR");
    return e ? std::atoi(e) : 0;
  }();
  if (!a_k_major || mode == 0) return false;
  if (mode == 1) return true;
  const int64_t pair_tiles = ((M + 255) / 256) * ((N + 255) / 256);
  return pair_tiles >= tc_host::sm_count() / 2;
}

// B tensor maps with 128-row boxes for the pair kernel (each CTA loads half of a 256-row tile);
// MN-major maps are already 64 x 64 boxes.
int pair_maps(CUtensorMap (&m)[4], const void* B0, int64_t ldb0, bool b0_mn, int64_t K0,
              const void* B1, int64_t ldb1, bool b1_mn, int64_t K1, int64_t N) {
  if (!b0_mn)
    if (int s = map_operand(&m[1], B0, ldb0, false, N, K0, tcp::kHalfN)) return s;
  if (!b1_mn)
    if (int s = map_operand(&m[3], B1, ldb1, false, N, K1, tcp::kHalfN)) return s;
  return QB_OK;
}

// The pair kernel's problem: 256-row m-blocks, the same 256-wide n-blocks.
tcg::Problem pair_problem(const tcg::Problem& pb) {
  tcg::Problem pp = pb;
  pp.num_m = (pb.M + 255) / 256;
  return pp;
}

template <int B0, int B1, typename OutT>
int run_pair(const CUtensorMap (&m)[4], const tcg::Problem& pb, void* c, int64_t ldc,
             const float* bias, const void* resid, int64_t ldr, bool vec, cudaStream_t s,
             const char* what) {
  EpiStoreRow<OutT> epi{static_cast<OutT*>(c), ldc, pb.M, pb.N, bias,
                        static_cast<const OutT*>(resid), ldr, vec};
  return tcp::launch<B0, B1>(m[0], m[1], m[2], m[3], pair_problem(pb), epi, s, what);
}

template <int A0, int B0, int A1, int B1>
int run_dtype(const CUtensorMap (&m)[4], const tcg::Problem& pb, void* c, int64_t ldc,
              int c_dtype, const float* bias, const void* resid, int64_t ldr, bool vec,
              cudaStream_t s, const char* what, const CUtensorMap* mpair = nullptr) {
  if constexpr (A0 == tcg::kTmaK && A1 == tcg::kTmaK) {
    if (mpair) {
      const CUtensorMap (&mp)[4] = *reinterpret_cast<const CUtensorMap(*)[4]>(mpair);
      if (c_dtype == QB_F32)
        return run_pair<B0, B1, float>(mp, pb, c, ldc, bias, resid, ldr, vec, s, what);
      return run_pair<B0, B1, __nv_bfloat16>(mp, pb, c, ldc, bias, resid, ldr, vec, s, what);
    }
  }
  if (c_dtype == QB_F32)
    return run<A0, B0, A1, B1, kBN, float>(m, pb, c, ldc, bias, resid, ldr, vec, s, what);
  return run<A0, B0, A1, B1, kBN, __nv_bfloat16>(m, pb, c, ldc, bias, resid, ldr, vec, s, what);
}

// run_dtype for a single-segment GEMM whose output tiles are `bn` wide (narrow_bn).
template <int A0, int B0>
int run_narrow(const CUtensorMap (&m)[4], const tcg::Problem& pb, void* c, int64_t ldc,
               int c_dtype, const float* bias, bool vec, cudaStream_t s, const char* what,
               int bn) {
  using tcg::kTmaK;
  if (bn == 64) {
    if (c_dtype == QB_F32)
      return run<A0, B0, kTmaK, kTmaK, 64, float>(m, pb, c, ldc, bias, nullptr, 0, vec, s, what);
    return run<A0, B0, kTmaK, kTmaK, 64, __nv_bfloat16>(m, pb, c, ldc, bias, nullptr, 0, vec, s,
                                                       what);
  }
  if (c_dtype == QB_F32)
    return run<A0, B0, kTmaK, kTmaK, 128, float>(m, pb, c, ldc, bias, nullptr, 0, vec, s, what);
  return run<A0, B0, kTmaK, kTmaK, 128, __nv_bfloat16>(m, pb, c, ldc, bias, nullptr, 0, vec, s,
                                                      what);
}

int check_common(const void* C, int c_dtype, int64_t M, int64_t N, const char* what) {
  if (M < 0 || N < 0 || M > (1 << 30) || N > (1 << 30))
    return qb::fail(QB_ERR_INVALID, "%s: bad shape", what);
  if (!C) return qb::fail(QB_ERR_INVALID, "%s: null output", what);
  if (c_dtype != QB_F32 && c_dtype != QB_BF16)
    return qb::fail(QB_ERR_INVALID, "%s: output must be F32 or BF16", what);
  return QB_OK;
}

tcg::Problem problem(int64_t M, int64_t N, int64_t K0, int64_t K1, int bn = kBN) {
  return tcg::Problem{static_cast<int>(M), static_cast<int>(N), static_cast<int>((K0 + 63) / 64),
                      static_cast<int>((K1 + 63) / 64), static_cast<int>((M + 127) / 128),
                      static_cast<int>((N + bn - 1) / bn), 1};
}

// Output tile width of a single-segment GEMM: skinny outputs (the rank-64 LoRA products) take
// 64- or 128-wide tiles instead of paying 256-wide MMAs for columns that do not exist.
int narrow_bn(int64_t N) { return N <= 64 ? 64 : (N <= 128 ? 128 : kBN); }

bool vec_ok(const void* C, int64_t ldc, int c_dtype) {
  return qb::aligned16(C) && (ldc * (c_dtype == QB_F32 ? 4 : 2)) % 16 == 0;
}

}  // namespace

extern "C" int qb_gemm_bf16(const void* A, int64_t lda, int a_mn_major, const void* B,
                            int64_t ldb, int b_mn_major, void* C, int64_t ldc, int c_dtype,
                            const float* bias, int64_t M, int64_t N, int64_t K,
                            cudaStream_t stream) {
  const char* what = "gemm_bf16";
  if (int s = check_common(C, c_dtype, M, N, what)) return s;
  if (K < 0 || K > (1 << 30)) return qb::fail(QB_ERR_INVALID, "%s: bad shape", what);
  if (M == 0 || N == 0) return QB_OK;
  if (K == 0) return qb::fail(QB_ERR_UNSUPPORTED, "%s: K == 0", what);
  if (!A || !B) return qb::fail(QB_ERR_INVALID, "%s: null pointer", what);
  CUtensorMap m[4];
  const bool pair = use_pair(!a_mn_major, M, N);
  const int bn = pair ? kBN : narrow_bn(N);
  if (int s = map_operand(&m[0], A, lda, a_mn_major != 0, M, K, tcg::BM)) return s;
  if (int s = map_operand(&m[1], B, ldb, b_mn_major != 0, N, K, bn)) return s;
  m[2] = m[0];
  m[3] = m[1];
  const tcg::Problem pb = problem(M, N, K, 0, bn);
  const bool vec = vec_ok(C, ldc, c_dtype);
  if (bn != kBN) {
    using namespace tcg;
    if (!a_mn_major && !b_mn_major)
      return run_narrow<kTmaK, kTmaK>(m, pb, C, ldc, c_dtype, bias, vec, stream, what, bn);
    if (!a_mn_major && b_mn_major)
      return run_narrow<kTmaK, kTmaMN>(m, pb, C, ldc, c_dtype, bias, vec, stream, what, bn);
    if (a_mn_major && !b_mn_major)
      return run_narrow<kTmaMN, kTmaK>(m, pb, C, ldc, c_dtype, bias, vec, stream, what, bn);
    return run_narrow<kTmaMN, kTmaMN>(m, pb, C, ldc, c_dtype, bias, vec, stream, what, bn);
  }
  CUtensorMap mp[4] = {m[0], m[1], m[2], m[3]};
  if (pair) {
    if (int s = pair_maps(mp, B, ldb, b_mn_major != 0, K, B, ldb, b_mn_major != 0, K, N)) return s;
  }
  const CUtensorMap* mpp = pair ? &mp[0] : nullptr;
  using namespace tcg;
  if (!a_mn_major && !b_mn_major)
    return run_dtype<kTmaK, kTmaK, kTmaK, kTmaK>(m, pb, C, ldc, c_dtype, bias, nullptr, 0, vec,
                                                 stream, what, mpp);
  if (!a_mn_major && b_mn_major)
    return run_dtype<kTmaK, kTmaMN, kTmaK, kTmaMN>(m, pb, C, ldc, c_dtype, bias, nullptr, 0, vec,
                                                   stream, what, mpp);
  if (a_mn_major && !b_mn_major)
    return run_dtype<kTmaMN, kTmaK, kTmaK, kTmaK>(m, pb, C, ldc, c_dtype, bias, nullptr, 0, vec,
                                                  stream, what);
  return run_dtype<kTmaMN, kTmaMN, kTmaK, kTmaK>(m, pb, C, ldc, c_dtype, bias, nullptr, 0, vec,
                                                 stream, what);
}

namespace {

// Split-K factor for `tiles` output tiles of `nk` k-blocks on `sms` persistent CTAs: the one that
// minimises waves x (k-blocks per item + a per-item cost of kItemCostKb k-blocks - the pipeline
// ramp and the partial tile's store), keeping 4 k-blocks per item at least. Few tiles (the LoRA
// weight gradients: 28 tiles over 256 k-blocks -> 5 splits, one wave) spread over the SMs.
constexpr int64_t kItemCostKb = 8;

int k_splits(int64_t tiles, int64_t nk, int64_t sms) {
  int64_t best = 1, best_cost = -1;
  const int64_t max_splits = nk / 4 > 1 ? (nk / 4 < 64 ? nk / 4 : 64) : 1;
  for (int64_t s = 1; s <= max_splits; ++s) {
    const int64_t waves = (tiles * s + sms - 1) / sms;
    const int64_t cost = waves * ((nk + s - 1) / s + kItemCostKb);
    if (best_cost < 0 || cost * 100 < best_cost * 99) {   // a split more must gain 1%
      best = s;
      best_cost = cost;
    }
  }
  return static_cast<int>(best);
}

struct AccPlan {
  tcg::Problem pb;
  int bn;
  int64_t ldw;         // workspace row stride (floats)
  int64_t ws_floats;   // 0 without split-K
};

AccPlan acc_plan(int64_t M, int64_t N, int64_t K) {
  AccPlan p;
  p.bn = narrow_bn(N);
  p.pb = problem(M, N, K, 0, p.bn);
  p.pb.splits = k_splits(static_cast<int64_t>(p.pb.num_m) * p.pb.num_n, p.pb.nk0,
                         tc_host::sm_count());
  p.ldw = (N + 3) / 4 * 4;
  p.ws_floats = p.pb.splits > 1
                    ? static_cast<int64_t>(p.pb.splits) * p.pb.num_m * tcg::BM * p.ldw : 0;
  return p;
}

template <bool VEC>
void launch_reduce(const AccPlan& p, float* ws, float alpha, bool acc, float* c, int64_t ldc,
                   unsigned blocks, cudaStream_t s) {
  const int64_t split_stride = static_cast<int64_t>(p.pb.num_m) * tcg::BM * p.ldw;
  if (acc)
    split_reduce_kernel<VEC, true><<<blocks, 256, 0, s>>>(ws, p.ldw, split_stride, p.pb.splits,
                                                          alpha, c, ldc, p.pb.M, p.pb.N);
  else
    split_reduce_kernel<VEC, false><<<blocks, 256, 0, s>>>(ws, p.ldw, split_stride, p.pb.splits,
                                                           alpha, c, ldc, p.pb.M, p.pb.N);
}

template <int A0, int B0, int BN>
int run_acc(const CUtensorMap (&m)[4], const AccPlan& p, float* c, int64_t ldc, float alpha,
            bool acc, float* ws, cudaStream_t s, const char* what) {
  const bool vec = qb::aligned16(c) && ldc % 4 == 0;
  if (p.pb.splits <= 1) {
    EpiAccF32 epi{c, ldc, p.pb.M, p.pb.N, alpha, vec, acc};
    return tcg::launch<A0, B0, tcg::kTmaK, tcg::kTmaK, BN>(m[0], m[1], m[2], m[3], p.pb, epi, s,
                                                           what);
  }
  EpiPartialF32 epi{ws, p.ldw, p.pb.N};
  if (int e = tcg::launch<A0, B0, tcg::kTmaK, tcg::kTmaK, BN>(m[0], m[1], m[2], m[3], p.pb, epi,
                                                              s, what))
    return e;
  const bool rvec = vec && p.pb.N % 4 == 0;
  const int64_t per_row = rvec ? p.pb.N / 4 : p.pb.N;
  int64_t blocks = (static_cast<int64_t>(p.pb.M) * per_row + 255) / 256;
  const int64_t cap = static_cast<int64_t>(tc_host::sm_count()) * 8;
  if (blocks > cap) blocks = cap;
  if (rvec)
    launch_reduce<true>(p, ws, alpha, acc, c, ldc, static_cast<unsigned>(blocks), s);
  else
    launch_reduce<false>(p, ws, alpha, acc, c, ldc, static_cast<unsigned>(blocks), s);
  return qb::check_launch(what);
}

template <int A0, int B0>
int run_acc_bn(const CUtensorMap (&m)[4], const AccPlan& p, float* c, int64_t ldc, float alpha,
               bool acc, float* ws, cudaStream_t s, const char* what) {
  if (p.bn == 64) return run_acc<A0, B0, 64>(m, p, c, ldc, alpha, acc, ws, s, what);
  if (p.bn == 128) return run_acc<A0, B0, 128>(m, p, c, ldc, alpha, acc, ws, s, what);
  return run_acc<A0, B0, kBN>(m, p, c, ldc, alpha, acc, ws, s, what);
}

}  // namespace

extern "C" int64_t qb_gemm_bf16_acc_f32_workspace(int64_t M, int64_t N, int64_t K) {
  if (M <= 0 || N <= 0 || K <= 0 || M > (1 << 30) || N > (1 << 30) || K > (1 << 30)) return 0;
  return acc_plan(M, N, K).ws_floats;
}

extern "C" int qb_gemm_bf16_acc_f32(const void* A, int64_t lda, int a_mn_major, const void* B,
                                    int64_t ldb, int b_mn_major, float alpha, float beta,
                                    float* C, int64_t ldc, int64_t M, int64_t N, int64_t K,
                                    float* workspace, int64_t workspace_floats,
                                    cudaStream_t stream) {
  const char* what = "gemm_bf16_acc_f32";
  if (int s = check_common(C, QB_F32, M, N, what)) return s;
  if (K < 0 || K > (1 << 30)) return qb::fail(QB_ERR_INVALID, "%s: bad shape", what);
  if (ldc < N) return qb::fail(QB_ERR_INVALID, "%s: output row stride", what);
  if (beta != 0.0f && beta != 1.0f) return qb::fail(QB_ERR_INVALID, "%s: beta is 0 or 1", what);
  if (M == 0 || N == 0) return QB_OK;
  if (K == 0) {   // C = beta * C: nothing to add; beta 0 clears C
    if (beta != 0.0f) return QB_OK;
    const cudaError_t e = cudaMemset2DAsync(C, ldc * sizeof(float), 0, N * sizeof(float), M,
                                            stream);
    if (e != cudaSuccess) return qb::fail(QB_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
    return QB_OK;
  }
  if (!A || !B) return qb::fail(QB_ERR_INVALID, "%s: null pointer", what);
  const AccPlan plan = acc_plan(M, N, K);
  if (plan.ws_floats > 0 &&
      (!workspace || workspace_floats < plan.ws_floats || !qb::aligned16(workspace)))
    return qb::fail(QB_ERR_INVALID, "%s: workspace of %lld floats (16-byte aligned) needed",
                    what, static_cast<long long>(plan.ws_floats));
  CUtensorMap m[4];
  if (int s = map_operand(&m[0], A, lda, a_mn_major != 0, M, K, tcg::BM)) return s;
  if (int s = map_operand(&m[1], B, ldb, b_mn_major != 0, N, K, plan.bn)) return s;
  m[2] = m[0];
  m[3] = m[1];
  using namespace tcg;
  const bool acc = beta != 0.0f;
  if (!a_mn_major && !b_mn_major)
    return run_acc_bn<kTmaK, kTmaK>(m, plan, C, ldc, alpha, acc, workspace, stream, what);
  if (!a_mn_major && b_mn_major)
    return run_acc_bn<kTmaK, kTmaMN>(m, plan, C, ldc, alpha, acc, workspace, stream, what);
  if (a_mn_major && !b_mn_major)
    return run_acc_bn<kTmaMN, kTmaK>(m, plan, C, ldc, alpha, acc, workspace, stream, what);
  return run_acc_bn<kTmaMN, kTmaMN>(m, plan, C, ldc, alpha, acc, workspace, stream, what);
}

extern "C" int qb_gemm2_bf16(const void* A0, int64_t lda0, int a0_mn_major, const void* B0,
                             int64_t ldb0, int b0_mn_major, int64_t K0, const void* A1,
                             int64_t lda1, int a1_mn_major, const void* B1, int64_t ldb1,
                             int b1_mn_major, int64_t K1, void* C, int64_t ldc, int c_dtype,
                             const float* bias, const void* residual, int64_t ldr, int64_t M,
                             int64_t N, cudaStream_t stream) {
  const char* what = "gemm2_bf16";
  if (K1 == 0 && !residual)
    return qb_gemm_bf16(A0, lda0, a0_mn_major, B0, ldb0, b0_mn_major, C, ldc, c_dtype, bias, M,
                        N, K0, stream);
  if (int s = check_common(C, c_dtype, M, N, what)) return s;
  if (K0 <= 0 || K1 < 0 || K0 > (1 << 30) || K1 > (1 << 30))
    return qb::fail(QB_ERR_INVALID, "%s: bad K", what);
  if (M == 0 || N == 0) return QB_OK;
  if (!A0 || !B0 || (K1 > 0 && (!A1 || !B1)))
    return qb::fail(QB_ERR_INVALID, "%s: null pointer", what);
  if (residual && ldr < N) return qb::fail(QB_ERR_INVALID, "%s: residual row stride", what);
  if (K1 == 0) {   // one segment with a residual
    A1 = A0; B1 = B0; lda1 = lda0; ldb1 = ldb0; K1 = K0;
    a1_mn_major = a0_mn_major; b1_mn_major = b0_mn_major;
  }
  const bool one = A1 == A0 && B1 == B0 && K1 == K0;
  // the two layouts a projection with its adapter term takes (forward / input gradient)
  const bool fwd = !a0_mn_major && !b0_mn_major && !a1_mn_major && !b1_mn_major;
  const bool bwd = !a0_mn_major && b0_mn_major && !a1_mn_major && b1_mn_major;
  if (!fwd && !bwd)
    return qb::fail(QB_ERR_UNSUPPORTED, "%s: A operands K-major, B operands both K- or MN-major",
                    what);
  CUtensorMap m[4];
  if (int s = map_operand(&m[0], A0, lda0, false, M, K0, tcg::BM)) return s;
  if (int s = map_operand(&m[1], B0, ldb0, bwd, N, K0, kBN)) return s;
  if (int s = map_operand(&m[2], A1, lda1, false, M, K1, tcg::BM)) return s;
  if (int s = map_operand(&m[3], B1, ldb1, bwd, N, K1, kBN)) return s;
  const tcg::Problem pb = problem(M, N, K0, one ? 0 : K1);
  const int es = c_dtype == QB_F32 ? 4 : 2;
  const bool vec = vec_ok(C, ldc, c_dtype) &&
                   (!residual || (qb::aligned16(residual) && (ldr * es) % 16 == 0));
  CUtensorMap mp[4] = {m[0], m[1], m[2], m[3]};
  const bool pair = use_pair(true, M, N);
  if (pair) {
    if (int s = pair_maps(mp, B0, ldb0, bwd, K0, B1, ldb1, bwd, K1, N)) return s;
  }
  const CUtensorMap* mpp = pair ? &mp[0] : nullptr;
  using namespace tcg;
  if (fwd)
    return run_dtype<kTmaK, kTmaK, kTmaK, kTmaK>(m, pb, C, ldc, c_dtype, bias, residual, ldr,
                                                 vec, stream, what, mpp);
  return run_dtype<kTmaK, kTmaMN, kTmaK, kTmaMN>(m, pb, C, ldc, c_dtype, bias, residual, ldr,
                                                 vec, stream, what, mpp);
}

namespace {

// Mask jobs of the C-ABI -> the kernel's side work (words, thresholds and each job's first word
// in the launch's word space).
int side_work(const qb_mask_job* jobs, int njobs, tcg::SideWork* side, const char* what) {
  if (njobs < 0 || njobs > tcg::kMaxMaskJobs || (njobs > 0 && !jobs))
    return qb::fail(QB_ERR_INVALID, "%s: 0..%d mask jobs", what, tcg::kMaxMaskJobs);
  *side = tcg::SideWork{};
  int64_t total = 0;
  for (int i = 0; i < njobs; ++i) {
    const qb_mask_job& j = jobs[i];
    if (j.rows < 0 || j.cols <= 0 || j.rows > (int64_t(1) << 31) || j.cols > (int64_t(1) << 31))
      return qb::fail(QB_ERR_INVALID, "%s: mask job %d: bad shape", what, i);
    if (!(j.p < 1.0f)) return qb::fail(QB_ERR_INVALID, "%s: mask job %d: p must be < 1", what, i);
    if (!j.bits || reinterpret_cast<uintptr_t>(j.bits) % 4)
      return qb::fail(QB_ERR_INVALID, "%s: mask job %d: bits must be 4-byte aligned", what, i);
    tcg::MaskJob& m = side->job[side->njobs++];
    m.bits = j.bits;
    m.rows = j.rows;
    m.cols = j.cols;
    m.words = (j.cols + 31) / 32;
    m.k0 = static_cast<uint32_t>(j.seed & 0xffffffffu);
    m.k1 = static_cast<uint32_t>(j.seed >> 32);
    m.thresh = qb::keep_threshold(j.p);
    m.first = total;
    total += j.rows * m.words;
  }
  side->total = total;
  return QB_OK;
}

// Side warps beside the GEMM's six: the 7B forward's seven masks (0.66 G Philox draws, 1.8 ms
// as their own launches) add 1.2 ms to the 3.3 ms gate/up GEMM with 8 side warps and 0.7-0.9 ms
// with 4 to 6 (the SMs share the power cap, so the draws are not free; fewer warps take fewer
// issue slots from the GEMM's producer, MMA and epilogue warps).
constexpr int kSideWarps = 6;

int gateup_swiglu(const void* x, int64_t ldx, const void* w_gate, const void* w_up, int64_t ldw,
                  int64_t K0, const void* u1, int64_t ldu1, const void* b1_gate,
                  const void* b1_up, int64_t ldb1, int64_t K1, void* h, int64_t ldh, void* g_out,
                  void* u_out, int64_t ldgu, int64_t M, int64_t I, const tcg::SideWork* side,
                  cudaStream_t stream) {
  const char* what = side ? "gemm_gateup_swiglu_masks" : "gemm_gateup_swiglu";
  if (M < 0 || I < 0 || K0 <= 0 || K1 < 0 || M > (1 << 30) || I > (1 << 29) || K0 > (1 << 30) ||
      K1 > (1 << 30))
    return qb::fail(QB_ERR_INVALID, "%s: bad shape", what);
  if (M == 0 || I == 0) return QB_OK;
  if (!x || !w_gate || !w_up || !h || (K1 > 0 && (!u1 || !b1_gate || !b1_up)))
    return qb::fail(QB_ERR_INVALID, "%s: null pointer", what);
  if ((g_out == nullptr) != (u_out == nullptr))
    return qb::fail(QB_ERR_INVALID, "%s: g and u outputs go together", what);
  if (ldh < I || (g_out && ldgu < I)) return qb::fail(QB_ERR_INVALID, "%s: output row stride", what);
  constexpr int kHalf = kBN / 2;
  CUtensorMap m[4], mb0b, mb1b;
  if (int s = map_operand(&m[0], x, ldx, false, M, K0, tcg::BM)) return s;
  if (int s = map_operand(&m[1], w_gate, ldw, false, I, K0, kHalf)) return s;
  if (int s = map_operand(&mb0b, w_up, ldw, false, I, K0, kHalf)) return s;
  if (K1 > 0) {
    if (int s = map_operand(&m[2], u1, ldu1, false, M, K1, tcg::BM)) return s;
    if (int s = map_operand(&m[3], b1_gate, ldb1, false, I, K1, kHalf)) return s;
    if (int s = map_operand(&mb1b, b1_up, ldb1, false, I, K1, kHalf)) return s;
  } else {
    m[2] = m[0];
    m[3] = m[1];
    mb1b = mb0b;
  }
  const int64_t halves = (I + kHalf - 1) / kHalf;
  tcg::Problem pb{static_cast<int>(M), static_cast<int>(2 * halves * kHalf),
                  static_cast<int>((K0 + 63) / 64), static_cast<int>((K1 + 63) / 64),
                  static_cast<int>((M + 127) / 128), static_cast<int>(halves)};
  const bool vec = qb::aligned16(h) && (ldh * 2) % 16 == 0 &&
                   (!g_out || (qb::aligned16(g_out) && qb::aligned16(u_out) && (ldgu * 2) % 16 == 0));
  EpiSwiGLU epi{static_cast<__nv_bfloat16*>(h), ldh, static_cast<__nv_bfloat16*>(g_out),
                static_cast<__nv_bfloat16*>(u_out), ldgu, static_cast<int>(M), static_cast<int>(I),
                vec};
  if (vec) {   // 16-byte aligned rows: h (and g, u) as TMA stores them from the staging boxes
    if (int e = tc_host::encode_2d(&epi.hmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, h, I, M, ldh * 2,
                                   32, 32, CU_TENSOR_MAP_SWIZZLE_64B))
      return e;
    if (g_out) {
      if (int e = tc_host::encode_2d(&epi.gmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, g_out, I, M,
                                     ldgu * 2, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B))
        return e;
      if (int e = tc_host::encode_2d(&epi.umap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, u_out, I, M,
                                     ldgu * 2, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B))
        return e;
    }
    epi.tma = true;
  }
  using namespace tcg;
  if (side)
    return launch<kTmaK, kTmaKDual, kTmaK, kTmaKDual, kBN, EpiSwiGLU, kSideWarps>(
        m[0], m[1], m[2], m[3], pb, epi, stream, what, &mb0b, &mb1b, *side);
  if (use_pair(true, M, 2 * halves * kHalf))   // the dual maps already have 128-row boxes
    return tcp::launch<kTmaKDual, kTmaKDual>(m[0], m[1], m[2], m[3], pair_problem(pb), epi, stream,
                                             what, &mb0b, &mb1b);
  return launch<kTmaK, kTmaKDual, kTmaK, kTmaKDual, kBN>(m[0], m[1], m[2], m[3], pb, epi, stream,
                                                         what, &mb0b, &mb1b);
}

}  // namespace

extern "C" int qb_gemm_gateup_swiglu(const void* x, int64_t ldx, const void* w_gate,
                                     const void* w_up, int64_t ldw, int64_t K0, const void* u1,
                                     int64_t ldu1, const void* b1_gate, const void* b1_up,
                                     int64_t ldb1, int64_t K1, void* h, int64_t ldh,
                                     void* g_out, void* u_out, int64_t ldgu, int64_t M,
                                     int64_t I, cudaStream_t stream) {
  return gateup_swiglu(x, ldx, w_gate, w_up, ldw, K0, u1, ldu1, b1_gate, b1_up, ldb1, K1, h, ldh,
                       g_out, u_out, ldgu, M, I, nullptr, stream);
}

extern "C" int64_t qb_mask_job_size(void) { return sizeof(qb_mask_job); }

extern "C" int qb_gemm_gateup_swiglu_masks(
    const void* x, int64_t ldx, const void* w_gate, const void* w_up, int64_t ldw, int64_t K0,
    const void* u1, int64_t ldu1, const void* b1_gate, const void* b1_up, int64_t ldb1,
    int64_t K1, void* h, int64_t ldh, void* g_out, void* u_out, int64_t ldgu, int64_t M,
    int64_t I, const qb_mask_job* jobs, int njobs, cudaStream_t stream) {
  tcg::SideWork side;
  if (int s = side_work(jobs, njobs, &side, "gemm_gateup_swiglu_masks")) return s;
  return gateup_swiglu(x, ldx, w_gate, w_up, ldw, K0, u1, ldu1, b1_gate, b1_up, ldb1, K1, h, ldh,
                       g_out, u_out, ldgu, M, I, njobs > 0 ? &side : nullptr, stream);
}

extern "C" int qb_gemm2_rope_bf16(const void* A0, int64_t lda0, const void* B0, int64_t ldb0,
                                  int64_t K0, const void* A1, int64_t lda1, const void* B1,
                                  int64_t ldb1, int64_t K1, void* C, int64_t ldc,
                                  const float* bias, const void* cos_, const void* sin_,
                                  int64_t cs_stride_s, int64_t S, int64_t head_dim, int64_t M,
                                  int64_t N, cudaStream_t stream) {
  const char* what = "gemm2_rope_bf16";
  if (M < 0 || N < 0 || K0 <= 0 || K1 < 0 || M > (1 << 30) || N > (1 << 30) || K0 > (1 << 30) ||
      K1 > (1 << 30) || S <= 0)
    return qb::fail(QB_ERR_INVALID, "%s: bad shape", what);
  if (head_dim != 128 || N % 128)
    return qb::fail(QB_ERR_UNSUPPORTED, "%s: heads of 128 dims, N a multiple of 128", what);
  if (M == 0 || N == 0) return QB_OK;
  if (!A0 || !B0 || !C || !cos_ || !sin_ || (K1 > 0 && (!A1 || !B1)))
    return qb::fail(QB_ERR_INVALID, "%s: null pointer", what);
  if (!qb::aligned16(cos_) || !qb::aligned16(sin_) || (cs_stride_s * 2) % 16)
    return qb::fail(QB_ERR_INVALID, "%s: cos/sin rows must be 16-byte aligned", what);
  CUtensorMap m[4];
  if (int s = map_operand(&m[0], A0, lda0, false, M, K0, tcg::BM)) return s;
  if (int s = map_operand(&m[1], B0, ldb0, false, N, K0, kBN)) return s;
  if (K1 > 0) {
    if (int s = map_operand(&m[2], A1, lda1, false, M, K1, tcg::BM)) return s;
    if (int s = map_operand(&m[3], B1, ldb1, false, N, K1, kBN)) return s;
  } else {
    m[2] = m[0];
    m[3] = m[1];
  }
  const tcg::Problem pb = problem(M, N, K0, K1);
  EpiStoreRope epi{static_cast<__nv_bfloat16*>(C), ldc, static_cast<int>(M), static_cast<int>(N),
                   static_cast<int>(S), bias, static_cast<const __nv_bfloat16*>(cos_),
                   static_cast<const __nv_bfloat16*>(sin_), cs_stride_s,
                   qb::aligned16(C) && (ldc * 2) % 16 == 0};
  if (epi.vec) {   // C as TMA stores it from the epilogue's staging boxes
    if (int e = tc_host::encode_2d(&epi.cmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, C, N, M, ldc * 2,
                                   32, 32, CU_TENSOR_MAP_SWIZZLE_64B))
      return e;
    epi.tma = true;
  }
  using namespace tcg;
  if (use_pair(true, M, N)) {
    if (int s = map_operand(&m[1], B0, ldb0, false, N, K0, tcp::kHalfN)) return s;
    if (K1 > 0) {
      if (int s = map_operand(&m[3], B1, ldb1, false, N, K1, tcp::kHalfN)) return s;
    } else {
      m[3] = m[1];
    }
    return tcp::launch<kTmaK, kTmaK>(m[0], m[1], m[2], m[3], pair_problem(pb), epi, stream, what);
  }
  return launch<kTmaK, kTmaK, kTmaK, kTmaK, kBN>(m[0], m[1], m[2], m[3], pb, epi, stream, what);
}
