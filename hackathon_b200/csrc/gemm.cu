// Plain bf16 GEMM on the tcgen05 kernel: C[M,N] = A[M,K] * B[N,K]^T (+ bias[N]), fp32
// accumulation, fp32 or bf16 output. A and B may each be K-major or MN-major in HBM, which covers
// every orientation the suite needs (logits = H W^T, dH = dZ W, LoRA products).
#include "tc_gemm.cuh"

namespace {

// Row-major store: each epilogue thread owns one output row of the tile and writes its 32
// consecutive columns per TMEM chunk with 16-byte stores.
template <typename OutT>
struct EpiStoreRow {
  OutT* c;
  int64_t ldc;
  int M, N;
  const float* bias;  // [N] or null
  bool vec;           // 16-byte aligned rows

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
      if (vec && n + 32 <= N) {
#pragma unroll
        for (int i = 0; i < 32; i += 8) qb::store8<OutT>(dst + i, v + i);
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (n + i < N) dst[i] = qb::from_f<OutT>(v[i]);
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

template <int AS, int BS, typename OutT>
int run(const CUtensorMap& ma, const CUtensorMap& mb, const tcg::Problem& pb, OutT* c,
        int64_t ldc, const float* bias, bool vec, cudaStream_t s) {
  EpiStoreRow<OutT> epi{c, ldc, pb.M, pb.N, bias, vec};
  return tcg::launch<AS, BS, tcg::kTmaK, tcg::kTmaK, 256>(ma, mb, ma, mb, pb, tcg::Nf4Operand{},
                                                          epi, s, "gemm_bf16");
}

}  // namespace

extern "C" int qb_gemm_bf16(const void* A, int64_t lda, int a_mn_major, const void* B,
                            int64_t ldb, int b_mn_major, void* C, int64_t ldc, int c_dtype,
                            const float* bias, int64_t M, int64_t N, int64_t K,
                            cudaStream_t stream) {
  if (M < 0 || N < 0 || K < 0 || M > (1 << 30) || N > (1 << 30) || K > (1 << 30))
    return qb::fail(QB_ERR_INVALID, "gemm_bf16: bad shape");
  if (M == 0 || N == 0) return QB_OK;
  if (K == 0) return qb::fail(QB_ERR_UNSUPPORTED, "gemm_bf16: K == 0");
  if (!A || !B || !C) return qb::fail(QB_ERR_INVALID, "gemm_bf16: null pointer");
  if (c_dtype != QB_F32 && c_dtype != QB_BF16)
    return qb::fail(QB_ERR_INVALID, "gemm_bf16: output must be F32 or BF16");
  CUtensorMap ma, mb;
  if (int s = map_operand(&ma, A, lda, a_mn_major != 0, M, K, 128)) return s;
  if (int s = map_operand(&mb, B, ldb, b_mn_major != 0, N, K, 256)) return s;
  tcg::Problem pb{static_cast<int>(M), static_cast<int>(N), static_cast<int>((K + 63) / 64), 0,
                  static_cast<int>((M + 127) / 128), static_cast<int>((N + 255) / 256)};
  const int es = c_dtype == QB_F32 ? 4 : 2;
  const bool vec = qb::aligned16(C) && (ldc * es) % 16 == 0;
#define QB_GEMM_CASE(AS, BS)                                                                 \
  if (c_dtype == QB_F32)                                                                     \
    return run<AS, BS, float>(ma, mb, pb, static_cast<float*>(C), ldc, bias, vec, stream);  \
  return run<AS, BS, __nv_bfloat16>(ma, mb, pb, static_cast<__nv_bfloat16*>(C), ldc, bias, \
                                    vec, stream);
  if (!a_mn_major && !b_mn_major) { QB_GEMM_CASE(tcg::kTmaK, tcg::kTmaK) }
  if (!a_mn_major && b_mn_major) { QB_GEMM_CASE(tcg::kTmaK, tcg::kTmaMN) }
  if (a_mn_major && !b_mn_major) { QB_GEMM_CASE(tcg::kTmaMN, tcg::kTmaK) }
  QB_GEMM_CASE(tcg::kTmaMN, tcg::kTmaMN)
#undef QB_GEMM_CASE
}
