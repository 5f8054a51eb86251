// The NF4-weight x LoRA projection on tcgen05, forward and input-gradient, with the base weight
// dequantised in registers straight into the MMA operand (no bf16 W in HBM).
//
// The GEMM runs "swapped": the weight is the A operand (128 weight rows or columns per tile,
// rebuilt by the dequant warps from packed codes that TMA brings in) and the tokens are B
// (512 per tile, by TMA, as two N=256 MMAs), so the dequant cost per flop is 1/512 weight per
// multiply-add. The epilogue writes the tile transposed into the
// row-major [tokens, features] output.
//
//   forward  Y^T[out, T]  = [ W | s*B_lora ] [ X | U ]^T (+ bias)       U = dropout(X) A_lora^T
//   dgrad    dX^T[in, T]  = [ W^T | A_lora^T ] [ dY | V ]^T             V = s * dY B_lora
// The LoRA term rides along as extra K (segment 1): the adapter's second GEMM, the reference's
// scaled add (solution/lora.py:49-60, :104) and the [T, out] adapter output disappear.
// Replaces solution/nf4.py:100-112 (F.linear / grad_out @ W on a dequantised weight) and the
// lora_B(lora_A(x)) + ScaledAdd of solution/lora.py:172-173.
#include "tc_nf4_gemm.cuh"

namespace {

constexpr int kBN = 256;

// Transposed store: D[m, t] -> out[t * ld + m] (+ bias[m]); lanes hold consecutive m, so every
// store instruction of a warp covers 64 contiguous bytes of one output row.
struct EpiStoreT {
  __nv_bfloat16* out;
  int64_t ld;
  const __nv_bfloat16* bias;  // [M] or null
  int M, N;

  template <int BN>
  __device__ __forceinline__ void tile(int m0, int n0, int row, uint32_t taddr) const {
    const int m = m0 + row;
    const float b = (bias && m < M) ? __bfloat162float(bias[m]) : 0.f;
#pragma unroll 1
    for (int ch = 0; ch < BN / 32; ++ch) {
      float v[32];
      tc::tmem_ld32(taddr + ch * 32, v);
      const int n = n0 + ch * 32;
      if (m >= M) continue;
      __nv_bfloat16* dst = out + static_cast<int64_t>(n) * ld + m;
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (n + i < N) dst[static_cast<int64_t>(i) * ld] = __float2bfloat16_rn(v[i] + b);
    }
  }
};

struct Nf4Ptrs {
  const uint8_t* packed;
  const uint8_t* absmax_q;
  const float* code2;
  const float* absmax2;
  float offset;
  int blocksize2;
  const float* lut16;
};

int check_nf4(const Nf4Ptrs& w, int64_t in_f, int64_t out_f, const char* what) {
  if (!w.packed || !w.absmax_q || !w.code2 || !w.absmax2 || !w.lut16)
    return qb::fail(QB_ERR_INVALID, "%s: null NF4 pointer", what);
  if (in_f <= 0 || out_f <= 0 || in_f % 64 || in_f > (1 << 30) || out_f > (1 << 30))
    return qb::fail(QB_ERR_INVALID, "%s: in_features must be a positive multiple of 64", what);
  if (w.blocksize2 <= 0) return qb::fail(QB_ERR_INVALID, "%s: blocksize2", what);
  if ((reinterpret_cast<uintptr_t>(w.packed) & 15u) != 0)
    return qb::fail(QB_ERR_INVALID, "%s: packed weights must be 16-byte aligned", what);
  return QB_OK;
}

tcn::Nf4Operand operand(const Nf4Ptrs& w, int64_t in_f, int64_t out_f) {
  tcn::Nf4Operand q;
  q.absmax_q = w.absmax_q;
  q.absmax2 = w.absmax2;
  q.code2 = w.code2;
  q.lut = w.lut16;
  q.offset = w.offset;
  q.blocksize2 = w.blocksize2;
  q.blocks_per_row = static_cast<int>(in_f / 64);
  q.rows = static_cast<int>(out_f);
  q.cols = static_cast<int>(in_f);
  return q;
}

int map_bf16(CUtensorMap* m, const void* p, int64_t inner, int64_t outer, int64_t ld, int box_in,
             int box_out) {
  return tc_host::encode_2d(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, p, inner, outer, ld * 2, box_in,
                            box_out, CU_TENSOR_MAP_SWIZZLE_128B);
}

int map_codes(CUtensorMap* m, const uint8_t* packed, int64_t in_f, int64_t out_f, int box_in,
              int box_out) {
  return tc_host::encode_2d(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, packed, in_f / 2, out_f, in_f / 2,
                            box_in, box_out, CU_TENSOR_MAP_SWIZZLE_NONE);
}

}  // namespace

extern "C" int qb_nf4_linear_fwd(const void* x, int64_t ldx, const uint8_t* packed,
                                 const uint8_t* absmax_q, const float* code2,
                                 const float* absmax2, float offset, int blocksize2,
                                 const float* lut16, int64_t tokens, int64_t in_f, int64_t out_f,
                                 const void* bias, const void* u, int64_t ldu,
                                 const void* lora_b_scaled, int64_t ldlb, int64_t r, void* y,
                                 int64_t ldy, cudaStream_t stream) {
  const Nf4Ptrs w{packed, absmax_q, code2, absmax2, offset, blocksize2, lut16};
  if (int s = check_nf4(w, in_f, out_f, "nf4_linear_fwd")) return s;
  if (tokens < 0 || tokens > (1 << 30)) return qb::fail(QB_ERR_INVALID, "nf4_linear_fwd: tokens");
  if (tokens == 0) return QB_OK;
  if (!x || !y) return qb::fail(QB_ERR_INVALID, "nf4_linear_fwd: null pointer");
  if (r < 0 || (r > 0 && (!u || !lora_b_scaled)))
    return qb::fail(QB_ERR_INVALID, "nf4_linear_fwd: LoRA operands");
  if (r > 0 && ((ldlb * 2) % 16 || r % 8 || (reinterpret_cast<uintptr_t>(lora_b_scaled) & 15u)))
    return qb::fail(QB_ERR_INVALID, "nf4_linear_fwd: LoRA B must have 16-byte rows and r %% 8 == 0");
  int shift = 0;
  while ((1 << shift) < blocksize2) ++shift;
  if ((1 << shift) != blocksize2) return qb::fail(QB_ERR_UNSUPPORTED, "nf4_linear_fwd: blocksize2 must be a power of two");
  CUtensorMap mC, mB0, mB1;
  if (int s = map_codes(&mC, packed, in_f, out_f, 32, tcg::BM)) return s;
  if (int s = map_bf16(&mB0, x, in_f, tokens, ldx, 64, kBN)) return s;
  if (r > 0) {
    if (int s = map_bf16(&mB1, u, r, tokens, ldu, 64, kBN)) return s;
  } else {
    mB1 = mB0;
  }
  tcn::NfProblem pb{static_cast<int>(out_f), static_cast<int>(tokens), static_cast<int>(in_f / 64),
                    static_cast<int>((r + 63) / 64), static_cast<int>((out_f + 127) / 128),
                    static_cast<int>((tokens + tcn::kTN - 1) / tcn::kTN), shift};
  tcn::LoraA lora{static_cast<const __nv_bfloat16*>(lora_b_scaled), ldlb, static_cast<int>(r)};
  EpiStoreT epi{static_cast<__nv_bfloat16*>(y), ldy, static_cast<const __nv_bfloat16*>(bias),
                static_cast<int>(out_f), static_cast<int>(tokens)};
  return tcn::launch_nf4<tcn::kNf4K>(mC, mB0, mB1, pb, operand(w, in_f, out_f), lora, epi, stream,
                                     "nf4_linear_fwd");
}

extern "C" int qb_nf4_linear_dgrad(const void* dy, int64_t lddy, const uint8_t* packed,
                                   const uint8_t* absmax_q, const float* code2,
                                   const float* absmax2, float offset, int blocksize2,
                                   const float* lut16, int64_t tokens, int64_t in_f,
                                   int64_t out_f, const void* v, int64_t ldv,
                                   const void* lora_a, int64_t ldla, int64_t r, void* dx,
                                   int64_t lddx, cudaStream_t stream) {
  const Nf4Ptrs w{packed, absmax_q, code2, absmax2, offset, blocksize2, lut16};
  if (int s = check_nf4(w, in_f, out_f, "nf4_linear_dgrad")) return s;
  if (in_f % 128) return qb::fail(QB_ERR_INVALID, "nf4_linear_dgrad: in_features must be a multiple of 128");
  if (tokens < 0 || tokens > (1 << 30)) return qb::fail(QB_ERR_INVALID, "nf4_linear_dgrad: tokens");
  if (tokens == 0) return QB_OK;
  if (!dy || !dx) return qb::fail(QB_ERR_INVALID, "nf4_linear_dgrad: null pointer");
  if (r < 0 || (r > 0 && (!v || !lora_a)))
    return qb::fail(QB_ERR_INVALID, "nf4_linear_dgrad: LoRA operands");
  if (r > 0 && ((ldla * 2) % 16 || r % 8 || (reinterpret_cast<uintptr_t>(lora_a) & 15u)))
    return qb::fail(QB_ERR_INVALID, "nf4_linear_dgrad: LoRA A must have 16-byte rows and r %% 8 == 0");
  int shift = 0;
  while ((1 << shift) < blocksize2) ++shift;
  if ((1 << shift) != blocksize2) return qb::fail(QB_ERR_UNSUPPORTED, "nf4_linear_dgrad: blocksize2 must be a power of two");
  CUtensorMap mC, mB0, mB1;
  if (int s = map_codes(&mC, packed, in_f, out_f, 64, 64)) return s;
  if (int s = map_bf16(&mB0, dy, out_f, tokens, lddy, 64, kBN)) return s;
  if (r > 0) {
    if (int s = map_bf16(&mB1, v, r, tokens, ldv, 64, kBN)) return s;
  } else {
    mB1 = mB0;
  }
  tcn::NfProblem pb{static_cast<int>(in_f), static_cast<int>(tokens),
                    static_cast<int>((out_f + 63) / 64), static_cast<int>((r + 63) / 64),
                    static_cast<int>(in_f / 128), static_cast<int>((tokens + tcn::kTN - 1) / tcn::kTN), shift};
  tcn::LoraA lora{static_cast<const __nv_bfloat16*>(lora_a), ldla, static_cast<int>(r)};
  EpiStoreT epi{static_cast<__nv_bfloat16*>(dx), lddx, nullptr, static_cast<int>(in_f),
                static_cast<int>(tokens)};
  return tcn::launch_nf4<tcn::kNf4MN>(mC, mB0, mB1, pb, operand(w, in_f, out_f), lora, epi,
                                      stream, "nf4_linear_dgrad");
}
