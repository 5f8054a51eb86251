// The persistent, warp-specialised tcgen05 GEMM every dense contraction of the suite runs on:
//
//     D[M, N] = A[M, K] * B[N, K]^T        bf16 operands, fp32 accumulation in TMEM
//
// with K split into two segments (segment 1 is optional), each with its own operand sources:
//   A: TMA, K-major or MN-major                    (activations, LoRA weights)
//      NF4, K-major or MN-major: packed codes arrive by TMA, eight dequant warps rebuild the bf16
//      tile in registers (bit-exact with qb_nf4_dequant) and write it to shared memory in the
//      swizzled layout the MMA reads — no bf16 weight ever reaches HBM
//   B: TMA, K-major or MN-major
// Segment 1 carries the LoRA term of a projection as extra K: Y = [W | s*B_lora] * [X | U]^T.
//
// Roles (one CTA per SM, persistent over output tiles of 128 x BN, m-blocks fastest so the
// CTAs of a wave share the same B tile in L2):
//   warp 0      TMA producer (one thread)        -> full[s]
//   warp 1      TMEM allocator + MMA issuer      full[s] (+ afull[s]) -> MMAs -> empty[s], tfull[b]
//   warps 2-5   epilogue: TMEM -> registers -> the epilogue functor; tempty[b]
//   warps 6-13  NF4 dequant (only when an A source is NF4): full[s] -> A tile -> afull[s]
// Accumulators are double-buffered in TMEM (2 x BN columns), so the epilogue of one tile runs
// under the MMAs of the next. Every wait is bounded (tc::mbar_wait): a wait that gives up
// raises the device error flag and every role drains out; TMEM is always released.
#pragma once

#include "qb_common.cuh"
#include "tc_common.cuh"

namespace tcg {

enum Src : int { kTmaK = 0, kTmaMN = 1, kNf4K = 2, kNf4MN = 3 };

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kEpiWarp0 = 2;
constexpr int kDeqWarp0 = 6;
constexpr int kDeqThreads = 256;  // 8 dequant warps: two per scheduler

struct Nf4Operand {
  const uint8_t* absmax_q;  // uint8 codes of the block scales [rows * blocks_per_row]
  const float* absmax2;     // second-level scales
  const float* code2;       // [256]
  const float* lut;         // NF4 code book [16]
  float offset;
  int blocksize2;
  int blocks_per_row;       // in_features / 64
  int rows;                 // out_features
  int cols;                 // in_features
};

struct Problem {
  int M, N;
  int nk0, nk1;   // k-blocks of 64 in segment 0 / segment 1
  int num_m, num_n;
};

template <int BN, bool NF4>
struct Cfg {
  static constexpr int A_BYTES = BM * 128;
  static constexpr int B_BYTES = BN * 128;
  static constexpr int C_BYTES = NF4 ? 4096 : 0;
  static constexpr int STAGE = A_BYTES + B_BYTES + C_BYTES;
  static constexpr int STAGES = (NF4 ? 208 : 196) * 1024 / STAGE;
  static constexpr int THREADS = NF4 ? 192 + kDeqThreads : 192;
  static constexpr int TMEM_COLS = 2 * BN <= 32 ? 32 : (2 * BN <= 64 ? 64 : (2 * BN <= 128 ? 128 : (2 * BN <= 256 ? 256 : 512)));
  static constexpr int EXTRA = 1024 /*align*/ + 512 /*barriers*/ + (NF4 ? (256 + 16) * 4 : 0);
  static constexpr int SMEM = STAGES * STAGE + EXTRA;
};

constexpr bool is_nf4(int s) { return s == kNf4K || s == kNf4MN; }
constexpr bool is_mn(int s) { return s == kTmaMN || s == kNf4MN; }

// One dequant thread rebuilds 32 consecutive weights (16 packed bytes, all in one scale block)
// as four 16-byte chunks of a 128-byte swizzled smem row: chunk c lands at chunk position
// c ^ swz. Byte j of the codes holds weights 2j (high nibble) and 2j+1 (low nibble).
//
// Per code byte: both nibble indices come pre-multiplied by 4 (one shift + mask per 4 bytes,
// one byte permute per index), the two table values are multiplied by the scale in one packed
// f32x2 multiply (two IEEE round-to-nearest products, as two scalar multiplies would give) and
// rounded to bf16 in one cvt.
__device__ __forceinline__ uint32_t nf4_pair(const float* lut, uint32_t hi4, uint32_t lo4, int b,
                                             uint64_t scale2) {
  const uint32_t ih = __byte_perm(hi4, 0u, 0x4440u | b);
  const uint32_t il = __byte_perm(lo4, 0u, 0x4440u | b);
  const float vh = *reinterpret_cast<const float*>(reinterpret_cast<const uint8_t*>(lut) + ih);
  const float vl = *reinterpret_cast<const float*>(reinterpret_cast<const uint8_t*>(lut) + il);
  uint64_t v, p;
  asm("mov.b64 %0, {%1, %2};" : "=l"(v) : "f"(vh), "f"(vl));
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(p) : "l"(v), "l"(scale2));
  float ph, pl;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(ph), "=f"(pl) : "l"(p));
  __nv_bfloat162 r = __floats2bfloat162_rn(ph, pl);   // weight 2j (high nibble) in the low half
  return *reinterpret_cast<uint32_t*>(&r);
}

__device__ __forceinline__ void dequant32(const uint8_t* codes, float scale, const float* lut,
                                          uint8_t* row, int c0, int swz) {
  const uint4 cw = *reinterpret_cast<const uint4*>(codes);
  const uint32_t w[4] = {cw.x, cw.y, cw.z, cw.w};
  uint64_t scale2;
  asm("mov.b64 %0, {%1, %1};" : "=l"(scale2) : "f"(scale));
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t x = w[j];
    const uint32_t hi4 = (x >> 2) & 0x3C3C3C3Cu;   // byte b: 4 * high nibble
    const uint32_t lo4 = (x << 2) & 0x3C3C3C3Cu;   // byte b: 4 * low nibble
    uint32_t o[4];
#pragma unroll
    for (int b = 0; b < 4; ++b) o[b] = nf4_pair(lut, hi4, lo4, b, scale2);
    *reinterpret_cast<uint4*>(row + (((c0 + j) ^ swz) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// The raw ingredients of one block scale (code of the first-level absmax, second-level scale),
// loaded a couple of k-steps before they are needed; code < 0 marks an out-of-range block.
struct ScaleRaw {
  int code;
  float a2;
};

__device__ __forceinline__ ScaleRaw scale_raw(const Nf4Operand& q, int row, int blk_in_row) {
  if (row >= q.rows || blk_in_row >= q.blocks_per_row) return ScaleRaw{-1, 0.f};
  const int64_t blk = static_cast<int64_t>(row) * q.blocks_per_row + blk_in_row;
  return ScaleRaw{static_cast<int>(__ldg(q.absmax_q + blk)), __ldg(q.absmax2 + blk / q.blocksize2)};
}

// scale = code2[code] * absmax2 + offset: a rounded multiply, then a rounded add (no FMA).
__device__ __forceinline__ float scale_of(const ScaleRaw& r, const float* s_code2, float offset) {
  return r.code < 0 ? 0.f : __fadd_rn(__fmul_rn(s_code2[r.code], r.a2), offset);
}

template <int A0, int B0, int A1, int B1, int BN, class Epi>
__global__ void __launch_bounds__(Cfg<BN, is_nf4(A0) || is_nf4(A1)>::THREADS, 1)
tc_gemm_kernel(const __grid_constant__ CUtensorMap mA0, const __grid_constant__ CUtensorMap mB0,
               const __grid_constant__ CUtensorMap mA1, const __grid_constant__ CUtensorMap mB1,
               const Problem pb, const Nf4Operand nf4, Epi epi, int* err) {
  constexpr bool kNF4 = is_nf4(A0) || is_nf4(A1);
  using C = Cfg<BN, kNF4>;
  constexpr int STAGES = C::STAGES;
  constexpr uint32_t kIdesc0 = tc::idesc_bf16(BM, BN, is_mn(A0), is_mn(B0));
  constexpr uint32_t kIdesc1 = tc::idesc_bf16(BM, BN, is_mn(A1), is_mn(B1));

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * C::STAGE);
  uint64_t* empty = full + STAGES;
  uint64_t* afull = empty + STAGES;
  uint64_t* tfull = afull + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  float* s_code2 = reinterpret_cast<float*>(smem + STAGES * C::STAGE + 512);
  float* s_lut = s_code2 + 256;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
      tc::mbar_init(&afull[s], kDeqThreads);
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(&tfull[b], 1);
      tc::mbar_init(&tempty[b], 128);
    }
    tc::mbar_init(drain, 1);
    tc::fence_mbar_init();
  }
  if (kNF4) {
    if (threadIdx.x < 256) s_code2[threadIdx.x] = nf4.code2[threadIdx.x];
    if (threadIdx.x < 16) s_lut[threadIdx.x] = nf4.lut[threadIdx.x];
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, C::TMEM_COLS);
    tc::tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tc::prefetch_tmap(&mA0);
    tc::prefetch_tmap(&mB0);
    if (pb.nk1 > 0) {
      tc::prefetch_tmap(&mA1);
      tc::prefetch_tmap(&mB1);
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;

  const int num_tiles = pb.num_m * pb.num_n;
  const int nk = pb.nk0 + pb.nk1;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      long issued = 0;
      for (int tile = blockIdx.x; tile < num_tiles && !tc::failed(err); tile += gridDim.x) {
        const int m0 = (tile % pb.num_m) * BM, n0 = (tile / pb.num_m) * BN;
        for (int kb = 0; kb < nk; ++kb) {
          if (!tc::mbar_wait(&empty[stage], phase ^ 1, err, 1)) break;
          uint8_t* sA = smem + stage * C::STAGE;
          uint8_t* sB = sA + C::A_BYTES;
          uint8_t* sC = sB + C::B_BYTES;
          const bool seg1 = kb >= pb.nk0;
          const int k = seg1 ? kb - pb.nk0 : kb;
          const int asrc = seg1 ? A1 : A0, bsrc = seg1 ? B1 : B0;
          const CUtensorMap* ma = seg1 ? &mA1 : &mA0;
          const CUtensorMap* mb = seg1 ? &mB1 : &mB0;
          tc::mbar_expect_tx(&full[stage], (is_nf4(asrc) ? C::C_BYTES : C::A_BYTES) + C::B_BYTES);
          if (asrc == kTmaK) {
            tc::tma_load_2d(sA, ma, &full[stage], k * BK, m0);
          } else if (asrc == kTmaMN) {
            tc::tma_load_2d(sA, ma, &full[stage], m0, k * BK);
            tc::tma_load_2d(sA + 8192, ma, &full[stage], m0 + 64, k * BK);
          } else if (asrc == kNf4K) {
            tc::tma_load_2d(sC, ma, &full[stage], k * 32, m0);         // 128 rows x 32 bytes
          } else {
            tc::tma_load_2d(sC, ma, &full[stage], m0 / 2, k * BK);     // 64 rows x 64 bytes
          }
          if (bsrc == kTmaK) {
            tc::tma_load_2d(sB, mb, &full[stage], k * BK, n0);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tc::tma_load_2d(sB + j * 8192, mb, &full[stage], n0 + j * 64, k * BK);
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
          ++issued;
        }
      }
      if (tc::failed(err)) {   // let this CTA's copies in flight land before it exits
        for (int i = 0; i < STAGES && i < issued; ++i) {
          if (--stage < 0) { stage = STAGES - 1; phase ^= 1; }
          tc::mbar_wait_quiet(&full[stage], phase);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int t = 0;
      for (int tile = blockIdx.x; tile < num_tiles && !tc::failed(err); tile += gridDim.x, ++t) {
        const int buf = t & 1;
        if (!tc::mbar_wait(&tempty[buf], ((t >> 1) & 1) ^ 1, err, 2)) break;
        tc::fence_after_sync();
        const uint32_t d = tmem_base + buf * BN;
        bool ok = true;
        for (int kb = 0; kb < nk; ++kb) {
          const bool seg1 = kb >= pb.nk0;
          const int asrc = seg1 ? A1 : A0, bsrc = seg1 ? B1 : B0;
          if (!tc::mbar_wait(&full[stage], phase, err, 3)) { ok = false; break; }
          if (kNF4 && !tc::mbar_wait(&afull[stage], phase, err, 4)) { ok = false; break; }
          tc::fence_after_sync();
          const uint32_t sA = tc::smem_u32(smem + stage * C::STAGE);
          const uint32_t sB = sA + C::A_BYTES;
          const uint32_t idesc = seg1 ? kIdesc1 : kIdesc0;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t a = is_mn(asrc) ? tc::sdesc_sw128(sA + kk * 2048, 8192, 1024)
                                           : tc::sdesc_sw128(sA + kk * 32, 16, 1024);
            const uint64_t b = is_mn(bsrc) ? tc::sdesc_sw128(sB + kk * 2048, 8192, 1024)
                                           : tc::sdesc_sw128(sB + kk * 32, 16, 1024);
            tc::mma_bf16(d, a, b, idesc, (kb | kk) != 0);
          }
          tc::mma_commit(&empty[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        tc::mma_commit(&tfull[buf]);
      }
      // every MMA this thread issued has completed before TMEM is released
      tc::mma_commit(drain);
      tc::mbar_wait_quiet(drain, 0);
    }
  } else if (warp < kDeqWarp0) {
    // ---------------------------------------------------------------- epilogue
    const int quarter = warp & 3;  // TMEM lanes this warp may read
    const int row = quarter * 32 + lane;
    int t = 0;
    // the loop condition and the break are warp-uniform: tcgen05.ld below is warp-collective
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++t) {
      const int buf = t & 1;
      const bool ready = tc::mbar_wait(&tfull[buf], (t >> 1) & 1, err, 5);
      if (!__all_sync(0xffffffffu, ready)) break;
      tc::fence_after_sync();
      const int m0 = (tile % pb.num_m) * BM, n0 = (tile / pb.num_m) * BN;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + buf * BN;
      epi.template tile<BN>(m0, n0, row, taddr);
      tc::fence_before_sync();
      tc::mbar_arrive(&tempty[buf]);
    }
  } else if (kNF4) {
    // ---------------------------------------------------------------- NF4 dequant
    // 256 threads, 32 weights each per k-block. These warps step through every k-block
    // (arriving on afull for TMA-fed blocks too), so afull's phases stay in lock step with
    // full's. Scale ingredients are loaded two k-blocks ahead of their use.
    const int d = threadIdx.x - kDeqWarp0 * 32;  // 0..255
    // K-major (A row = weight row): thread -> (row, half of the 64 k)
    const int kr_row = d >> 1, k_half = d & 1;
    // MN-major (A = W^T, k rows are weight rows): thread -> (k row, quarter of the 128 m)
    const int mn_kr = d >> 2, mn_q = d & 3;
    int off_codes, off_row, c0, swz;
    if (A0 == kNf4K || A1 == kNf4K) {
      off_codes = kr_row * 32 + k_half * 16;
      off_row = kr_row * 128;
      c0 = k_half * 4;
      swz = kr_row & 7;
    } else {
      off_codes = mn_kr * 64 + mn_q * 16;
      off_row = (mn_q >> 1) * 8192 + mn_kr * 128;
      c0 = (mn_q & 1) * 4;
      swz = mn_kr & 7;
    }
    auto raw_for = [&](int m0, int kb) -> ScaleRaw {
      if (kb >= pb.nk0) return ScaleRaw{-1, 0.f};   // segment 1 is TMA-fed
      if (A0 == kNf4K) return scale_raw(nf4, m0 + kr_row, kb);
      return scale_raw(nf4, kb * BK + mn_kr, (m0 >> 6) + (mn_q >> 1));
    };
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < num_tiles && ok && !tc::failed(err); tile += gridDim.x) {
      const int m0 = (tile % pb.num_m) * BM;
      ScaleRaw r0 = raw_for(m0, 0), r1 = raw_for(m0, 1);
      for (int kb = 0; kb < nk; ++kb) {
        const bool seg1 = kb >= pb.nk0;
        const int asrc = seg1 ? A1 : A0;
        const ScaleRaw cur = r0;
        r0 = r1;
        r1 = raw_for(m0, kb + 2);
        if (!tc::mbar_wait(&full[stage], phase, err, 6)) { ok = false; break; }
        if (is_nf4(asrc)) {
          uint8_t* sA = smem + stage * C::STAGE;
          const uint8_t* sC = sA + C::A_BYTES + C::B_BYTES;
          dequant32(sC + off_codes, scale_of(cur, s_code2, nf4.offset), s_lut, sA + off_row, c0,
                    swz);
          tc::fence_proxy_async_smem();
        }
        tc::mbar_arrive(&afull[stage]);
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
    }
  }

  // ------------------------------------------------------------------ teardown
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// Host: one launch of the kernel above on a persistent grid.
template <int A0, int B0, int A1, int B1, int BN, class Epi>
int launch(const CUtensorMap& mA0, const CUtensorMap& mB0, const CUtensorMap& mA1,
           const CUtensorMap& mB1, const Problem& pb, const Nf4Operand& nf4, const Epi& epi,
           cudaStream_t stream, const char* what) {
  constexpr bool kNF4 = is_nf4(A0) || is_nf4(A1);
  using C = Cfg<BN, kNF4>;
  auto kernel = tc_gemm_kernel<A0, B0, A1, B1, BN, Epi>;
  static bool configured[64] = {};  // per instantiation and device
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return qb::fail(QB_ERR_UNSUPPORTED, "%s: device %d", what, dev);
  if (!configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return qb::fail(QB_ERR_CUDA, "%s: smem attribute: %s", what, cudaGetErrorString(e));
    configured[dev] = true;
  }
  int* err = tc_host::device_error_flag();
  if (!err) return qb::fail(QB_ERR_CUDA, "%s: no device error flag", what);
  const int tiles = pb.num_m * pb.num_n;
  if (tiles == 0) return QB_OK;
  int grid = tc_host::sm_count();
  if (grid > tiles) grid = tiles;
  kernel<<<grid, C::THREADS, C::SMEM, stream>>>(mA0, mB0, mA1, mB1, pb, nf4, epi, err);
  return qb::check_launch(what);
}

}  // namespace tcg
