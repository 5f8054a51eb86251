// The persistent, warp-specialised tcgen05 GEMM every TMA-fed dense contraction of the suite
// runs on:
//
//     D[M, N] = A0[M, K0] * B0[N, K0]^T  +  A1[M, K1] * B1[N, K1]^T     bf16, fp32 in TMEM
//
// Segment 1 is optional (K1 = 0); it carries the LoRA term of a projection as extra K
// (Y = [X | U] [W | s*B_lora]^T). Every operand comes in by TMA, K-major or MN-major in HBM.
//
// Roles (one CTA per SM, persistent over output tiles of 128 x BN):
//   warp 0      TMA producer (one thread)        -> full[s]
//   warp 1      TMEM allocator + MMA issuer      full[s] -> MMAs -> empty[s], tfull[b]
//   warps 2-5   epilogue: TMEM -> registers -> the epilogue functor; tempty[b]
// Accumulators are double-buffered in TMEM (2 x BN columns), so the epilogue of one tile runs
// under the MMAs of the next. Tiles are visited in groups of kGroupM m-blocks (m fastest inside
// a group), so the CTAs of one wave touch a ~16 x 9 block of tiles and both operands of the
// wave stay in L2 whichever of them is the long one. Every wait is bounded (tc::mbar_wait): a
// wait that gives up raises the device error flag and every role drains out; TMEM is always
// released.
#pragma once

#include "qb_common.cuh"
#include "tc_common.cuh"
#include "philox.cuh"

#include <type_traits>

namespace tcg {

// B sources: K-major or MN-major by TMA; kTmaKDual = K-major whose BN-row tile is two BN/2-row
// halves from two tensors at the same row (the "top" map and the segment's second map): the
// output tile's first BN/2 columns come from one weight, the last BN/2 from the other (a gate /
// up pair computed by one GEMM).
enum Src : int { kTmaK = 0, kTmaMN = 1, kTmaKDual = 2 };

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kGroupM = 16;
constexpr int kThreads = 192;

struct Problem {
  int M, N;
  int nk0, nk1;   // k-blocks of 64 in segment 0 / segment 1
  int num_m, num_n;
  int splits;     // split-K: each tile's k-blocks in this many consecutive ranges (0 or 1: none)
};

// Work item `item` of a launch -> (tile, first k-block, end k-block): with split-K the items are
// the tiles times the splits, split fastest, each a contiguous range of the tile's k-blocks (the
// epilogue then stores its partial product, `split` x the padded M rows down).
__device__ __forceinline__ void item_range(const Problem& pb, int item, int& tile, int& kb0,
                                           int& kb1) {
  const int splits = pb.splits > 1 ? pb.splits : 1;
  const int nk = pb.nk0 + pb.nk1;
  tile = item / splits;
  const int sp = item - tile * splits;
  kb0 = static_cast<int>(static_cast<int64_t>(nk) * sp / splits);
  kb1 = static_cast<int>(static_cast<int64_t>(nk) * (sp + 1) / splits);
}

// Output tile `tile` -> (m-block, n-block) in the grouped order described above.
__device__ __forceinline__ void tile_blocks(const Problem& pb, int tile, int& mb, int& nb) {
  const int per_group = kGroupM * pb.num_n;
  const int g = tile / per_group, r = tile - g * per_group;
  const int gm0 = g * kGroupM;
  const int gm = min(kGroupM, pb.num_m - gm0);
  mb = gm0 + r % gm;
  nb = r / gm;
}

template <int BN>
struct Cfg {
  static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "UMMA N for M=128, whole TMEM chunks");
  static constexpr int A_BYTES = BM * 128;
  static constexpr int B_BYTES_K = BN * 128;                // K-major B: BN rows of 128 bytes
  static constexpr int B_BYTES_MN = ((BN + 63) / 64) * 8192; // MN-major B: whole 64-wide boxes
  static constexpr int B_BYTES = B_BYTES_MN > B_BYTES_K ? B_BYTES_MN : B_BYTES_K;  // stage slot
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int STAGES = 196 * 1024 / STAGE;
  static constexpr int TMEM_COLS = 2 * BN <= 32 ? 32 : (2 * BN <= 64 ? 64 : (2 * BN <= 128 ? 128 : (2 * BN <= 256 ? 256 : 512)));
  static constexpr int BUF_COLS = TMEM_COLS / 2;   // accumulator b starts at column b * BUF_COLS
  static constexpr int EXTRA = 1024 /*align*/ + 512 /*barriers*/;
  static constexpr int SMEM = STAGES * STAGE + EXTRA;
};

constexpr bool is_mn(int s) { return s == kTmaMN; }

// Epilogues that store through shared memory declare kStageBytes: the bytes each of the four
// epilogue warps gets for staging its 32 rows of the output before a TMA store. Others get none.
template <class E, class = void>
struct EpiStage {
  static constexpr int bytes = 0;
};
template <class E>
struct EpiStage<E, std::void_t<decltype(E::kStageBytes)>> {
  static constexpr int bytes = E::kStageBytes;
};

// Row `lane` of a [32 x 32] bf16 staging box (64-byte rows) from 32 floats, in the 64-byte swizzle
// of the box's tensor map: 16-byte piece p of row r sits at r * 64 + ((p ^ ((r >> 1) & 3)) * 16),
// so the 32 lanes' writes of one piece cover every bank once per 128 bytes.
__device__ __forceinline__ void stage_row_bf16(uint8_t* box, int lane, const float* v) {
  uint8_t* dst = box + lane * 64;
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    qb::Vec16<__nv_bfloat16> w;
#pragma unroll
    for (int i = 0; i < 8; ++i) w.v[i] = __float2bfloat16_rn(v[8 * p + i]);
    *reinterpret_cast<uint4*>(dst + ((p ^ ((lane >> 1) & 3)) << 4)) = w.u;
  }
}

// Ring stages of Cfg<BN> that fit beside `epi_bytes` of epilogue staging in the 227 KB a CTA
// may have.
template <int BN>
constexpr int stages_with(int epi_bytes) {
  using C = Cfg<BN>;
  return (232448 - C::EXTRA - epi_bytes) / C::STAGE < C::STAGES
             ? (232448 - C::EXTRA - epi_bytes) / C::STAGE
             : C::STAGES;
}

// Side work for warps past the GEMM's six: dropout-mask words (the Philox stream of philox.cuh)
// drawn on the integer pipes while the tensor cores run the product. The jobs' words form one
// index space (job j owns [first, first + rows * words)); the side warps stride over it with the
// whole grid and never wait on the GEMM's barriers, so they only meet the other warps at the
// block's entry and exit.
struct MaskJob {
  uint32_t* bits;       // [rows, words]: bit (c & 31) of word c / 32 keeps column c
  int64_t rows, cols, words;
  uint32_t k0, k1;      // the seed's low and high words
  int32_t thresh;       // keep when the folded Philox word is above this (qb::keep_threshold)
  int64_t first;
};
constexpr int kMaxMaskJobs = 8;
struct SideWork {
  int njobs;
  int64_t total;
  MaskJob job[kMaxMaskJobs];
};
struct NoSide {};
template <int SIDE>
using SideArg = typename std::conditional<SIDE == 0, NoSide, SideWork>::type;

template <int SIDE>
__device__ __forceinline__ void side_masks(const SideArg<SIDE>& side, int side_thread) {
  if constexpr (SIDE > 0) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * (SIDE * 32);
    for (int64_t t = static_cast<int64_t>(blockIdx.x) * (SIDE * 32) + side_thread; t < side.total;
         t += stride) {
      int j = 0;
      while (j + 1 < side.njobs && t >= side.job[j + 1].first) ++j;
      const MaskJob& jb = side.job[j];
      const int64_t local = t - jb.first;
      const int64_t row = local / jb.words, w = local - row * jb.words;
      const int64_t c0 = w * 32;
      const int n = jb.cols - c0 < 32 ? static_cast<int>(jb.cols - c0) : 32;
      jb.bits[local] = qb::mask_word(row, jb.cols, c0, n, jb.k0, jb.k1, jb.thresh);
    }
  }
}

template <int A0, int B0, int A1, int B1, int BN, class Epi, int SIDE = 0>
__global__ void __launch_bounds__(kThreads + 32 * SIDE, 1)
tc_gemm_kernel(const __grid_constant__ CUtensorMap mA0, const __grid_constant__ CUtensorMap mB0,
               const __grid_constant__ CUtensorMap mA1, const __grid_constant__ CUtensorMap mB1,
               const __grid_constant__ CUtensorMap mB0b, const __grid_constant__ CUtensorMap mB1b,
               const Problem pb, const __grid_constant__ Epi epi, const tc::Ctl ctl,
               const __grid_constant__ SideArg<SIDE> side) {
  using C = Cfg<BN>;
  int* err = ctl.err;
  tc::trace_begin(ctl);
  constexpr int kEpiWarpBytes = EpiStage<Epi>::bytes;
  constexpr int kEpiBytes = 4 * kEpiWarpBytes;
  constexpr int STAGES = stages_with<BN>(kEpiBytes);
  static_assert(STAGES >= 2, "at least two ring stages");
  constexpr uint32_t kIdesc0 = tc::idesc_bf16(BM, BN, is_mn(A0), is_mn(B0));
  constexpr uint32_t kIdesc1 = tc::idesc_bf16(BM, BN, is_mn(A1), is_mn(B1));

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* epi_stage = smem + STAGES * C::STAGE;   // 1024-aligned: STAGE is a multiple of 1024
  uint64_t* full = reinterpret_cast<uint64_t*>(epi_stage + kEpiBytes);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(&tfull[b], 1);
      tc::mbar_init(&tempty[b], 128);
    }
    tc::mbar_init(drain, 1);
    tc::fence_mbar_init();
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

  const int num_items = pb.num_m * pb.num_n * (pb.splits > 1 ? pb.splits : 1);

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      long issued = 0;
      for (int item = blockIdx.x; item < num_items && !tc::failed(err); item += gridDim.x) {
        int tile, kb0, kb1, mb, nb;
        item_range(pb, item, tile, kb0, kb1);
        tile_blocks(pb, tile, mb, nb);
        const int m0 = mb * BM, n0 = nb * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!tc::mbar_wait(&empty[stage], phase ^ 1, err, 1)) break;
          uint8_t* sA = smem + stage * C::STAGE;
          uint8_t* sB = sA + C::A_BYTES;
          const bool seg1 = kb >= pb.nk0;
          const int k = seg1 ? kb - pb.nk0 : kb;
          const int asrc = seg1 ? A1 : A0, bsrc = seg1 ? B1 : B0;
          const CUtensorMap* ma = seg1 ? &mA1 : &mA0;
          const CUtensorMap* mb_ = seg1 ? &mB1 : &mB0;
          tc::mbar_expect_tx(&full[stage], C::A_BYTES + (bsrc == kTmaMN ? C::B_BYTES_MN : C::B_BYTES_K));
          if (asrc == kTmaK) {
            tc::tma_load_2d(sA, ma, &full[stage], k * BK, m0);
          } else {
            tc::tma_load_2d(sA, ma, &full[stage], m0, k * BK);
            tc::tma_load_2d(sA + 8192, ma, &full[stage], m0 + 64, k * BK);
          }
          if (bsrc == kTmaK) {
            tc::tma_load_2d(sB, mb_, &full[stage], k * BK, n0);
          } else if (bsrc == kTmaKDual) {
            tc::tma_load_2d(sB, mb_, &full[stage], k * BK, n0 / 2);
            tc::tma_load_2d(sB + (BN / 2) * 128, seg1 ? &mB1b : &mB0b, &full[stage], k * BK,
                            n0 / 2);
          } else {
#pragma unroll   // a partial last box (BN = 224) brings columns the MMA does not read
            for (int j = 0; j < (BN + 63) / 64; ++j)
              tc::tma_load_2d(sB + j * 8192, mb_, &full[stage], n0 + j * 64, k * BK);
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
      for (int item = blockIdx.x; item < num_items && !tc::failed(err); item += gridDim.x, ++t) {
        int tile, kb0, kb1;
        item_range(pb, item, tile, kb0, kb1);
        const int buf = t & 1;
        if (!tc::mbar_wait(&tempty[buf], ((t >> 1) & 1) ^ 1, err, 2)) break;
        tc::fence_after_sync();
        const uint32_t d = tmem_base + buf * C::BUF_COLS;
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb) {
          const bool seg1 = kb >= pb.nk0;
          const int asrc = seg1 ? A1 : A0, bsrc = seg1 ? B1 : B0;
          if (!tc::mbar_wait(&full[stage], phase, err, 3)) { ok = false; break; }
          // TMA -> MMA is ordered by the barrier's transaction count: no tcgen05 fence here
          const uint32_t sA = tc::smem_u32(smem + stage * C::STAGE);
          const uint32_t sB = sA + C::A_BYTES;
          const uint32_t idesc = seg1 ? kIdesc1 : kIdesc0;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t a = is_mn(asrc) ? tc::sdesc_sw128(sA + kk * 2048, 8192, 1024)
                                           : tc::sdesc_sw128(sA + kk * 32, 16, 1024);
            const uint64_t b = is_mn(bsrc) ? tc::sdesc_sw128(sB + kk * 2048, 8192, 1024)
                                           : tc::sdesc_sw128(sB + kk * 32, 16, 1024);
            tc::mma_bf16(d, a, b, idesc, (kb != kb0 || kk != 0) ? 1u : 0u);
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
  } else if (warp < kThreads / 32) {
    // ---------------------------------------------------------------- epilogue
    const int quarter = warp & 3;  // TMEM lanes this warp may read
    const int row = quarter * 32 + lane;
    int t = 0;
    // the loop condition and the break are warp-uniform: tcgen05.ld below is warp-collective
    for (int item = blockIdx.x; item < num_items; item += gridDim.x, ++t) {
      int tile, kb0, kb1;
      item_range(pb, item, tile, kb0, kb1);
      const int buf = t & 1;
      const bool ready = tc::mbar_wait(&tfull[buf], (t >> 1) & 1, err, 5);
      if (!__all_sync(0xffffffffu, ready)) break;
      tc::fence_after_sync();
      int mb, nb;
      tile_blocks(pb, tile, mb, nb);
      const uint32_t taddr =
          tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + buf * C::BUF_COLS;
      // with split-K, split sp's partial tile lands sp x (padded M) rows further down: the
      // epilogue of a split launch writes partial products that a reduction sums in split order
      const int m_off = (item - tile * (pb.splits > 1 ? pb.splits : 1)) * pb.num_m * BM;
      if constexpr (kEpiWarpBytes > 0)
        epi.template tile<BN>(mb * BM + m_off, nb * BN, row, taddr,
                              epi_stage + (warp - 2) * kEpiWarpBytes);
      else
        epi.template tile<BN>(mb * BM + m_off, nb * BN, row, taddr);
      tc::fence_before_sync();
      tc::mbar_arrive(&tempty[buf]);
    }
    if constexpr (kEpiWarpBytes > 0) {   // this warp's TMA stores are complete before exit
      if (lane == 0) tc::bulk_wait_all();
      __syncwarp();
    }
  } else {
    // ---------------------------------------------------------------- side warps
    side_masks<SIDE>(side, threadIdx.x - kThreads);
  }

  // ------------------------------------------------------------------ teardown
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem_base, C::TMEM_COLS);
    if (lane == 0) tc::trace_end(ctl);
  }
}

// Host: one launch of the kernel above on a persistent grid.
template <int A0, int B0, int A1, int B1, int BN, class Epi, int SIDE = 0>
int launch(const CUtensorMap& mA0, const CUtensorMap& mB0, const CUtensorMap& mA1,
           const CUtensorMap& mB1, const Problem& pb, const Epi& epi, cudaStream_t stream,
           const char* what, const CUtensorMap* mB0b = nullptr,
           const CUtensorMap* mB1b = nullptr, const SideArg<SIDE>& side = SideArg<SIDE>{}) {
  static_assert(B0 != kTmaKDual || BN % 2 == 0, "dual B splits the tile in halves");
  using C = Cfg<BN>;
  auto kernel = tc_gemm_kernel<A0, B0, A1, B1, BN, Epi, SIDE>;
  constexpr int kEpiBytes = 4 * EpiStage<Epi>::bytes;
  constexpr int kSmem = stages_with<BN>(kEpiBytes) * C::STAGE + kEpiBytes + C::EXTRA;
  static_assert(kSmem <= 232448, "shared memory of one CTA");
  if (int s = tc_host::ensure_smem(reinterpret_cast<const void*>(kernel), kSmem, what)) return s;
  const int tiles = pb.num_m * pb.num_n * (pb.splits > 1 ? pb.splits : 1);
  if (tiles == 0) return QB_OK;
  if (pb.splits > pb.nk0 + pb.nk1)
    return qb::fail(QB_ERR_INVALID, "%s: more k-splits (%d) than k-blocks", what, pb.splits);
  int grid = tc_host::sm_count();
  if (grid > tiles) grid = tiles;
  if ((B0 == kTmaKDual && !mB0b) || (B1 == kTmaKDual && !mB1b))
    return qb::fail(QB_ERR_INVALID, "%s: dual B needs its second tensor map", what);
  tc::Ctl ctl;
  if (int s = tc_host::launch_ctl(&ctl, what)) return s;
  kernel<<<grid, kThreads + 32 * SIDE, kSmem, stream>>>(mA0, mB0, mA1, mB1, mB0b ? *mB0b : mB0,
                                                         mB1b ? *mB1b : mB1, pb, epi, ctl, side);
  return qb::check_launch(what);
}

}  // namespace tcg
