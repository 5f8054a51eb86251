// The 2-SM variant of the TMA-fed tcgen05 GEMM (same contract as tc_gemm.cuh, A operands
// K-major):
//
//     D[M, N] = A0[M, K0] * B0[N, K0]^T  +  A1[M, K1] * B1[N, K1]^T     bf16, fp32 in TMEM
//
// CTA pairs (clusters of 2) compute 256 x 256 output tiles with tcgen05.mma.cta_group::2: each
// CTA loads 128 rows of A and 128 of the tile's 256 B rows (columns, for MN-major B) into the
// same shared-memory offsets, and the even CTA (the leader) issues M=256, N=256 MMAs that read
// both CTAs' halves and accumulate each CTA's 128 rows in its own TMEM. Per SM that halves the
// B bytes brought in and read by the tensor core per flop against the one-CTA 128 x 256 tile.
// A dual B source (the gate / up pair) is natural here: CTA 0 loads its half from the first
// weight and CTA 1 from the second, at the same rows.
//
// Roles per CTA (one CTA per SM, persistent over the pair's tiles):
//   warp 0      TMA producer of this CTA's halves; both CTAs' loads complete on the LEADER's
//               full[s], whose expected byte count the leader alone arms (for both CTAs)
//   warp 1      TMEM allocation (both CTAs); the leader's lane 0 issues the MMAs and commits each
//               stage's completion with one arrive on the same barrier in both CTAs (empty[s],
//               tfull[b])
//   warps 2-5   epilogue of this CTA's 128 rows; arrive on the leader's tempty[b]
// Per k-block there is no signal from one CTA's threads to the other's: an earlier version in
// which the other CTA armed its own bytes on the leader's barrier and the leader committed to each
// CTA separately ran at half this throughput (0.72 against 1.47-1.50 PFLOP/s).
// 6 stages of 32 KiB, accumulators double-buffered (2 x 256 TMEM columns). Every wait is bounded;
// a wait that gives up raises the device error flag and every role drains out (the two producers
// first agree on what each issued, so that every copy in flight completes on an armed phase and
// is waited for), and the two CTAs meet on a bounded mbarrier handshake before TMEM is released.
// No load multicasts.
#pragma once

#include "tc_gemm.cuh"

namespace tcp {

using tcg::BK;
using tcg::kTmaK;
using tcg::kTmaMN;
using tcg::Problem;   // num_m counts 256-row pair blocks here

constexpr int BMC = 128;              // rows per CTA
constexpr int BN = 256;               // columns per pair tile
constexpr int kHalfN = BN / 2;        // B rows (or columns) each CTA loads
constexpr int kA = BMC * 128;         // 16 KiB
constexpr int kB = kHalfN * 128;      // 16 KiB (K-major: 128 rows; MN-major: two 64-wide boxes)
constexpr int kStage = kA + kB;
constexpr int kStages = 6;
constexpr int kThreads = 192;
constexpr int kGroupM = 8;            // pair m-blocks per raster group (2048 rows, as tcg)
constexpr int kSmem = kStages * kStage + 1024 /*barriers*/ + 1024 /*align*/;

__device__ __forceinline__ void pair_tile_blocks(const Problem& pb, int tile, int& mb, int& nb) {
  const int per_group = kGroupM * pb.num_n;
  const int g = tile / per_group, r = tile - g * per_group;
  const int gm0 = g * kGroupM;
  const int gm = min(kGroupM, pb.num_m - gm0);
  mb = gm0 + r % gm;
  nb = r / gm;
}

template <int B0, int B1, class Epi>
__global__ void __launch_bounds__(kThreads, 1)
tc_gemm_pair_kernel(const __grid_constant__ CUtensorMap mA0, const __grid_constant__ CUtensorMap mB0,
                    const __grid_constant__ CUtensorMap mA1, const __grid_constant__ CUtensorMap mB1,
                    const __grid_constant__ CUtensorMap mB0b, const __grid_constant__ CUtensorMap mB1b,
                    const Problem pb, Epi epi, const tc::Ctl ctl) {
  int* err = ctl.err;
  tc::trace_begin(ctl);
  constexpr uint32_t kIdesc0 = tc::idesc_bf16(2 * BMC, BN, false, B0 == kTmaMN);
  constexpr uint32_t kIdesc1 = tc::idesc_bf16(2 * BMC, BN, false, B1 == kTmaMN);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStage);  // leader: both CTAs' bytes
  uint64_t* empty = full + kStages;     // each CTA: the stage's MMAs completed
  uint64_t* tfull = empty + kStages;    // each CTA: accumulator b ready
  uint64_t* tempty = tfull + 2;         // leader: both CTAs' epilogues drained accumulator b
  uint64_t* drain = tempty + 2;         // leader: every MMA completed (teardown)
  uint64_t* peer_done = drain + 1;      // each CTA: the other CTA has finished (teardown)
  uint64_t* stopped = peer_done + 1;    // each CTA: the other producer's issued count is here
  uint64_t* drained = stopped + 1;      // follower: the leader waited out both CTAs' copies
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drained + 1);
  uint32_t* peer_issued = tmem_slot + 1;  // written by the other CTA's producer (error path)

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = tc::cluster_rank();
  const bool leader = rank == 0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) { tc::mbar_init(&full[s], 1); tc::mbar_init(&empty[s], 1); }
    for (int b = 0; b < 2; ++b) { tc::mbar_init(&tfull[b], 1); tc::mbar_init(&tempty[b], 8); }
    tc::mbar_init(drain, 1);
    tc::mbar_init(peer_done, 1);
    tc::mbar_init(stopped, 1);
    tc::mbar_init(drained, 1);
    tc::fence_mbar_init();
  }
  if (warp == 1) {
    tc::tmem_alloc_pair(tmem_slot, 2 * BN);
    tc::tmem_relinquish_pair();
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
  tc::cluster_sync();   // both CTAs' barriers exist before either signals the other's
  tc::fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;
  const int num_tiles = pb.num_m * pb.num_n;
  const int nk = pb.nk0 + pb.nk1;
  const int cl = blockIdx.x >> 1, ncl = gridDim.x >> 1;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const uint32_t full_l = tc::mapa(full, 0);
      int s = 0;
      uint32_t ph = 0;
      long issued = 0;
      for (int tile = cl; tile < num_tiles && !tc::failed(err); tile += ncl) {
        int mb, nb;
        pair_tile_blocks(pb, tile, mb, nb);
        const int m0 = mb * 2 * BMC + static_cast<int>(rank) * BMC;
        const int nh = nb * BN + static_cast<int>(rank) * kHalfN;   // dual B: nb * kHalfN
        bool ok = true;
        for (int kb = 0; kb < nk; ++kb) {
          if (!tc::mbar_wait(&empty[s], ph ^ 1, err, 21)) { ok = false; break; }
          uint8_t* sA = smem + s * kStage;
          uint8_t* sB = sA + kA;
          const bool seg1 = kb >= pb.nk0;
          const int k = (seg1 ? kb - pb.nk0 : kb) * BK;
          const int bsrc = seg1 ? B1 : B0;
          const CUtensorMap* ma = seg1 ? &mA1 : &mA0;
          const CUtensorMap* mb_ = seg1 ? (bsrc == tcg::kTmaKDual && rank ? &mB1b : &mB1)
                                        : (bsrc == tcg::kTmaKDual && rank ? &mB0b : &mB0);
          const uint32_t bar = full_l + s * 8;
          if (leader) tc::mbar_expect_tx(&full[s], 2 * kStage);   // both CTAs' bytes
          tc::tma_load_2d_pair(sA, ma, bar, k, m0);
          if (bsrc == kTmaK) {
            tc::tma_load_2d_pair(sB, mb_, bar, k, nh);
          } else if (bsrc == tcg::kTmaKDual) {
            tc::tma_load_2d_pair(sB, mb_, bar, k, nb * kHalfN);
          } else {
            tc::tma_load_2d_pair(sB, mb_, bar, nh, k);
            tc::tma_load_2d_pair(sB + 8192, mb_, bar, nh + 64, k);
          }
          if (++s == kStages) { s = 0; ph ^= 1; }
          ++issued;
        }
        if (!ok) break;
      }
      if (tc::failed(err)) {
        // After a give-up the two producers may have stopped at different items (a wait that
        // finds its phase complete does not look at the flag), and all their copies complete on
        // the leader's full[] barriers. Each tells the other how many items it issued; the
        // leader then makes every phase either CTA started completable - arming the ones only
        // the follower issued (its bytes alone), counting as arrived the follower bytes of the
        // ones only the leader issued - and waits for the last phase of each stage, which
        // completes once every copy in flight has landed. The follower leaves only after that.
        const uint32_t peer = rank ^ 1u;
        tc::st_cluster_u32(tc::mapa(peer_issued, peer), static_cast<uint32_t>(issued));
        tc::mbar_arrive_cluster(tc::mapa(stopped, peer));
        const bool heard = tc::mbar_wait_cluster_quiet(stopped, 0);
        if (leader) {
          const long f = heard ? static_cast<long>(*reinterpret_cast<volatile uint32_t*>(peer_issued))
                               : issued;
          for (long i = issued; i < f; ++i)   // follower-only items: arm the follower's bytes
            tc::mbar_expect_tx(&full[i % kStages], kStage);
          for (long i = f; i < issued; ++i)   // leader-only items: the follower's bytes never come
            tc::mbar_complete_tx(&full[i % kStages], kStage);
          const long n = f > issued ? f : issued;
          for (long i = n - kStages < 0 ? 0 : n - kStages; i < n; ++i)
            tc::mbar_wait_quiet(&full[i % kStages], static_cast<uint32_t>((i / kStages) & 1));
          tc::mbar_arrive_cluster(tc::mapa(drained, 1));
        } else if (heard) {
          tc::mbar_wait_cluster_quiet(drained, 0);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer (leader)
    if (lane == 0 && leader) {
      auto both = [&](uint64_t* bar) { tc::mma_commit_pair_both(bar); };
      int s = 0;
      uint32_t ph = 0;
      int t = 0;
      for (int tile = cl; tile < num_tiles && !tc::failed(err); tile += ncl, ++t) {
        const int buf = t & 1;
        if (!tc::mbar_wait(&tempty[buf], ((t >> 1) & 1) ^ 1, err, 22)) break;
        tc::fence_after_sync();
        const uint32_t d = tmem_base + buf * BN;
        bool ok = true;
        for (int kb = 0; kb < nk; ++kb) {
          if (!tc::mbar_wait(&full[s], ph, err, 23)) { ok = false; break; }
          // TMA -> MMA is ordered by the barrier's transaction count: no tcgen05 fence here
          const bool seg1 = kb >= pb.nk0;
          const bool bmn = (seg1 ? B1 : B0) == kTmaMN;
          const uint32_t idesc = seg1 ? kIdesc1 : kIdesc0;
          const uint32_t sA = tc::smem_u32(smem + s * kStage);
          const uint32_t sB = sA + kA;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t a = tc::sdesc_sw128(sA + kk * 32, 16, 1024);
            const uint64_t b = bmn ? tc::sdesc_sw128(sB + kk * 2048, 8192, 1024)
                                   : tc::sdesc_sw128(sB + kk * 32, 16, 1024);
            tc::mma_bf16_pair(d, a, b, idesc, (kb | kk) != 0);
          }
          both(&empty[s]);
          if (++s == kStages) { s = 0; ph ^= 1; }
        }
        if (!ok) break;
        both(&tfull[buf]);
      }
      tc::mma_commit_pair_to(tc::mapa(drain, 0));
      tc::mbar_wait_quiet(drain, 0);
    }
  } else {
    // ------------------------------------------------------------------ epilogue (warps 2-5)
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t tempty_l = tc::mapa(tempty, 0);
    int t = 0;
    for (int tile = cl; tile < num_tiles; tile += ncl, ++t) {
      const int buf = t & 1;
      const bool ready = tc::mbar_wait(&tfull[buf], (t >> 1) & 1, err, 24);
      if (!__all_sync(0xffffffffu, ready)) break;   // warp-uniform: tcgen05.ld is collective
      tc::fence_after_sync();
      int mb, nb;
      pair_tile_blocks(pb, tile, mb, nb);
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + buf * BN;
      epi.template tile<BN>(mb * 2 * BMC + static_cast<int>(rank) * BMC, nb * BN, row, taddr);
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive_cluster(tempty_l + buf * 8);
    }
  }

  // Neither CTA leaves while the pair's MMAs or signals may touch it: each tells the other it is
  // done (its last access to the other's shared memory) and waits for the other's word, bounded
  // (a partner that never comes raises the flag instead of holding this SM for good).
  tc::fence_before_sync();
  __syncthreads();
  if (threadIdx.x == 0) {
    tc::mbar_arrive_cluster(tc::mapa(peer_done, rank ^ 1u));
    if (!tc::mbar_wait_cluster_quiet(peer_done, 0, tc::kWaitLimitNs)) tc::raise_error(err, 26);
  }
  __syncthreads();
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc_pair(tmem_base, 2 * BN);
    if (lane == 0) tc::trace_end(ctl);
  }
}

// Host: one launch on a persistent grid of CTA pairs.
template <int B0, int B1, class Epi>
int launch(const CUtensorMap& mA0, const CUtensorMap& mB0, const CUtensorMap& mA1,
           const CUtensorMap& mB1, const Problem& pb, const Epi& epi, cudaStream_t stream,
           const char* what, const CUtensorMap* mB0b = nullptr,
           const CUtensorMap* mB1b = nullptr) {
  if ((B0 == tcg::kTmaKDual && !mB0b) || (B1 == tcg::kTmaKDual && !mB1b))
    return qb::fail(QB_ERR_INVALID, "%s: dual B needs its second tensor map", what);
  auto kernel = tc_gemm_pair_kernel<B0, B1, Epi>;
  if (int s = tc_host::ensure_smem(reinterpret_cast<const void*>(kernel), kSmem, what)) return s;
  const int tiles = pb.num_m * pb.num_n;
  if (tiles == 0) return QB_OK;
  tc::Ctl ctl;
  if (int s = tc_host::launch_ctl(&ctl, what)) return s;
  int pairs = tc_host::sm_count() / 2;
  if (pairs > tiles) pairs = tiles;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, mA0, mB0, mA1, mB1, mB0b ? *mB0b : mB0,
                                     mB1b ? *mB1b : mB1, pb, epi, ctl);
  if (e != cudaSuccess) return qb::fail(QB_ERR_CUDA, "%s: launch: %s", what, cudaGetErrorString(e));
  return qb::check_launch(what);
}

}  // namespace tcp
