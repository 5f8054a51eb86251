// The input gradient of a dropped-out LoRA branch, added in place to the base projection's dx:
//
//     dx[M, N] (bf16) += scale * mask .* (V[M, K] B[N, K]^T)      V = dy (s B_lora), B = A_lora^T
//
// mask bit (n & 31) of bits[m * ldbits + n / 32] (the words qb_dropout_mask records). The rank-K
// product (K = the LoRA rank, one or two 64-wide k-blocks) is a handful of tcgen05 MMAs per
// 128 x 256 tile; the kernel's cost is moving dx, so dx goes through shared memory by TMA both
// ways: the producer loads each dx tile (four 128 x 64 slabs, 128-byte swizzle) into one of two
// buffers while the MMAs run; the epilogue warps (one TMEM lane per thread = one row) read the
// product from TMEM, apply mask and scale to the row in shared memory — with the swizzle, a warp's
// 16-byte row accesses hit 32 distinct banks per 8 lanes — and one thread TMA-stores the tile.
// Global traffic is dx read once and written once (coalesced by TMA) plus the mask words.
// Tiles are 128 x 128 (32 KiB of dx) in a ring of four buffers, so the producer keeps up to three
// tiles of loads in flight ahead of the epilogue; the storing thread does not wait for its own
// store: it hands a buffer back once the store issued after it has been read out.
//
// Roles (one CTA per SM, persistent over tiles): warp 0 TMA loads (operands, dx tiles),
// warp 1 TMEM allocation + MMA issue, warps 2-9 epilogue, two per TMEM lane quarter, each
// taking one 64-column slab of the rows (thread 64 also issues the stores).
// Hand-offs are mbarriers only, every wait bounded (tc::mbar_wait): a wait that gives up raises
// the device error flag, the roles drain their copies in flight and TMEM is released.
#include "qb_common.cuh"
#include "tc_common.cuh"

namespace {

constexpr int BM = 128, BN = 128, BK = 64;
constexpr int kStages = 2;
constexpr int kA = BM * 128;          // 16 KiB: V tile, 128 rows x 64 k
constexpr int kB = BN * 128;          // 16 KiB: B tile, 128 n x 64 k
constexpr int kSlab = BM * 128;       // 16 KiB: 128 rows x 64 columns of dx
constexpr int kSlabs = BN / 64;
constexpr int kC = kSlabs * kSlab;    // 32 KiB: one dx tile
constexpr int kCBufs = 4;             // dx tiles in the ring
constexpr int kEpiWarps = 8;          // two per TMEM lane quarter, each half of a row's columns
constexpr int kEpiThreads = 32 * kEpiWarps;
constexpr int kThreads = 64 + kEpiThreads;
constexpr int kSmem = kStages * (kA + kB) + kCBufs * kC + 1024 /*barriers*/ + 1024 /*align*/;

struct Problem {
  int M, N, nk, num_m, num_n;
  int64_t ldbits;
  float scale;
  bool bits_vec;   // a row's 8 mask words of a tile are two aligned 16-byte loads
};

template <bool kBmn>
__global__ void __launch_bounds__(kThreads, 1)
lora_dx_kernel(const __grid_constant__ CUtensorMap mV, const __grid_constant__ CUtensorMap mB,
               const __grid_constant__ CUtensorMap mC, const uint32_t* __restrict__ bits,
               const Problem pb, const tc::Ctl ctl) {
  int* err = ctl.err;
  tc::trace_begin(ctl);
  constexpr uint32_t kIdesc = tc::idesc_bf16(BM, BN, false, kBmn);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* ringAB = smem;                           // kStages x (A | B)
  uint8_t* cbuf = ringAB + kStages * (kA + kB);     // kCBufs x dx tile
  uint64_t* bar = reinterpret_cast<uint64_t*>(cbuf + kCBufs * kC);
  uint64_t* full = bar;               // [kStages] operands landed
  uint64_t* empty = full + kStages;   // [kStages] MMAs done with the stage
  uint64_t* cfull = empty + kStages;  // [kCBufs] dx tile landed
  uint64_t* cdone = cfull + kCBufs;   // [kCBufs] the 128 epilogue threads rewrote the tile
  uint64_t* cempty = cdone + kCBufs;  // [kCBufs] the store has read the tile out
  uint64_t* tfull = cempty + kCBufs;  // [2] accumulator ready
  uint64_t* tempty = tfull + 2;       // [2] accumulator drained
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) { tc::mbar_init(&full[s], 1); tc::mbar_init(&empty[s], 1); }
    for (int b = 0; b < kCBufs; ++b) {
      tc::mbar_init(&cfull[b], 1);
      tc::mbar_init(&cdone[b], kEpiThreads);
      tc::mbar_init(&cempty[b], 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(&tfull[b], 1);
      tc::mbar_init(&tempty[b], kEpiThreads);
    }
    tc::mbar_init(drain, 1);
    tc::fence_mbar_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, 2 * BN);
    tc::tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tc::prefetch_tmap(&mV);
    tc::prefetch_tmap(&mB);
    tc::prefetch_tmap(&mC);
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;
  const int num_tiles = pb.num_m * pb.num_n;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA loads
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      long issued = 0, c_issued = 0;
      int i = 0;
      for (int tile = blockIdx.x; tile < num_tiles && !tc::failed(err); tile += gridDim.x, ++i) {
        const int m0 = (tile % pb.num_m) * BM, n0 = (tile / pb.num_m) * BN;
        const int cb = i % kCBufs;
        if (!tc::mbar_wait(&cempty[cb], ((i / kCBufs) & 1) ^ 1, err, 41)) break;
        tc::mbar_expect_tx(&cfull[cb], kC);
#pragma unroll
        for (int j = 0; j < kSlabs; ++j)
          tc::tma_load_2d(cbuf + cb * kC + j * kSlab, &mC, &cfull[cb], n0 + 64 * j, m0);
        ++c_issued;
        bool ok = true;
        for (int kb = 0; kb < pb.nk; ++kb) {
          if (!tc::mbar_wait(&empty[s], ph ^ 1, err, 42)) { ok = false; break; }
          uint8_t* sA = ringAB + s * (kA + kB);
          uint8_t* sB = sA + kA;
          tc::mbar_expect_tx(&full[s], kA + kB);
          tc::tma_load_2d(sA, &mV, &full[s], kb * BK, m0);
          if (kBmn) {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tc::tma_load_2d(sB + j * 8192, &mB, &full[s], n0 + 64 * j, kb * BK);
          } else {
            tc::tma_load_2d(sB, &mB, &full[s], kb * BK, n0);
          }
          if (++s == kStages) { s = 0; ph ^= 1; }
          ++issued;
        }
        if (!ok) break;
      }
      if (tc::failed(err)) {   // let this CTA's copies in flight land before it exits
        for (int k = 0; k < kStages && k < issued; ++k) {
          if (--s < 0) { s = kStages - 1; ph ^= 1; }
          tc::mbar_wait_quiet(&full[s], ph);
        }
        for (long k = c_issued - 1; k >= 0 && k >= c_issued - kCBufs; --k)
          tc::mbar_wait_quiet(&cfull[k % kCBufs], (k / kCBufs) & 1);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issue
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      int i = 0;
      for (int tile = blockIdx.x; tile < num_tiles && !tc::failed(err); tile += gridDim.x, ++i) {
        const int buf = i & 1;
        if (!tc::mbar_wait(&tempty[buf], ((i >> 1) & 1) ^ 1, err, 43)) break;
        tc::fence_after_sync();
        const uint32_t d = tmem_base + buf * BN;
        bool ok = true;
        for (int kb = 0; kb < pb.nk; ++kb) {
          if (!tc::mbar_wait(&full[s], ph, err, 44)) { ok = false; break; }
          // TMA -> MMA is ordered by the barrier's transaction count: no tcgen05 fence here
          const uint32_t sA = tc::smem_u32(ringAB + s * (kA + kB));
          const uint32_t sB = sA + kA;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t a = tc::sdesc_sw128(sA + kk * 32, 16, 1024);
            const uint64_t b = kBmn ? tc::sdesc_sw128(sB + kk * 2048, 8192, 1024)
                                    : tc::sdesc_sw128(sB + kk * 32, 16, 1024);
            tc::mma_bf16(d, a, b, kIdesc, (kb | kk) != 0);
          }
          tc::mma_commit(&empty[s]);
          if (++s == kStages) { s = 0; ph ^= 1; }
        }
        if (!ok) break;
        tc::mma_commit(&tfull[buf]);
      }
      tc::mma_commit(drain);
      tc::mbar_wait_quiet(drain, 0);
    }
  } else {
    // ------------------------------------------------------------------ epilogue (warps 2-9)
    const int quarter = warp & 3;            // TMEM lanes this warp may read
    const int half = (warp - 2) >> 2;        // which 64 of the tile's 128 columns (one slab)
    const int row = quarter * 32 + lane;     // this thread's row of the tile
    const bool storer = threadIdx.x == 64;
    const int swz = row & 7;
    constexpr int kWords = BN / 64;          // mask words of a row's half tile
    // this row's mask words of its half of a tile (they depend on nothing in flight): fetched
    // one tile ahead, so their load latency hides under the previous tile's epilogue
    auto fetch_words = [&](int tile, uint32_t (&w)[kWords]) {
      const int m = (tile % pb.num_m) * BM + row, n0 = (tile / pb.num_m) * BN + half * 64;
      const int64_t w0 = static_cast<int64_t>(m) * pb.ldbits + (n0 >> 5);
      if (tile >= num_tiles || m >= pb.M) {
#pragma unroll
        for (int c = 0; c < kWords; ++c) w[c] = 0u;
      } else if (pb.bits_vec && (n0 >> 5) + kWords <= pb.ldbits) {
        const uint2 q = __ldg(reinterpret_cast<const uint2*>(bits + w0));
        w[0] = q.x; w[1] = q.y;
      } else {
#pragma unroll
        for (int c = 0; c < kWords; ++c)
          w[c] = (n0 >> 5) + c < pb.ldbits ? __ldg(bits + w0 + c) : 0u;
      }
    };
    uint32_t next[kWords];
    fetch_words(blockIdx.x, next);
    int i = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++i) {
      const int m0 = (tile % pb.num_m) * BM, n0 = (tile / pb.num_m) * BN;
      const int buf = i & 1, cb = i % kCBufs;
      const uint32_t par = (i >> 1) & 1, cpar = (i / kCBufs) & 1;
      uint32_t words[kWords];
#pragma unroll
      for (int c = 0; c < kWords; ++c) words[c] = next[c];
      fetch_words(tile + gridDim.x, next);
      const bool ready = tc::mbar_wait(&tfull[buf], par, err, 45) &&
                         tc::mbar_wait(&cfull[cb], cpar, err, 46);
      if (!__all_sync(0xffffffffu, ready)) break;   // warp-uniform: tcgen05.ld is collective
      tc::fence_after_sync();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + buf * BN;
      uint8_t* crow = cbuf + cb * kC + row * 128;
#pragma unroll
      for (int cc = 0; cc < kWords; ++cc) {
        const int ch = half * kWords + cc;   // 32-column chunk of the tile
        float v[32];
        tc::tmem_ld32(taddr + ch * 32, v);
        const uint32_t word = words[cc];
        uint8_t* slab_row = crow + (ch >> 1) * kSlab;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4* p = reinterpret_cast<uint4*>(slab_row + ((((ch & 1) * 4 + q) ^ swz) << 4));
          uint4 x = *p;
          uint32_t w4[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            __nv_bfloat162 pr = *reinterpret_cast<__nv_bfloat162*>(&w4[e]);
            float lo = __low2float(pr), hi = __high2float(pr);
            const int c = 8 * q + 2 * e;
            if ((word >> c) & 1u) lo = __fmaf_rn(pb.scale, v[c], lo);
            if ((word >> (c + 1)) & 1u) hi = __fmaf_rn(pb.scale, v[c + 1], hi);
            pr = __floats2bfloat162_rn(lo, hi);
            w4[e] = *reinterpret_cast<uint32_t*>(&pr);
          }
          *p = make_uint4(w4[0], w4[1], w4[2], w4[3]);
        }
      }
      tc::fence_before_sync();
      tc::mbar_arrive(&tempty[buf]);          // accumulator drained
      tc::fence_proxy_async_smem();           // the rewritten tile -> visible to the TMA store
      tc::mbar_arrive(&cdone[cb]);
      if (warp == 2) {   // the storer's outcome is made warp-uniform before the next tile
        bool stored = true;
        if (storer) {
          stored = tc::mbar_wait(&cdone[cb], cpar, err, 47);
          if (stored) {
#pragma unroll
            for (int j = 0; j < kSlabs; ++j)
              if (n0 + 64 * j < pb.N)
                tc::tma_store_2d(&mC, cbuf + cb * kC + j * kSlab, n0 + 64 * j, m0);
            tc::bulk_commit();
            // the store before this one has read its buffer out: hand that buffer back
            if (i > 0) {
              tc::bulk_wait_read_newest_pending();
              tc::mbar_arrive(&cempty[(i - 1) % kCBufs]);
            }
          }
        }
        if (!__shfl_sync(0xffffffffu, stored, 0)) break;
      }
    }
    if (storer) tc::bulk_wait_all();
  }

  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem_base, 2 * BN);
    if (lane == 0) tc::trace_end(ctl);
  }
}

}  // namespace

extern "C" int qb_gemm_bf16_mask_acc(const void* A, int64_t lda, const void* B, int64_t ldb,
                                     int b_mn_major, const uint32_t* bits, int64_t ldbits,
                                     float scale, void* C, int64_t ldc, int64_t M, int64_t N,
                                     int64_t K, cudaStream_t stream) {
  const char* what = "gemm_bf16_mask_acc";
  if (M < 0 || N < 0 || K < 0 || M > (1 << 30) || N > (1 << 30) || K > (1 << 30))
    return qb::fail(QB_ERR_INVALID, "%s: bad shape", what);
  if (M == 0 || N == 0) return QB_OK;
  if (K == 0) return qb::fail(QB_ERR_UNSUPPORTED, "%s: K == 0", what);
  if (!A || !B || !bits || !C) return qb::fail(QB_ERR_INVALID, "%s: null pointer", what);
  if (ldbits < (N + 31) / 32) return qb::fail(QB_ERR_INVALID, "%s: mask row stride", what);
  if (ldc < N) return qb::fail(QB_ERR_INVALID, "%s: output row stride", what);
  CUtensorMap mV, mB, mC;
  if (int s = tc_host::encode_2d(&mV, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, A, K, M, lda * 2, 64, BM,
                                 CU_TENSOR_MAP_SWIZZLE_128B))
    return s;
  if (b_mn_major) {
    if (int s = tc_host::encode_2d(&mB, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, B, N, K, ldb * 2, 64, 64,
                                   CU_TENSOR_MAP_SWIZZLE_128B))
      return s;
  } else {
    if (int s = tc_host::encode_2d(&mB, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, B, K, N, ldb * 2, 64, BN,
                                   CU_TENSOR_MAP_SWIZZLE_128B))
      return s;
  }
  if (int s = tc_host::encode_2d(&mC, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, C, N, M, ldc * 2, 64, BM,
                                 CU_TENSOR_MAP_SWIZZLE_128B))
    return s;
  Problem pb{static_cast<int>(M), static_cast<int>(N), static_cast<int>((K + BK - 1) / BK),
             static_cast<int>((M + BM - 1) / BM), static_cast<int>((N + BN - 1) / BN), ldbits,
             scale, qb::aligned16(bits) && ldbits % 4 == 0};
  auto kernel = b_mn_major ? lora_dx_kernel<true> : lora_dx_kernel<false>;
  if (int s = tc_host::ensure_smem(reinterpret_cast<const void*>(kernel), kSmem, what)) return s;
  const int tiles = pb.num_m * pb.num_n;
  int grid = tc_host::sm_count();
  if (grid > tiles) grid = tiles;
  tc::Ctl ctl;
  if (int s = tc_host::launch_ctl(&ctl, what)) return s;
  kernel<<<grid, kThreads, kSmem, stream>>>(mV, mB, mC, bits, pb, ctl);
  return qb::check_launch(what);
}
