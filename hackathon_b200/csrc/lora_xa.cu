// The LoRA down-projection of a dropped-out input, straight from the input and the mask bits:
//
//     U[M, R] = xd[M, K] A[R, K]^T,   xd = bf16(x * scale) where the mask bit is set, else 0
//
// mask bit (k & 31) of bits[m * ldbits + k / 32] (the words qb_dropout_mask / qb_dropout_bits
// write). xd is the very tensor qb_dropout_apply writes; here it lives only in shared memory
// (and, when the caller asks for it, is stored once by TMA), so the step no longer writes xd
// to HBM and reads it back for the adapter product. Without bits, xd = x (no dropout).
//
// Layout of the work: one CTA per 128-row block of x (persistent over blocks), the rank R
// (32..256, a multiple of 32) is the MMA's N, K streams through a ring of stages, each holding
// a 128 x 64 x tile and an R x 64 tile of A (both 128-byte swizzled, K-major, by TMA).
//   warp 0       TMA loads (x tile, A tile per stage)
//   warp 1       TMEM allocation; one thread issues tcgen05.mma (M = 128, N = R, K = 16) x 4
//   warps 2-17   masking: four threads per row, each rewrites one 32-byte quarter of its row
//                of the stage in place (bf16 -> fp32, packed * scale, -> bf16; or 0) with its
//                mask word (prefetched four k-blocks ahead), proxy fence, arrive; after a row
//                block's last stage, warps 2-9 move TMEM -> registers -> U (a warp pair per
//                TMEM lane quarter splits the columns)
//   warp 18      (xd requested) TMA-stores each masked stage tile to xd
// The masking is issue-bound work (a few instructions per element); sixteen warps keep four
// per scheduler so that the shared-memory and mask-word latencies hide behind one another.
// Every mbarrier wait is bounded (tc::mbar_wait): a wait that gives up raises the device error
// flag, the roles drain what they have in flight, and TMEM is released.
#include "qb_common.cuh"
#include "tc_common.cuh"

namespace {

constexpr int BM = 128, BK = 64;
constexpr int kMaxStages = 8;
constexpr int kMaskWarps = 16;
constexpr int kMaskThreads = kMaskWarps * 32;
constexpr int kStoreWarp = 2 + kMaskWarps;
constexpr int kThreads = (kStoreWarp + 1) * 32;
constexpr int kGroup = 4;                    // k-blocks whose mask words one prefetch covers
constexpr int kX = BM * 128;                 // 16 KiB: 128 rows x 64 bf16
constexpr int kRingBytes = 200 * 1024;       // stage ring budget
constexpr int kSmem = kRingBytes + 1024 /*barriers*/ + 1024 /*align*/;

struct Problem {
  int M, K, R, nk, num_m, stages, stage_bytes;
  int64_t ldbits, ldu;
  int kwords;          // ceil(K / 32): mask words a row holds
  float scale;
  bool masked, store_xd, bits_vec;   // bits_vec: a row's mask words load as aligned uint4
};

// The 8 mask words of k-blocks kb0 .. kb0 + 3 of one row (0 past the row's words).
__device__ __forceinline__ void load_words(const uint32_t* __restrict__ brow, int kb0,
                                           const Problem& pb, bool live, uint32_t* w) {
  const int w0 = 2 * kb0;
  if (live && pb.bits_vec && w0 + 8 <= pb.kwords) {
    const uint4 lo = __ldg(reinterpret_cast<const uint4*>(brow + w0));
    const uint4 hi = __ldg(reinterpret_cast<const uint4*>(brow + w0 + 4));
    w[0] = lo.x; w[1] = lo.y; w[2] = lo.z; w[3] = lo.w;
    w[4] = hi.x; w[5] = hi.y; w[6] = hi.z; w[7] = hi.w;
  } else {
#pragma unroll
    for (int c = 0; c < 8; ++c) w[c] = (live && w0 + c < pb.kwords) ? __ldg(brow + w0 + c) : 0u;
  }
}

// One bf16 pair of x -> bf16(x * scale) where its mask bit is set, else +0: two IEEE products
// in one packed f32x2 multiply (as two scalar multiplies round), one rounding to bf16 each.
__device__ __forceinline__ uint32_t drop_pair(uint32_t xp, uint32_t word, int c, uint64_t s2) {
  const float lo = __uint_as_float(xp << 16), hi = __uint_as_float(xp & 0xffff0000u);
  uint64_t v, pr;
  asm("mov.b64 %0, {%1, %2};" : "=l"(v) : "f"(lo), "f"(hi));
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(pr) : "l"(v), "l"(s2));
  float pl, ph;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(pl), "=f"(ph) : "l"(pr));
  pl = ((word >> c) & 1u) ? pl : 0.0f;
  ph = ((word >> (c + 1)) & 1u) ? ph : 0.0f;
  __nv_bfloat162 r = __floats2bfloat162_rn(pl, ph);
  return *reinterpret_cast<uint32_t*>(&r);
}

__global__ void __launch_bounds__(kThreads, 1)
lora_xa_kernel(const __grid_constant__ CUtensorMap mX, const __grid_constant__ CUtensorMap mA,
               const __grid_constant__ CUtensorMap mXd, const uint32_t* __restrict__ bits,
               __nv_bfloat16* __restrict__ u, const Problem pb, const tc::Ctl ctl) {
  int* err = ctl.err;
  tc::trace_begin(ctl);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* ring = smem;
  uint64_t* bar = reinterpret_cast<uint64_t*>(ring + kRingBytes);
  uint64_t* full = bar;                     // [stages] x and A landed
  uint64_t* masked = full + kMaxStages;     // [stages] the 128 rows rewritten
  uint64_t* empty = masked + kMaxStages;    // [stages] MMAs (and the xd store) done with it
  uint64_t* tfull = empty + kMaxStages;     // [2] accumulator ready
  uint64_t* tempty = tfull + 2;             // [2] accumulator drained
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = pb.stages;
  uint32_t tcols = 32;
  while (tcols < static_cast<uint32_t>(2 * pb.R)) tcols <<= 1;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&masked[s], kMaskThreads);
      tc::mbar_init(&empty[s], pb.store_xd ? 2 : 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(&tfull[b], 1);
      tc::mbar_init(&tempty[b], kMaskThreads);
    }
    tc::mbar_init(drain, 1);
    tc::fence_mbar_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, tcols);
    tc::tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tc::prefetch_tmap(&mX);
    tc::prefetch_tmap(&mA);
    if (pb.store_xd) tc::prefetch_tmap(&mXd);
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t kA = static_cast<uint32_t>(pb.R) * 128;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA loads
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      long issued = 0;
      bool ok = true;
      for (int mb = blockIdx.x; mb < pb.num_m && ok && !tc::failed(err); mb += gridDim.x) {
        for (int kb = 0; kb < pb.nk; ++kb) {
          if (!tc::mbar_wait(&empty[s], ph ^ 1, err, 61)) { ok = false; break; }
          uint8_t* sx = ring + s * pb.stage_bytes;
          tc::mbar_expect_tx(&full[s], kX + kA);
          tc::tma_load_2d(sx, &mX, &full[s], kb * BK, mb * BM);
          tc::tma_load_2d(sx + kX, &mA, &full[s], kb * BK, 0);
          if (++s == S) { s = 0; ph ^= 1; }
          ++issued;
        }
      }
      if (tc::failed(err)) {   // let this CTA's copies in flight land before it exits
        for (int k = 0; k < S && k < issued; ++k) {
          if (--s < 0) { s = S - 1; ph ^= 1; }
          tc::mbar_wait_quiet(&full[s], ph);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issue
    if (lane == 0) {
      const uint32_t idesc = tc::idesc_bf16(BM, pb.R, false, false);
      uint64_t* ready = pb.masked ? masked : full;
      int s = 0;
      uint32_t ph = 0;
      int i = 0;
      bool ok = true;
      for (int mb = blockIdx.x; mb < pb.num_m && ok && !tc::failed(err); mb += gridDim.x, ++i) {
        const int buf = i & 1;
        if (!tc::mbar_wait(&tempty[buf], ((i >> 1) & 1) ^ 1, err, 62)) break;
        tc::fence_after_sync();
        const uint32_t d = tmem_base + buf * pb.R;
        for (int kb = 0; kb < pb.nk; ++kb) {
          if (!tc::mbar_wait(&ready[s], ph, err, 63)) { ok = false; break; }
          const uint32_t sx = tc::smem_u32(ring + s * pb.stage_bytes);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t a = tc::sdesc_sw128(sx + kk * 32, 16, 1024);
            const uint64_t b = tc::sdesc_sw128(sx + kX + kk * 32, 16, 1024);
            tc::mma_bf16(d, a, b, idesc, (kb | kk) != 0);
          }
          tc::mma_commit(&empty[s]);
          if (++s == S) { s = 0; ph ^= 1; }
        }
        if (!ok) break;
        tc::mma_commit(&tfull[buf]);
      }
      tc::mma_commit(drain);
      tc::mbar_wait_quiet(drain, 0);
    }
  } else if (warp == kStoreWarp) {
    // ------------------------------------------------------------------ xd stores
    if (pb.store_xd && lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int mb = blockIdx.x; mb < pb.num_m && ok; mb += gridDim.x) {
        for (int kb = 0; kb < pb.nk; ++kb) {
          if (!tc::mbar_wait(&masked[s], ph, err, 64)) { ok = false; break; }
          tc::tma_store_2d(&mXd, ring + s * pb.stage_bytes, kb * BK, mb * BM);
          tc::bulk_commit();
          tc::bulk_wait_read_all();           // the tile is read out: the stage may refill
          tc::mbar_arrive(&empty[s]);
          if (++s == S) { s = 0; ph ^= 1; }
        }
      }
      tc::bulk_wait_all();
    }
  } else {
    // ------------------------------------------------------------------ masking + epilogue
    const int mw = warp - 2;                 // 0 .. 15
    const int part = mw >> 2;                // which 16 columns of a k-block this thread masks
    const int row = (mw & 3) * 32 + lane;    // this thread's row while masking
    const int swz = row & 7;
    const int quarter = warp & 3;            // TMEM lanes this warp may read (epilogue row)
    const int erow = quarter * 32 + lane;
    const int half = part & 1;               // warps 2-9 drain: parts 0 and 1
    const bool split = pb.R % 64 == 0;       // the warp pair of a quarter splits the columns
    const int ecols = split ? pb.R / 2 : pb.R;
    const int ecol0 = split ? half * ecols : 0;
    const bool drains = part < 2 && (split || half == 0);
    uint64_t s2;
    asm("mov.b64 %0, {%1, %1};" : "=l"(s2) : "f"(pb.scale));
    int s = 0;
    uint32_t ph = 0;
    int i = 0;
    for (int mb = blockIdx.x; mb < pb.num_m; mb += gridDim.x, ++i) {
      bool ok = true;
      if (pb.masked) {
        const int m = mb * BM + row;
        const bool live = m < pb.M;
        const uint32_t* brow = bits + static_cast<int64_t>(live ? m : 0) * pb.ldbits;
        uint32_t cur[8], nxt[8];
        load_words(brow, 0, pb, live, cur);
        for (int kb0 = 0; kb0 < pb.nk && ok; kb0 += kGroup) {
          load_words(brow, kb0 + kGroup, pb, live, nxt);   // in flight while this group runs
#pragma unroll
          for (int j = 0; j < kGroup; ++j) {
            if (kb0 + j >= pb.nk) break;
            const bool landed = tc::mbar_wait(&full[s], ph, err, 65);
            if (!__all_sync(0xffffffffu, landed)) { ok = false; break; }
            // columns 16 part .. 16 part + 15: bits (16 part) & 31 .. of word 2 kb + part / 2
            const uint32_t word =
                (part >= 2 ? cur[2 * j + 1] : cur[2 * j]) >> ((part & 1) * 16);
            uint8_t* srow = ring + s * pb.stage_bytes + row * 128;
            uint4 xv[2];
#pragma unroll
            for (int q = 0; q < 2; ++q)
              xv[q] = *reinterpret_cast<const uint4*>(srow + (((2 * part + q) ^ swz) << 4));
#pragma unroll
            for (int q = 0; q < 2; ++q)
              xv[q] = make_uint4(drop_pair(xv[q].x, word, 8 * q + 0, s2),
                                 drop_pair(xv[q].y, word, 8 * q + 2, s2),
                                 drop_pair(xv[q].z, word, 8 * q + 4, s2),
                                 drop_pair(xv[q].w, word, 8 * q + 6, s2));
#pragma unroll
            for (int q = 0; q < 2; ++q)
              *reinterpret_cast<uint4*>(srow + (((2 * part + q) ^ swz) << 4)) = xv[q];
            tc::fence_proxy_async_smem();   // rewritten row quarter -> visible to MMA / store
            tc::mbar_arrive(&masked[s]);
            if (++s == S) { s = 0; ph ^= 1; }
          }
#pragma unroll
          for (int c = 0; c < 8; ++c) cur[c] = nxt[c];
        }
      }
      if (!ok) break;
      const int buf = i & 1;
      const bool ready = tc::mbar_wait(&tfull[buf], (i >> 1) & 1, err, 66);
      if (!__all_sync(0xffffffffu, ready)) break;   // warp-uniform: tcgen05.ld is collective
      tc::fence_after_sync();
      if (drains) {
        const int m = mb * BM + erow;
        const bool live = m < pb.M;
        const uint32_t taddr =
            tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + buf * pb.R + ecol0;
        __nv_bfloat16* urow = u + static_cast<int64_t>(live ? m : 0) * pb.ldu + ecol0;
        for (int ch = 0; ch < ecols / 32; ++ch) {
          float v[32];
          tc::tmem_ld32(taddr + ch * 32, v);
          if (live) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              uint32_t w4[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                __nv_bfloat162 pr =
                    __floats2bfloat162_rn(v[8 * q + 2 * e], v[8 * q + 2 * e + 1]);
                w4[e] = *reinterpret_cast<uint32_t*>(&pr);
              }
              *reinterpret_cast<uint4*>(urow + ch * 32 + 8 * q) =
                  make_uint4(w4[0], w4[1], w4[2], w4[3]);
            }
          }
        }
      }
      tc::fence_before_sync();
      tc::mbar_arrive(&tempty[buf]);          // accumulator drained
    }
  }

  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem_base, tcols);
    if (lane == 0) tc::trace_end(ctl);
  }
}

}  // namespace

extern "C" int qb_lora_xa(const void* x, int64_t ldx, const void* a, int64_t lda,
                          const uint32_t* bits, int64_t ldbits, float scale, void* u, int64_t ldu,
                          void* xd, int64_t ldxd, int64_t M, int64_t K, int64_t R,
                          cudaStream_t stream) {
  const char* what = "lora_xa";
  if (M < 0 || K < 0 || M > (1 << 30) || K > (1 << 30))
    return qb::fail(QB_ERR_INVALID, "%s: bad shape", what);
  if (R < 32 || R > 256 || R % 32)
    return qb::fail(QB_ERR_UNSUPPORTED, "%s: rank must be a multiple of 32 in 32..256", what);
  if (M == 0) return QB_OK;
  if (K == 0) return qb::fail(QB_ERR_UNSUPPORTED, "%s: K == 0", what);
  if (!x || !a || !u) return qb::fail(QB_ERR_INVALID, "%s: null pointer", what);
  if (xd && !bits) return qb::fail(QB_ERR_INVALID, "%s: xd is stored only with a mask", what);
  if (bits && ldbits < (K + 31) / 32) return qb::fail(QB_ERR_INVALID, "%s: mask row stride", what);
  if (ldx < K || lda < K || ldu < R || (xd && ldxd < K))
    return qb::fail(QB_ERR_INVALID, "%s: row stride", what);
  if (!qb::aligned16(u) || (ldu * 2) % 16)
    return qb::fail(QB_ERR_INVALID, "%s: U rows must be 16-byte aligned", what);
  CUtensorMap mX, mA, mXd;
  if (int s = tc_host::encode_2d(&mX, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, x, K, M, ldx * 2, 64, BM,
                                 CU_TENSOR_MAP_SWIZZLE_128B))
    return s;
  if (int s = tc_host::encode_2d(&mA, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a, K, R, lda * 2, 64,
                                 static_cast<uint32_t>(R), CU_TENSOR_MAP_SWIZZLE_128B))
    return s;
  mXd = mX;
  if (xd) {
    if (int s = tc_host::encode_2d(&mXd, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, xd, K, M, ldxd * 2, 64,
                                   BM, CU_TENSOR_MAP_SWIZZLE_128B))
      return s;
  }
  Problem pb{};
  pb.M = static_cast<int>(M);
  pb.K = static_cast<int>(K);
  pb.R = static_cast<int>(R);
  pb.nk = static_cast<int>((K + BK - 1) / BK);
  pb.num_m = static_cast<int>((M + BM - 1) / BM);
  pb.stage_bytes = kX + static_cast<int>(R) * 128;
  pb.stages = kRingBytes / pb.stage_bytes;
  if (pb.stages > kMaxStages) pb.stages = kMaxStages;
  pb.ldbits = ldbits;
  pb.ldu = ldu;
  pb.kwords = static_cast<int>((K + 31) / 32);
  pb.scale = bits ? scale : 1.0f;
  pb.masked = bits != nullptr;
  pb.store_xd = xd != nullptr;
  pb.bits_vec = bits && qb::aligned16(bits) && ldbits % 4 == 0;
  if (int s = tc_host::ensure_smem(reinterpret_cast<const void*>(lora_xa_kernel), kSmem, what))
    return s;
  int grid = tc_host::sm_count();
  if (grid > pb.num_m) grid = pb.num_m;
  tc::Ctl ctl;
  if (int s = tc_host::launch_ctl(&ctl, what)) return s;
  lora_xa_kernel<<<grid, kThreads, kSmem, stream>>>(mX, mA, mXd, bits,
                                                    static_cast<__nv_bfloat16*>(u), pb, ctl);
  return qb::check_launch(what);
}
