// The NF4-weight GEMM on tcgen05: D[M, N] = A[M, K] * B[N, K]^T where A is an NF4 weight
// (K-major: A = W, or MN-major: A = W^T) rebuilt to bf16 inside the kernel, optionally followed
// by a second K segment whose A is a bf16 LoRA matrix (the adapter term as extra K), and B is
// bf16 activations brought in by TMA.
//
// Three shared-memory rings decouple the latencies:
//   codes ring (8 x 4 KiB)   packed NF4 codes of one 128 x 64 A tile, TMA (warp 6)
//   B ring     (2 x 64 KiB)  512 x 64 activation tile (two 256-row halves), TMA (warp 0)
//   A ring     (3 x 16 KiB)  the bf16 A tile in the swizzled layout the MMA reads, written by
//                            two groups of eight dequant warps (warps 7-22) taking alternate k-blocks
//                            (32 weights per thread): NF4 codes x block scale for segment 0, a copy
//                            of the LoRA matrix for segment 1
// The codes ring runs far ahead of the dequant warps, which run up to three k-blocks ahead of
// the MMA; with alternate k-blocks each warp has two MMA k-steps to turn one tile around.
// An output tile is 128 x 512: each dequantised A k-slice feeds two N=256 MMAs, which halves the
// dequant work and its shared-memory traffic per flop. The hand-off of the thread-written A
// operand (stores, proxy fence, barrier round trip), not the tensor pipe, bounds this kernel:
// with the dequant arithmetic removed it still runs at ~1.1 PFLOP/s, against ~1.4 for the same
// contraction with A brought in by TMA. Long token counts therefore go through a transient
// bf16 weight and the TMA-fed GEMM instead (the host-side dispatch); this kernel serves the
// short ones, where reading 0.5 byte per weight instead of 2 is what counts. The two 256-column
// accumulators fill all 512 TMEM columns, so the epilogue (warps 2-5) drains a tile before the
// MMAs of the next one start. Warp 1 issues the MMAs (one thread). Every wait is bounded; a
// wait that gives up raises the device error flag and every role drains out; TMEM is always
// released.
#pragma once

#include "tc_gemm.cuh"

namespace tcn {

using tcg::BK;
using tcg::BM;

enum Nf4Src : int { kNf4K = 2, kNf4MN = 3 };   // A = W (K-major) or A = W^T (MN-major)

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

// Per code byte: both nibble indices come pre-multiplied by 4 (one shift + mask per 4 bytes,
// one byte permute per index), the two table values are multiplied by the scale in one packed
// f32x2 multiply (two IEEE round-to-nearest products, as two scalar multiplies would give) and
// rounded to bf16 in one cvt. Byte j of the codes holds weights 2j (high nibble) and 2j+1.
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

// The raw ingredients of one block scale (code of the first-level absmax, second-level scale),
// loaded a couple of k-steps before they are needed; code < 0 marks an out-of-range block.
struct ScaleRaw {
  int code;
  float a2;
};

// scale = code2[code] * absmax2 + offset: a rounded multiply, then a rounded add (no FMA).
__device__ __forceinline__ float scale_of(const ScaleRaw& r, const float* s_code2, float offset) {
  return r.code < 0 ? 0.f : __fadd_rn(__fmul_rn(s_code2[r.code], r.a2), offset);
}

constexpr int kBN = 256;            // N of one MMA
constexpr int kNT = 2;              // MMAs per k-step: the output tile is 128 x 512
constexpr int kTN = kBN * kNT;
constexpr int kStagesB = 2, kStagesA = 3, kStagesC = 8;
constexpr int kA = BM * 128;        // 16 KiB
constexpr int kB = kTN * 128;       // 64 KiB
constexpr int kC = 4096;            // packed codes of one A tile
constexpr int kThreads = 736;       // 23 warps
constexpr int kWarpCodes = 6, kWarpDeq0 = 7;
constexpr int kGroups = 2;            // dequant warp-groups, alternating k-blocks
constexpr int kGroupThreads = 256;    // one group rebuilds a whole 128 x 64 tile
constexpr int kDeqThreads = kGroups * kGroupThreads;
// A group waits for an item's codes after that item's A slot is free; its own previous item read
// the codes stage before that, so the phase-parity wait on a codes stage is never two
// generations ahead of its fills as long as the ring has a stage per group.
static_assert(kStagesC >= kGroups, "codes ring shorter than the number of dequant groups");
constexpr int kSmem = kStagesB * kB + kStagesA * kA + kStagesC * kC + 1024 + 1024 + (256 + 16) * 4;

struct LoraA {               // segment-1 A operand (bf16), read by the dequant warps
  const __nv_bfloat16* p;    // K-major: [M rows, r] (row stride ld); MN-major: [r, M] (stride ld)
  int64_t ld;
  int r;
};

struct NfProblem {
  int M, N;
  int nk0, nk1;
  int num_m, num_n;
  int bs2_shift;   // log2(blocksize2)
};

// 32 bf16 values (4 chunks) of one thread's share of a segment-1 A tile, straight from global:
// chunk j of the thread goes to chunk position (c0 + (j ^ rot)) ^ swz and holds elements
// k0 + 8 * (j ^ rot) .. + 7 (zero past r).
__device__ __forceinline__ void copy32(const __nv_bfloat16* src, bool row_ok, int k0, int r,
                                       uint8_t* row, int c0, int rot, int swz) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int cl = j ^ rot;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (row_ok && k0 + 8 * cl < r) v = __ldg(reinterpret_cast<const uint4*>(src + 8 * cl));
    *reinterpret_cast<uint4*>(row + (((c0 + cl) ^ swz) << 4)) = v;
  }
}

// 32 weights (16 packed bytes, one scale block) into four 16-byte chunks of a swizzled row,
// stored in the rotated order j ^ rot so the lanes of a warp hit distinct banks.
__device__ __forceinline__ void dequant32(const uint8_t* codes, float scale, const float* lut,
                                          uint8_t* row, int c0, int rot, int swz) {
  const uint4 cw = *reinterpret_cast<const uint4*>(codes);
  const uint32_t w[4] = {cw.x, cw.y, cw.z, cw.w};
  uint64_t scale2;
  asm("mov.b64 %0, {%1, %1};" : "=l"(scale2) : "f"(scale));
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int cl = j ^ rot;
    const uint32_t x = w[cl];
    const uint32_t hi4 = (x >> 2) & 0x3C3C3C3Cu;
    const uint32_t lo4 = (x << 2) & 0x3C3C3C3Cu;
    uint32_t o[4];
#pragma unroll
    for (int b = 0; b < 4; ++b) o[b] = nf4_pair(lut, hi4, lo4, b, scale2);
    *reinterpret_cast<uint4*>(row + (((c0 + cl) ^ swz) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

template <int A0, class Epi>
__global__ void __launch_bounds__(kThreads, 1)
tc_nf4_kernel(const __grid_constant__ CUtensorMap mCodes, const __grid_constant__ CUtensorMap mB0,
              const __grid_constant__ CUtensorMap mB1, const NfProblem pb,
              const Nf4Operand nf4, const LoraA lora, Epi epi, const tc::Ctl ctl) {
  int* err = ctl.err;
  tc::trace_begin(ctl);
  static_assert(A0 == kNf4K || A0 == kNf4MN, "A0 is an NF4 source");
  constexpr bool kMN = A0 == kNf4MN;
  constexpr uint32_t kIdesc0 = tc::idesc_bf16(BM, kBN, kMN, false);
  constexpr uint32_t kIdesc1 = kIdesc0;   // segment-1 A uses the same major-ness

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* ringB = smem;
  uint8_t* ringA = ringB + kStagesB * kB;
  uint8_t* ringC = ringA + kStagesA * kA;
  uint64_t* bar = reinterpret_cast<uint64_t*>(ringC + kStagesC * kC);
  uint64_t* fullB = bar;
  uint64_t* emptyB = fullB + kStagesB;
  uint64_t* fullA = emptyB + kStagesB;
  uint64_t* emptyA = fullA + kStagesA;
  uint64_t* fullC = emptyA + kStagesA;
  uint64_t* emptyC = fullC + kStagesC;
  uint64_t* tfull = emptyC + kStagesC;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  float* s_code2 = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bar) + 1024);
  float* s_lut = s_code2 + 256;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStagesB; ++s) { tc::mbar_init(&fullB[s], 1); tc::mbar_init(&emptyB[s], 1); }
    for (int s = 0; s < kStagesA; ++s) { tc::mbar_init(&fullA[s], kGroupThreads); tc::mbar_init(&emptyA[s], 1); }
    for (int s = 0; s < kStagesC; ++s) { tc::mbar_init(&fullC[s], 1); tc::mbar_init(&emptyC[s], kGroupThreads / 32); }
    for (int b = 0; b < 2; ++b) { tc::mbar_init(&tfull[b], 1); tc::mbar_init(&tempty[b], 128); }
    tc::mbar_init(drain, 1);
    tc::fence_mbar_init();
  }
  if (threadIdx.x < 256) s_code2[threadIdx.x] = nf4.code2[threadIdx.x];
  if (threadIdx.x < 16) s_lut[threadIdx.x] = nf4.lut[threadIdx.x];
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, 2 * kBN);
    tc::tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tc::prefetch_tmap(&mB0);
    if (pb.nk1 > 0) tc::prefetch_tmap(&mB1);
  }
  if (warp == kWarpCodes && lane == 0) tc::prefetch_tmap(&mCodes);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;
  const int num_tiles = pb.num_m * pb.num_n;
  const int nk = pb.nk0 + pb.nk1;

  if (warp == 0) {
    // ------------------------------------------------------------ B producer (activations)
    if (lane == 0) {
      int st = 0;
      uint32_t ph = 0;
      long issued = 0;
      for (int tile = blockIdx.x; tile < num_tiles && !tc::failed(err); tile += gridDim.x) {
        const int n0 = (tile / pb.num_m) * kTN;
        for (int kb = 0; kb < nk; ++kb) {
          if (!tc::mbar_wait(&emptyB[st], ph ^ 1, err, 11)) break;
          const bool seg1 = kb >= pb.nk0;
          const int k = (seg1 ? kb - pb.nk0 : kb) * BK;
          tc::mbar_expect_tx(&fullB[st], kB);
#pragma unroll
          for (int j = 0; j < kNT; ++j)
            tc::tma_load_2d(ringB + st * kB + j * (kBN * 128), seg1 ? &mB1 : &mB0, &fullB[st], k,
                            n0 + j * kBN);
          if (++st == kStagesB) { st = 0; ph ^= 1; }
          ++issued;
        }
      }
      if (tc::failed(err))
        for (int i = 0; i < kStagesB && i < issued; ++i) {
          if (--st < 0) { st = kStagesB - 1; ph ^= 1; }
          tc::mbar_wait_quiet(&fullB[st], ph);
        }
    }
  } else if (warp == kWarpCodes) {
    // ------------------------------------------------------------ codes producer
    if (lane == 0) {
      int st = 0;
      uint32_t ph = 0;
      long issued = 0;
      for (int tile = blockIdx.x; tile < num_tiles && !tc::failed(err); tile += gridDim.x) {
        const int m0 = (tile % pb.num_m) * BM;
        for (int kb = 0; kb < pb.nk0; ++kb) {
          if (!tc::mbar_wait(&emptyC[st], ph ^ 1, err, 12)) break;
          tc::mbar_expect_tx(&fullC[st], kC);
          if (!kMN) tc::tma_load_2d(ringC + st * kC, &mCodes, &fullC[st], kb * 32, m0);
          else tc::tma_load_2d(ringC + st * kC, &mCodes, &fullC[st], m0 / 2, kb * BK);
          if (++st == kStagesC) { st = 0; ph ^= 1; }
          ++issued;
        }
      }
      if (tc::failed(err))
        for (int i = 0; i < kStagesC && i < issued; ++i) {
          if (--st < 0) { st = kStagesC - 1; ph ^= 1; }
          tc::mbar_wait_quiet(&fullC[st], ph);
        }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int sb = 0, sa = 0;
      uint32_t pbh = 0, pah = 0;
      int t = 0;
      for (int tile = blockIdx.x; tile < num_tiles && !tc::failed(err); tile += gridDim.x, ++t) {
        // one accumulator set (all 512 columns): wait until the epilogue drained the last tile
        if (!tc::mbar_wait(&tempty[0], (t & 1) ^ 1, err, 13)) break;
        tc::fence_after_sync();
        const uint32_t d = tmem_base;
        bool ok = true;
        for (int kb = 0; kb < nk; ++kb) {
          if (!tc::mbar_wait(&fullB[sb], pbh, err, 14) || !tc::mbar_wait(&fullA[sa], pah, err, 15)) {
            ok = false;
            break;
          }
          tc::fence_after_sync();
          const uint32_t a_s = tc::smem_u32(ringA + sa * kA);
          const uint32_t b_s = tc::smem_u32(ringB + sb * kB);
          const uint32_t idesc = kb >= pb.nk0 ? kIdesc1 : kIdesc0;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t a = kMN ? tc::sdesc_sw128(a_s + kk * 2048, 8192, 1024)
                                   : tc::sdesc_sw128(a_s + kk * 32, 16, 1024);
#pragma unroll
            for (int j = 0; j < kNT; ++j) {
              const uint64_t b = tc::sdesc_sw128(b_s + j * (kBN * 128) + kk * 32, 16, 1024);
              tc::mma_bf16(d + j * kBN, a, b, idesc, (kb | kk) != 0);
            }
          }
          tc::mma_commit(&emptyB[sb]);
          tc::mma_commit(&emptyA[sa]);
          if (++sb == kStagesB) { sb = 0; pbh ^= 1; }
          if (++sa == kStagesA) { sa = 0; pah ^= 1; }
        }
        if (!ok) break;
        tc::mma_commit(&tfull[0]);
      }
      tc::mma_commit(drain);
      tc::mbar_wait_quiet(drain, 0);
    }
  } else if (warp < kWarpCodes) {
    // ------------------------------------------------------------ epilogue (warps 2-5)
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    int t = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++t) {
      const bool ready = tc::mbar_wait(&tfull[0], t & 1, err, 16);
      if (!__all_sync(0xffffffffu, ready)) break;
      tc::fence_after_sync();
      const int m0 = (tile % pb.num_m) * BM, n0 = (tile / pb.num_m) * kTN;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
#pragma unroll 1
      for (int j = 0; j < kNT; ++j) epi.template tile<kBN>(m0, n0 + j * kBN, row, taddr + j * kBN);
      tc::fence_before_sync();
      tc::mbar_arrive(&tempty[0]);
    }
  } else {
    // ------------------------------------------------------------ dequant (warps 7-22)
    const int d = threadIdx.x - kWarpDeq0 * 32;
    const int group = d / kGroupThreads, dl = d % kGroupThreads;
    int off_codes, off_row, c0, rot, swz, a_row, a_blk;
    if (!kMN) {              // thread -> (A row = weight row, half of the 64 k)
      const int r = dl >> 1, h = dl & 1;
      off_codes = r * 32 + h * 16;
      off_row = r * 128;
      c0 = h * 4;
      rot = 0;
      swz = r & 7;
      a_row = r;             // + m0
      a_blk = h;             // which 32 of the 64 k (segment-1 copy)
    } else {                 // thread -> (k row = weight row, quarter of the 128 m)
      const int kr = dl >> 2, q = dl & 3;
      off_codes = kr * 64 + q * 16;
      off_row = (q >> 1) * 8192 + kr * 128;
      c0 = (q & 1) * 4;
      rot = (q >> 1) * 2;    // the two 64-wide halves store their chunks in different orders
      swz = kr & 7;
      a_row = kr;
      a_blk = q;
    }
    const float offset = nf4.offset;
    auto raw_for = [&](int tile, int kb) -> ScaleRaw {
      if (tile >= num_tiles || kb >= pb.nk0) return ScaleRaw{-1, 0.f};
      const int m0 = (tile % pb.num_m) * BM;
      const int row = kMN ? kb * BK + a_row : m0 + a_row;
      const int blk_in_row = kMN ? (m0 >> 6) + (a_blk >> 1) : kb;
      if (row >= nf4.rows || blk_in_row >= nf4.blocks_per_row) return ScaleRaw{-1, 0.f};
      const int64_t blk = static_cast<int64_t>(row) * nf4.blocks_per_row + blk_in_row;
      return ScaleRaw{static_cast<int>(__ldg(nf4.absmax_q + blk)),
                           __ldg(nf4.absmax2 + (blk >> pb.bs2_shift))};
    };
    // the item (tile, kb) two k-blocks after (tile, kb): this group's next one
    auto next2 = [&](int& tile, int& kb) {
      kb += kGroups;
      while (kb >= nk && tile < num_tiles) { kb -= nk; tile += gridDim.x; }
    };
    int sa = 0, sc = 0;
    uint32_t pah = 0, pch = 0;
    long it = 0;
    bool ok = true;
    int pt = blockIdx.x, pk = group;              // this group's next item to prefetch
    while (pk >= nk && pt < num_tiles) { pk -= nk; pt += gridDim.x; }
    ScaleRaw pre = raw_for(pt, pk);
    for (int tile = blockIdx.x; tile < num_tiles && ok && !tc::failed(err); tile += gridDim.x) {
      const int m0 = (tile % pb.num_m) * BM;
      for (int kb = 0; kb < nk; ++kb, ++it) {
        const bool seg0 = kb < pb.nk0;
        if ((it % kGroups) == group) {
          const ScaleRaw cur = pre;
          next2(pt, pk);
          pre = raw_for(pt, pk);
          if (!tc::mbar_wait(&emptyA[sa], pah ^ 1, err, 17)) { ok = false; break; }
          uint8_t* a_dst = ringA + sa * kA + off_row;
          if (seg0) {
            if (!tc::mbar_wait(&fullC[sc], pch, err, 18)) { ok = false; break; }
            dequant32(ringC + sc * kC + off_codes, scale_of(cur, s_code2, offset), s_lut,
                      a_dst, c0, rot, swz);
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&emptyC[sc]);
          } else {
            const int kb1 = kb - pb.nk0;
            if (!kMN) {      // s*B_lora [M rows, r]: row m0 + a_row, k = kb1*64 + 32*half
              const int row = m0 + a_row, k0 = kb1 * BK + a_blk * 32;
              copy32(lora.p + static_cast<int64_t>(row) * lora.ld + k0, row < pb.M, k0, lora.r,
                     a_dst, c0, rot, swz);
            } else {         // A_lora [r, M]: k row kb1*64 + a_row, m = m0 + 32*quarter
              const int kr = kb1 * BK + a_row, m = m0 + a_blk * 32;
              copy32(lora.p + static_cast<int64_t>(kr) * lora.ld + m, kr < lora.r && m < pb.M, 0,
                     32, a_dst, c0, rot, swz);
            }
          }
          tc::fence_proxy_async_smem();
          tc::mbar_arrive(&fullA[sa]);
        }
        if (++sa == kStagesA) { sa = 0; pah ^= 1; }
        if (seg0 && ++sc == kStagesC) { sc = 0; pch ^= 1; }
      }
    }
  }

  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem_base, 2 * kBN);
    if (lane == 0) tc::trace_end(ctl);
  }
}

template <int A0, class Epi>
int launch_nf4(const CUtensorMap& mCodes, const CUtensorMap& mB0, const CUtensorMap& mB1,
               const NfProblem& pb, const Nf4Operand& nf4, const LoraA& lora,
               const Epi& epi, cudaStream_t stream, const char* what) {
  auto kernel = tc_nf4_kernel<A0, Epi>;
  if (int s = tc_host::ensure_smem(reinterpret_cast<const void*>(kernel), kSmem, what)) return s;
  const int tiles = pb.num_m * pb.num_n;
  if (tiles == 0) return QB_OK;
  int grid = tc_host::sm_count();
  if (grid > tiles) grid = tiles;
  tc::Ctl ctl;
  if (int s = tc_host::launch_ctl(&ctl, what)) return s;
  kernel<<<grid, kThreads, kSmem, stream>>>(mCodes, mB0, mB1, pb, nf4, lora, epi, ctl);
  return qb::check_launch(what);
}

}  // namespace tcn
