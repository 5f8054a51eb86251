// Blackwell (sm_100a) building blocks for the tensor-core kernels: mbarriers with bounded waits,
// TMA tile loads, tcgen05 MMA / commit / TMEM load, shared-memory matrix descriptors, and the
// host-side tensor-map encoder.
//
// Shared-memory operand layout used throughout: 128-byte-swizzled tiles ("SW128").
//   K-major tile (rows x 64 bf16): row r occupies 128 bytes at r*128; its 16-byte chunk c sits
//     at chunk position c ^ (r & 7); 8-row groups are 1024 bytes apart (SBO = 1024).
//   MN-major tile (64 k-rows x N bf16, N in chunks of 64): chunk j of 64 MN-elements is an
//     8 KiB block of 64 k-rows x 128 bytes (same swizzle); chunks are 8 KiB apart (LBO = 8192),
//     8-row k groups 1024 bytes apart (SBO = 1024).
// TMA with CU_TENSOR_MAP_SWIZZLE_128B writes exactly these layouts; the NF4 producers write them
// from registers.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace tc {

// ------------------------------------------------------------------------------------------
// error flag + bounded waits. A wait that gives up records `code` in *err (first one wins) and
// returns false; every role checks the flag and leaves its loop, so the CTA drains and exits.
//
// *err is word 0 of the device's ErrBlock. Its `host` member points into pinned host memory
// mapped into the device (the launch monitor, tc_host.cu): the wait that raises the flag also
// writes its site there, so a host thread can read it with a plain load while the device is
// still busy, with no CUDA call that could queue behind the stuck work.

struct ErrBlock {
  int flag;          // polled by every bounded wait (device memory: cheap to read)
  int pad;
  int* host;         // mapped host record {site, block, sm} or null
};

// Per launch: the error flag and the launch monitor's trace. Each CTA writes 2 * seq into
// trace[blockIdx.x] as it starts and 2 * seq + 1 once it has released TMEM and is leaving,
// so a CTA that never leaves (and the launch it belongs to) can be named from the host.
struct Ctl {
  int* err;
  uint32_t* trace;   // mapped host memory, kTraceSlots entries, or null
  uint32_t seq;      // the host's launch sequence number
};

constexpr int kTraceSlots = 1024;

constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s: far above any legitimate wait

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Elapsed-time test of every bounded wait: limit_ns passed on %globaltimer AND at least
// limit_ns / 2 cycles passed on this SM's free-running cycle counter. %globaltimer is kept by
// the driver and may step forward when it is resynchronised; the cycle counter cannot jump, so
// a timer step alone never makes a healthy wait give up. At any SM clock of 0.5 GHz or more the
// cycle test holds by the time the timer test does, so the bound stays limit_ns.
__device__ __forceinline__ uint64_t sm_cycles() {
  uint64_t c;
  asm volatile("mov.u64 %0, %%clock64;" : "=l"(c));
  return c;
}

__device__ __forceinline__ uint32_t sm_id() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%smid;" : "=r"(r));
  return r;
}

// System-scope store into mapped host memory (the launch monitor): no cache keeps it.
__device__ __forceinline__ void st_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ void trace_begin(const Ctl& c) {
  if (threadIdx.x == 0 && c.trace && blockIdx.x < static_cast<unsigned>(kTraceSlots))
    st_sys(c.trace + blockIdx.x, 2u * c.seq);
}

__device__ __forceinline__ void trace_end(const Ctl& c) {
  if (c.trace && blockIdx.x < static_cast<unsigned>(kTraceSlots))
    st_sys(c.trace + blockIdx.x, 2u * c.seq + 1u);
}

// Raises the flag with `code` (first one wins) and, for the first, writes the site, the CTA
// and its SM into the mapped host record.
__device__ __forceinline__ void raise_error(int* err, int code) {
  if (atomicCAS(err, 0, code) != 0) return;
  int* host = reinterpret_cast<ErrBlock*>(err)->host;
  if (host) {
    st_sys(reinterpret_cast<uint32_t*>(host) + 1, blockIdx.x);
    st_sys(reinterpret_cast<uint32_t*>(host) + 2, sm_id());
    st_sys(reinterpret_cast<uint32_t*>(host), static_cast<uint32_t>(code));
    __threadfence_system();
  }
}

struct WaitClock {
  uint64_t t0, c0;
  __device__ __forceinline__ WaitClock() {
    t0 = globaltimer();
    c0 = sm_cycles();
  }
  __device__ __forceinline__ bool expired(uint64_t limit_ns) const {
    return globaltimer() - t0 > limit_ns && sm_cycles() - c0 > limit_ns / 2;
  }
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

// try_wait with a suspend-time hint: a waiting warp sleeps in hardware until the phase completes
// (or ~0.5 ms pass) instead of spinning, so it does not take issue slots from working warps.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(500000u)
      : "memory");
  return ok != 0;
}

// How many failed try_waits pass between two looks at the error flag and the clock. Each failed
// try_wait may sleep up to its 0.5 ms suspend hint, so a wait notices another role's (or an
// earlier launch's) error within ~4 ms: after a give-up, the remaining launches of a step drain
// in milliseconds each instead of stalling the stream for minutes.
constexpr uint32_t kWaitCheckMask = 7u;

// Waits for the phase with the given parity to complete. Gives up (false) after limit_ns —
// recording `code` in *err — or as soon as another role has raised the error flag.
__device__ __forceinline__ bool mbar_wait_for(uint64_t* bar, uint32_t parity, int* err, int code,
                                              uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const WaitClock clk;
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & kWaitCheckMask) == 0) {
      if (*reinterpret_cast<volatile int*>(err) != 0) return false;
      if (clk.expired(limit_ns)) {
        raise_error(err, code);
        return false;
      }
    }
  }
}

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int code) {
  return mbar_wait_for(bar, parity, err, code, kWaitLimitNs);
}

// Bounded wait that only reports (used while draining after an error).
__device__ __forceinline__ bool mbar_wait_quiet(uint64_t* bar, uint32_t parity) {
  const WaitClock clk;
  while (!mbar_try_wait(bar, parity))
    if (clk.expired(kWaitLimitNs / 16)) return false;
  return true;
}

// Counts `bytes` of a phase's expected transaction bytes as arrived without a copy (the error
// path of the 2-SM kernel: the bytes of loads its partner never issued).
__device__ __forceinline__ void mbar_complete_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.complete_tx.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool failed(int* err) {
  return *reinterpret_cast<volatile int*>(err) != 0;
}

// ------------------------------------------------------------------------------------------
// TMA (no multicast: every CTA loads its own tiles from this GPU's memory)

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// Shared -> global tile store (bulk-group completion), its commit and the waits on it. The waits
// are hardware waits on this thread's own bulk copies, which always complete.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(src)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// every committed store of this thread has finished reading shared memory
__device__ __forceinline__ void bulk_wait_read_all() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

// every committed store of this thread but the newest one has finished reading shared memory
__device__ __forceinline__ void bulk_wait_read_newest_pending() {
  asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}

// every committed store of this thread has completed
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Generic-proxy shared-memory writes (st.shared) -> visible to the async proxy (tcgen05.mma).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ------------------------------------------------------------------------------------------
// tcgen05

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void fence_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, bf16 inputs, fp32 accumulate; one thread issues.
__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives on `bar` once every MMA this thread issued before has completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// 32 lanes x 32 columns of fp32: this thread gets its lane's 32 consecutive columns. The load is
// warp-collective (.sync.aligned): the warp is reconverged first, so a lane-dependent `continue`
// in a caller's previous loop iteration cannot leave it split at the instruction.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  __syncwarp();
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// ------------------------------------------------------------------------------------------
// CTA pairs (cluster of 2) for the 2-SM MMA: the even CTA ("leader") issues the MMAs for both;
// the other CTA's TMA loads complete on the leader's barriers (shared::cluster addresses), and the
// leader's MMA completions arrive on the barriers of both CTAs. No load multicasts: every CTA
// loads its own tiles from this GPU's memory.

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// shared::cluster address of the same shared variable in CTA `rank` of this cluster
__device__ __forceinline__ uint32_t mapa(const void* p, uint32_t rank) {
  uint32_t a;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_u32(p)), "r"(rank));
  return a;
}

__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}

// 32-bit store into a shared variable of another CTA of the cluster (a mapa address).
__device__ __forceinline__ void st_cluster_u32(uint32_t cluster_addr, uint32_t v) {
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(cluster_addr), "r"(v) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx_cluster(uint32_t cluster_addr, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cluster.shared::cluster.b64 _, [%0], %1;" ::"r"(
                   cluster_addr),
               "r"(bytes)
               : "memory");
}

// try_wait that also acquires what the other CTA of the pair released before arriving
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(500000u)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, int* err,
                                                  int code) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const WaitClock clk;
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if ((i & kWaitCheckMask) == 0) {
      if (*reinterpret_cast<volatile int*>(err) != 0) return false;
      if (clk.expired(kWaitLimitNs)) {
        raise_error(err, code);
        return false;
      }
    }
  }
}

// Bounded wait that does not look at the error flag (the error path, and the pair's teardown
// handshake, which must be waited out whether or not a wait gave up).
__device__ __forceinline__ bool mbar_wait_cluster_quiet(uint64_t* bar, uint32_t parity,
                                                        uint64_t limit_ns = kWaitLimitNs / 16) {
  const WaitClock clk;
  while (!mbar_try_wait_cluster(bar, parity))
    if (clk.expired(limit_ns)) return false;
  return true;
}

// Tile load into this CTA's shared memory whose completion is counted on the pair leader's
// mbarrier (bar_cluster = mapa(bar, 0)). No multicast.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map,
                                                 uint32_t bar_cluster, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y)
      : "memory");
}

// D (M = 256 over the pair, 128 TMEM lanes in each CTA) (+)= A * B^T; issued by the leader.
__device__ __forceinline__ void mma_bf16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                              uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on the barrier at the same shared-memory offset in both CTAs of the pair once the pair
// MMAs this thread issued so far complete: one commit signals both (an mbarrier arrive; no data
// moves). Two separate commits, one per CTA, measured at half the pair's MMA throughput.
__device__ __forceinline__ void mma_commit_pair_both(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 "
      "[%0], %1;" ::"r"(smem_u32(bar)),
      "h"(static_cast<uint16_t>(0x3))
      : "memory");
}

// Arrive on one barrier (shared::cluster address) once the pair MMAs issued so far complete.
__device__ __forceinline__ void mma_commit_pair_to(uint32_t bar_cluster) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar_cluster)
               : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" :::
                   "memory");
}

// Shared-memory matrix descriptor, 128-byte swizzle (layout type 2), sm_100 version bit.
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

// Instruction descriptor of kind::f16 with bf16 A and B, fp32 accumulator.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, bool a_mn_major,
                                                  bool b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(a_mn_major) << 15) |
         (static_cast<uint32_t>(b_mn_major) << 16) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(M >> 4) << 24);
}

}  // namespace tc

// ---------------------------------------------------------------------------------------------
// host side

namespace tc_host {

// Encodes a 2-D tensor map (inner dimension first) through the driver entry point, so the
// library needs no link-time dependency on libcuda. Returns 0 on success.
int encode_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t inner,
              uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
              CUtensorMapSwizzle swizzle);

// SM count of the current device (cached).
int sm_count();

// Raises `kernel`'s dynamic shared-memory limit to `bytes` once per kernel and driver context
// (a function attribute belongs to the context: after cudaDeviceReset the new context needs it
// again). Thread-safe. Returns 0 or the library's error status.
int ensure_smem(const void* kernel, int bytes, const char* what);

// Per-device error flag the tensor-core kernels raise when a bounded wait gives up (word 0 of
// the device's tc::ErrBlock).
int* device_error_flag();
// Reads and clears the current device's flag (synchronises the stream).
int take_device_error(cudaStream_t stream);
// The control block of one tensor-core launch on the current device: the error flag and the
// launch monitor's trace, with the next launch sequence number, recorded under `what`.
int launch_ctl(tc::Ctl* ctl, const char* what);

}  // namespace tc_host
