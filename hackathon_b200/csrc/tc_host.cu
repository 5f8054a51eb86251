// Host-side helpers of the tensor-core kernels: tensor-map encoding through the driver entry
// point, SM count, and the per-device error flag the bounded waits raise.
#include <cstddef>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <set>
#include <utility>

#include "qb_common.cuh"
#include "tc_common.cuh"

// Raised (non-zero) by a tensor-core kernel whose bounded wait gave up; the value says which
// wait. Static device memory: nothing is allocated for it. Its `host` member is set once per
// context to the mapped host record of the launch monitor.
static __device__ tc::ErrBlock g_tc_error;

namespace tc_host {

namespace {
using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                              const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                              const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                              CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
using CtxFn = CUresult (*)(CUcontext*);

constexpr int kMaxDev = 64;
constexpr int kNames = 4096;   // the last launches' names, by sequence number

// The launch monitor of one device: pinned host memory mapped into the device. The kernels write
// it (the error site of a wait that gives up; per CTA index the launch it started or finished),
// a host thread reads it with plain loads: no CUDA call, so it answers while the device is stuck.
struct MonitorPage {
  uint32_t err[4];   // site, CTA, SM of the wait that last raised the flag (site 0: none yet)
  uint32_t trace[tc::kTraceSlots];  // 2 * seq begun, 2 * seq + 1 finished (seq 0: never)
};

struct DeviceState {
  CUcontext ctx = nullptr;          // the context the addresses below belong to
  int* err = nullptr;               // device address of g_tc_error
  MonitorPage* page = nullptr;      // host address of the monitor
  uint32_t* trace_dev = nullptr;    // device address of page->trace
  uint32_t seq = 0;                 // last launch sequence number given out
  const char* names[kNames] = {};
};

std::mutex g_mu;
EncodeFn g_encode = nullptr;
CtxFn g_ctx_get = nullptr;
int g_sms[kMaxDev] = {};
DeviceState g_dev[kMaxDev];

int current_device() {
  int d = 0;
  cudaGetDevice(&d);
  return d;
}

// The calling thread's current driver context (null when none is current).
CUcontext current_context() {
  if (!g_ctx_get) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_ctx_get = reinterpret_cast<CtxFn>(fn);
  }
  CUcontext c = nullptr;
  if (g_ctx_get) g_ctx_get(&c);
  return c;
}

// Makes the runtime's current device's primary context current on this thread, once per thread
// and device (threads the caller's runtime never made a context current on - autograd's backward
// worker of device 0, for one - need it for the driver calls below).
void ensure_context(int d) {
  thread_local int ready = -1;
  if (ready != d) {
    cudaFree(nullptr);
    ready = d;
  }
}

// Sets up (once per context) the flag's address and the launch monitor of device d; g_mu held.
// A context created anew (after cudaDeviceReset, say) gets everything looked up again.
DeviceState* state_locked(int d) {
  ensure_context(d);
  DeviceState& st = g_dev[d];
  const CUcontext ctx = current_context();
  if (st.err && st.ctx == ctx) return &st;
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_tc_error) != cudaSuccess) return nullptr;
  st.err = static_cast<int*>(p);
  st.ctx = ctx;
  st.page = nullptr;
  st.trace_dev = nullptr;
  // The monitor is optional: without it the kernels run the same, only the host-side report
  // has nothing to read. Its pinned page is kept until exit (one per context).
  void* h = nullptr;
  void* dp = nullptr;
  bool ok = cudaHostAlloc(&h, sizeof(MonitorPage), cudaHostAllocMapped | cudaHostAllocPortable) ==
            cudaSuccess;
  if (ok) {
    memset(h, 0, sizeof(MonitorPage));
    ok = cudaHostGetDevicePointer(&dp, h, 0) == cudaSuccess;
  }
  if (ok) {
    // the device block's `host` member: set once, before this context's first launch
    int* rec = reinterpret_cast<int*>(static_cast<MonitorPage*>(dp)->err);
    ok = cudaMemcpy(reinterpret_cast<char*>(p) + offsetof(tc::ErrBlock, host), &rec, sizeof(rec),
                    cudaMemcpyHostToDevice) == cudaSuccess;
  }
  if (ok) {
    st.page = static_cast<MonitorPage*>(h);
    st.trace_dev = static_cast<MonitorPage*>(dp)->trace;
  } else {
    if (h) cudaFreeHost(h);
    cudaGetLastError();   // a monitor that could not be set up is no error of the next launch
  }
  return &st;
}
}  // namespace

void* current_context_handle() {
  std::lock_guard<std::mutex> lock(g_mu);
  ensure_context(current_device());
  return current_context();
}

int encode_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t inner,
              uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
              CUtensorMapSwizzle swizzle) {
  // The encoder is a driver call and needs a current context on this thread.
  ensure_context(current_device());
  {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_encode) {
      void* fn = nullptr;
      cudaDriverEntryPointQueryResult q;
      cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
      if (e != cudaSuccess || !fn || q != cudaDriverEntryPointSuccess)
        return qb::fail(QB_ERR_CUDA, "cuTensorMapEncodeTiled unavailable: %s", cudaGetErrorString(e));
      g_encode = reinterpret_cast<EncodeFn>(fn);
    }
  }
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0)
    return qb::fail(QB_ERR_INVALID, "tensor map: base address not 16-byte aligned");
  if ((row_stride_bytes & 15u) != 0 || row_stride_bytes == 0)
    return qb::fail(QB_ERR_INVALID, "tensor map: row stride %llu bytes not a positive multiple of 16",
                    (unsigned long long)row_stride_bytes);
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return qb::fail(QB_ERR_INVALID, "cuTensorMapEncodeTiled failed (%d): dims %llu x %llu, box %u x %u",
                    (int)r, (unsigned long long)inner, (unsigned long long)outer, box_inner, box_outer);
  return QB_OK;
}

int ensure_smem(const void* kernel, int bytes, const char* what) {
  static std::mutex mu;
  static std::set<std::pair<const void*, void*>> done;   // (kernel, context) already raised
  const auto key = std::make_pair(kernel, current_context_handle());
  std::lock_guard<std::mutex> lock(mu);
  if (done.count(key)) return QB_OK;
  const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             bytes);
  if (e != cudaSuccess)
    return qb::fail(QB_ERR_CUDA, "%s: smem attribute: %s", what, cudaGetErrorString(e));
  done.insert(key);
  return QB_OK;
}

int sm_count() {
  const int d = current_device();
  if (d < 0 || d >= kMaxDev) return 148;
  if (!g_sms[d]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, d);
    g_sms[d] = n > 0 ? n : 148;
  }
  return g_sms[d];
}

int* device_error_flag() {
  const int d = current_device();
  if (d < 0 || d >= kMaxDev) return nullptr;
  std::lock_guard<std::mutex> lock(g_mu);
  DeviceState* st = state_locked(d);
  return st ? st->err : nullptr;
}

int launch_ctl(tc::Ctl* ctl, const char* what) {
  const int d = current_device();
  if (d < 0 || d >= kMaxDev) return qb::fail(QB_ERR_UNSUPPORTED, "%s: device %d", what, d);
  std::lock_guard<std::mutex> lock(g_mu);
  DeviceState* st = state_locked(d);
  if (!st) return qb::fail(QB_ERR_CUDA, "%s: no device error flag", what);
  if (++st->seq >= 0x7fffffffu) st->seq = 1;
  st->names[st->seq % kNames] = what;
  ctl->err = st->err;
  ctl->trace = st->trace_dev;
  ctl->seq = st->seq;
  return QB_OK;
}

int take_device_error(cudaStream_t stream) {
  int* flag = device_error_flag();
  if (!flag) return -1;
  int v = 0;
  if (cudaMemcpyAsync(&v, flag, sizeof(int), cudaMemcpyDeviceToHost, stream) != cudaSuccess) return -1;
  if (cudaStreamSynchronize(stream) != cudaSuccess) return -1;
  if (v) {
    const int zero = 0;
    cudaMemcpyAsync(flag, &zero, sizeof(int), cudaMemcpyHostToDevice, stream);
    cudaStreamSynchronize(stream);
  }
  return v;
}

// Text report of device d's launch monitor from host memory alone (see qb_monitor_report).
int monitor_report(int d, char* buf, int64_t len) {
  if (!buf || len <= 0) return qb::fail(QB_ERR_INVALID, "monitor_report: no buffer");
  buf[0] = 0;
  if (d < 0 || d >= kMaxDev) return qb::fail(QB_ERR_INVALID, "monitor_report: device %d", d);
  // no lock: the watchdog calls this while another thread may be stuck holding nothing but a
  // CUDA call; the fields read here are written once (page) or are single words (seq, names)
  const DeviceState& st = g_dev[d];
  const volatile MonitorPage* pg = st.page;
  if (!pg) {
    snprintf(buf, static_cast<size_t>(len), "no launch monitor on device %d", d);
    return QB_OK;
  }
  const uint32_t last = st.seq;
  auto name = [&](uint32_t q) -> const char* {
    if (q == 0 || q > last || last - q >= static_cast<uint32_t>(kNames)) return "?";
    const char* n = st.names[q % kNames];
    return n ? n : "?";
  };
  // unfinished CTAs grouped by launch (few distinct launches: a handful of groups)
  uint32_t useq[8] = {}, ucnt[8] = {}, ufirst[8] = {};
  int ngroups = 0, unfinished = 0;
  uint32_t max_done = 0, max_begun = 0;
  for (int b = 0; b < tc::kTraceSlots; ++b) {
    const uint32_t v = pg->trace[b];
    if (v == 0) continue;
    const uint32_t q = v >> 1;
    if (v & 1u) {
      if (q > max_done) max_done = q;
      continue;
    }
    if (q > max_begun) max_begun = q;
    ++unfinished;
    int g = 0;
    while (g < ngroups && useq[g] != q) ++g;
    if (g == ngroups && ngroups < 8) { useq[g] = q; ufirst[g] = b; ++ngroups; }
    if (g < ngroups) ++ucnt[g];
  }
  int n = snprintf(buf, static_cast<size_t>(len),
                   "launches issued: %u (last %s); finished through #%u (%s); ", last, name(last),
                   max_done, name(max_done));
  const uint32_t site = pg->err[0];
  if (n < len) {
    if (site)
      n += snprintf(buf + n, static_cast<size_t>(len - n),
                    "last wait that gave up: site %u, CTA %u, SM %u; ", site, pg->err[1],
                    pg->err[2]);
    else
      n += snprintf(buf + n, static_cast<size_t>(len - n), "no wait has given up; ");
  }
  if (n < len) {
    if (unfinished == 0)
      n += snprintf(buf + n, static_cast<size_t>(len - n), "no CTA of these launches is running");
    else
      n += snprintf(buf + n, static_cast<size_t>(len - n), "%d CTA(s) started but not finished:",
                    unfinished);
  }
  for (int g = 0; g < ngroups && n < len; ++g)
    n += snprintf(buf + n, static_cast<size_t>(len - n), " #%u %s x%u (first CTA %u)", useq[g],
                  name(useq[g]), ucnt[g], ufirst[g]);
  return QB_OK;
}

}  // namespace tc_host

namespace {

constexpr int kProbeSite = 99;

// One thread waits on an mbarrier that nothing ever arrives on: the bounded wait gives up after
// limit_ns and records its site in the error flag, exactly as a stuck tensor-core kernel would.
__global__ void bounded_wait_probe(const tc::Ctl ctl, uint64_t limit_ns) {
  __shared__ uint64_t bar;
  tc::trace_begin(ctl);
  if (threadIdx.x == 0) {
    tc::mbar_init(&bar, 1);
    tc::fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    tc::mbar_wait_for(&bar, 0, ctl.err, kProbeSite, limit_ns);
    tc::trace_end(ctl);
  }
}

}  // namespace

extern "C" int qb_selftest_bounded_wait(int64_t limit_ns, cudaStream_t stream) {
  if (limit_ns < 1000000 || limit_ns > 2000000000)
    return qb::fail(QB_ERR_INVALID, "selftest_bounded_wait: limit must be 1 ms .. 2 s");
  tc::Ctl ctl;
  if (int s = tc_host::launch_ctl(&ctl, "selftest_bounded_wait")) return s;
  bounded_wait_probe<<<1, 32, 0, stream>>>(ctl, static_cast<uint64_t>(limit_ns));
  return qb::check_launch("selftest_bounded_wait");
}

extern "C" int qb_monitor_report(int device, char* buf, int64_t len) {
  return tc_host::monitor_report(device, buf, len);
}

extern "C" int qb_device_error(cudaStream_t stream) {
  const int v = tc_host::take_device_error(stream);
  if (v < 0) return qb::fail(QB_ERR_CUDA, "could not read the device error flag");
  if (v > 0) return qb::fail(QB_ERR_TIMEOUT, "a tensor-core kernel gave up a bounded wait (site %d)", v);
  return QB_OK;
}
