// Host-side helpers of the tensor-core kernels: tensor-map encoding through the driver entry
// point, SM count, and the per-device error flag the bounded waits raise.
#include <mutex>

#include "qb_common.cuh"
#include "tc_common.cuh"

// Raised (non-zero) by a tensor-core kernel whose bounded wait gave up; the value says which
// wait. Static device memory: nothing is allocated for it.
static __device__ int g_tc_error;

namespace tc_host {

namespace {
using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                              const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                              const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                              CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
std::mutex g_mu;
EncodeFn g_encode = nullptr;
int g_sms[64] = {};
int* g_err_addr[64] = {};

int current_device() {
  int d = 0;
  cudaGetDevice(&d);
  return d;
}
}  // namespace

int encode_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t inner,
              uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
              CUtensorMapSwizzle swizzle) {
  // The encoder is a driver call and needs a current context on this thread. Threads the
  // caller's runtime never made a context current on (autograd's backward worker of device 0,
  // for one) get the runtime's current device's primary context here.
  cudaFree(nullptr);
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

int sm_count() {
  const int d = current_device();
  if (d < 0 || d >= 64) return 148;
  if (!g_sms[d]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, d);
    g_sms[d] = n > 0 ? n : 148;
  }
  return g_sms[d];
}

int* device_error_flag() {
  const int d = current_device();
  if (d < 0 || d >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_err_addr[d]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_tc_error) != cudaSuccess) return nullptr;
    g_err_addr[d] = static_cast<int*>(p);
  }
  return g_err_addr[d];
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

}  // namespace tc_host

namespace {

constexpr int kProbeSite = 99;

// One thread waits on an mbarrier that nothing ever arrives on: the bounded wait gives up after
// limit_ns and records its site in the error flag, exactly as a stuck tensor-core kernel would.
__global__ void bounded_wait_probe(int* err, uint64_t limit_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    tc::mbar_init(&bar, 1);
    tc::fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) tc::mbar_wait_for(&bar, 0, err, kProbeSite, limit_ns);
}

}  // namespace

extern "C" int qb_selftest_bounded_wait(int64_t limit_ns, cudaStream_t stream) {
  if (limit_ns < 1000000 || limit_ns > 2000000000)
    return qb::fail(QB_ERR_INVALID, "selftest_bounded_wait: limit must be 1 ms .. 2 s");
  int* err = tc_host::device_error_flag();
  if (!err) return qb::fail(QB_ERR_CUDA, "selftest_bounded_wait: no device error flag");
  bounded_wait_probe<<<1, 32, 0, stream>>>(err, static_cast<uint64_t>(limit_ns));
  return qb::check_launch("selftest_bounded_wait");
}

extern "C" int qb_device_error(cudaStream_t stream) {
  const int v = tc_host::take_device_error(stream);
  if (v < 0) return qb::fail(QB_ERR_CUDA, "could not read the device error flag");
  if (v > 0) return qb::fail(QB_ERR_TIMEOUT, "a tensor-core kernel gave up a bounded wait (site %d)", v);
  return QB_OK;
}
