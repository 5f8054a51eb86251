// NF4 + double-quant dequantisation (standalone, HBM-bound) and the NF4 quantiser that produces
// the format.
//
// Dequant data flow per weight (bit-exact with solution/nf4.py:25-49 on the GPU):
//   scale = code2[absmax_q[blk]] * absmax2[blk / blocksize2]   (fp32, rounded)
//   scale = scale + offset                                     (fp32, rounded; never an FMA)
//   w     = lut16[nibble] * scale                              (fp32, rounded)
//   out   = round_to_nearest_even(w) in the output dtype
// Byte i holds weights 2i (high nibble) and 2i+1 (low nibble); blk = weight_index / blocksize.
//
// The fast path gives each thread one 4-byte word (8 weights) per step, so a warp reads 128
// contiguous bytes and writes 512 (bf16/fp16) or 1024 (fp32) contiguous bytes per step: every
// load and store instruction is fully coalesced; the lookup tables sit in shared memory.
#include <mutex>

#include "qb_common.cuh"

namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 4;  // words per thread per CTA

// SHIFT: the block sizes are powers of two and indices divide by shifting (bs2_shift =
// log2(blocksize2)); a 64-bit division costs more than the dequantisation of a word.
template <bool NESTED, bool SHIFT>
__device__ __forceinline__ float block_scale(int64_t blk, const void* absmax, const float* s_code2,
                                             const float* absmax2, float offset, int blocksize2,
                                             int bs2_shift) {
  if (NESTED) {
    const uint8_t q = static_cast<const uint8_t*>(absmax)[blk];
    const float a2 = __ldg(absmax2 + (SHIFT ? blk >> bs2_shift : blk / blocksize2));
    return __fadd_rn(__fmul_rn(s_code2[q], a2), offset);
  }
  return __ldg(static_cast<const float*>(absmax) + blk);
}

// One word = 4 packed bytes = 8 weights that share one scale block (blocksize % 8 == 0);
// wpb_shift = log2(blocksize / 8) when SHIFT.
template <typename OutT, bool NESTED, bool SHIFT>
__global__ void __launch_bounds__(kThreads)
nf4_dequant_word_kernel(const uint32_t* __restrict__ packed, int64_t n_words,
                        const void* __restrict__ absmax, const float* __restrict__ code2,
                        const float* __restrict__ absmax2, float offset, int blocksize,
                        int blocksize2, int wpb_shift, int bs2_shift,
                        const float* __restrict__ lut16, OutT* __restrict__ out) {
  __shared__ float s_lut[16];
  __shared__ float s_code2[NESTED ? 256 : 1];
  if (threadIdx.x < 16) s_lut[threadIdx.x] = lut16[threadIdx.x];
  if (NESTED) s_code2[threadIdx.x] = code2[threadIdx.x];  // kThreads == 256
  __syncthreads();

  const int words_per_block = blocksize / 8;
  const int64_t base = static_cast<int64_t>(blockIdx.x) * (kThreads * kUnroll) + threadIdx.x;
  uint32_t word[kUnroll];
#pragma unroll
  for (int u = 0; u < kUnroll; ++u) {
    const int64_t i = base + u * kThreads;
    word[u] = i < n_words ? __ldcs(packed + i) : 0u;  // streamed: read once
  }
#pragma unroll
  for (int u = 0; u < kUnroll; ++u) {
    const int64_t i = base + u * kThreads;
    if (i >= n_words) break;
    const int64_t blk = SHIFT ? i >> wpb_shift : i / words_per_block;
    const float scale = block_scale<NESTED, SHIFT>(blk, absmax, s_code2, absmax2, offset,
                                                   blocksize2, bs2_shift);
    float w[8];
    const uint32_t x = word[u];
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const uint32_t byte = (x >> (8 * b)) & 0xffu;  // little endian: byte b of the word
      w[2 * b] = __fmul_rn(s_lut[byte >> 4], scale);
      w[2 * b + 1] = __fmul_rn(s_lut[byte & 15u], scale);
    }
    qb::store8<OutT>(out + i * 8, w);
  }
}

// Any even blocksize, any length: one byte (two weights) per thread.
template <typename OutT, bool NESTED>
__global__ void __launch_bounds__(kThreads)
nf4_dequant_byte_kernel(const uint8_t* __restrict__ packed, int64_t n_bytes,
                        const void* __restrict__ absmax, const float* __restrict__ code2,
                        const float* __restrict__ absmax2, float offset, int blocksize,
                        int blocksize2, const float* __restrict__ lut16, OutT* __restrict__ out) {
  __shared__ float s_lut[16];
  __shared__ float s_code2[NESTED ? 256 : 1];
  if (threadIdx.x < 16) s_lut[threadIdx.x] = lut16[threadIdx.x];
  if (NESTED) s_code2[threadIdx.x] = code2[threadIdx.x];
  __syncthreads();
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; i < n_bytes;
       i += static_cast<int64_t>(gridDim.x) * kThreads) {
    const uint32_t byte = packed[i];
    const int64_t blk = (2 * i) / blocksize;
    const float scale = block_scale<NESTED, false>(blk, absmax, s_code2, absmax2, offset,
                                                   blocksize2, 0);
    out[2 * i] = qb::from_f<OutT>(__fmul_rn(s_lut[byte >> 4], scale));
    out[2 * i + 1] = qb::from_f<OutT>(__fmul_rn(s_lut[byte & 15u], scale));
  }
}

template <typename OutT, bool NESTED>
int launch_dequant(const uint8_t* packed, int64_t n_weights, const void* absmax,
                   const float* code2, const float* absmax2, float offset, int blocksize,
                   int blocksize2, const float* lut16, OutT* out, cudaStream_t stream) {
  const int64_t n_bytes = n_weights / 2;
  const bool word_path = blocksize % 8 == 0 && n_bytes % 4 == 0 &&
                         (reinterpret_cast<uintptr_t>(packed) & 3u) == 0 && qb::aligned16(out);
  if (word_path) {
    const int64_t n_words = n_bytes / 4;
    const int64_t grid = (n_words + kThreads * kUnroll - 1) / (kThreads * kUnroll);
    if (grid > 0x7fffffff) return qb::fail(QB_ERR_INVALID, "nf4_dequant: tensor too large");
    const int wpb = blocksize / 8;
    const bool pow2 = (wpb & (wpb - 1)) == 0 &&
                      (!NESTED || (blocksize2 > 0 && (blocksize2 & (blocksize2 - 1)) == 0));
    const int wpb_shift = __builtin_ctz(static_cast<unsigned>(wpb));
    const int bs2_shift = NESTED && blocksize2 > 0 ? __builtin_ctz(static_cast<unsigned>(blocksize2))
                                                   : 0;
    const auto* pw = reinterpret_cast<const uint32_t*>(packed);
    if (pow2)
      nf4_dequant_word_kernel<OutT, NESTED, true><<<static_cast<unsigned>(grid), kThreads, 0,
                                                    stream>>>(
          pw, n_words, absmax, code2, absmax2, offset, blocksize, blocksize2, wpb_shift,
          bs2_shift, lut16, out);
    else
      nf4_dequant_word_kernel<OutT, NESTED, false><<<static_cast<unsigned>(grid), kThreads, 0,
                                                     stream>>>(
          pw, n_words, absmax, code2, absmax2, offset, blocksize, blocksize2, 0, 0, lut16, out);
  } else {
    int64_t grid = (n_bytes + kThreads - 1) / kThreads;
    if (grid > 148 * 64) grid = 148 * 64;
    nf4_dequant_byte_kernel<OutT, NESTED><<<static_cast<unsigned>(grid), kThreads, 0, stream>>>(
        packed, n_bytes, absmax, code2, absmax2, offset, blocksize, blocksize2, lut16, out);
  }
  return qb::check_launch("nf4_dequant");
}

// ---------------------------------------------------------------------------------------------
// quantiser: one warp per scale block

template <typename InT>
__global__ void nf4_quantize_kernel(const InT* __restrict__ w, int64_t n_weights, int blocksize,
                                    const float* __restrict__ lut16, uint8_t* __restrict__ packed,
                                    float* __restrict__ absmax, int64_t n_blocks) {
  __shared__ float s_lut[16];
  if (threadIdx.x < 16) s_lut[threadIdx.x] = lut16[threadIdx.x];
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t blk = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (blk >= n_blocks) return;
  const int64_t start = blk * blocksize;
  int64_t stop = start + blocksize;
  if (stop > n_weights) stop = n_weights;
  float amax = 0.f;
  for (int64_t i = start + lane; i < stop; i += 32) amax = fmaxf(amax, fabsf(qb::to_f(w[i])));
  amax = qb::warp_max(amax);
  if (lane == 0) absmax[blk] = amax;
  const float inv = amax > 0.f ? 1.f / amax : 0.f;
  // pairs of weights -> one byte, high nibble first
  for (int64_t p = start / 2 + lane; p < (stop + 1) / 2; p += 32) {
    uint32_t byte = 0;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int64_t i = 2 * p + h;
      const float v = i < stop ? qb::to_f(w[i]) * inv : 0.f;
      int best = 0;
      float best_d = fabsf(v - s_lut[0]);
#pragma unroll
      for (int c = 1; c < 16; ++c) {
        const float d = fabsf(v - s_lut[c]);
        if (d < best_d) { best_d = d; best = c; }
      }
      byte |= static_cast<uint32_t>(best) << (h == 0 ? 4 : 0);
    }
    packed[p] = static_cast<uint8_t>(byte);
  }
}

// double quant, stage 1: per-CTA partial sums in double (fixed order -> deterministic)
constexpr int kPartials = 1024;

__global__ void dq_partial_sum_kernel(const float* __restrict__ a, int64_t n,
                                      double* __restrict__ partial) {
  __shared__ double s[kThreads];
  const int64_t per = (n + gridDim.x - 1) / gridDim.x;
  const int64_t lo = blockIdx.x * per;
  int64_t hi = lo + per;
  if (hi > n) hi = n;
  double acc = 0.0;
  for (int64_t i = lo + threadIdx.x; i < hi; i += kThreads) acc += a[i];
  s[threadIdx.x] = acc;
  __syncthreads();
  for (int o = kThreads / 2; o > 0; o >>= 1) {
    if (threadIdx.x < o) s[threadIdx.x] += s[threadIdx.x + o];
    __syncthreads();
  }
  if (threadIdx.x == 0) partial[blockIdx.x] = s[0];
}

__global__ void dq_mean_kernel(const double* __restrict__ partial, int n_partial, int64_t n,
                               float* __restrict__ offset) {
  if (threadIdx.x == 0) {
    double acc = 0.0;
    for (int i = 0; i < n_partial; ++i) acc += partial[i];
    *offset = static_cast<float>(acc / static_cast<double>(n));
  }
}

// stage 2: one CTA (256 threads) per block of up to 256 scales
__global__ void dq_quantize_kernel(const float* __restrict__ a, int64_t n, int blocksize2,
                                   const float* __restrict__ code2, const float* __restrict__ offset,
                                   uint8_t* __restrict__ q, float* __restrict__ absmax2) {
  __shared__ float s_code[256];
  __shared__ float s_red[32];
  s_code[threadIdx.x] = code2[threadIdx.x];
  const float off = *offset;
  const int64_t start = static_cast<int64_t>(blockIdx.x) * blocksize2;
  int64_t stop = start + blocksize2;
  if (stop > n) stop = n;
  float m = 0.f;
  for (int64_t i = start + threadIdx.x; i < stop; i += blockDim.x) m = fmaxf(m, fabsf(a[i] - off));
  m = qb::warp_max(m);
  if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? s_red[threadIdx.x] : 0.f;
    t = qb::warp_max(t);
    if (threadIdx.x == 0) s_red[0] = t;
  }
  __syncthreads();
  const float amax = s_red[0];
  if (threadIdx.x == 0) absmax2[blockIdx.x] = amax;
  const float inv = amax > 0.f ? 1.f / amax : 0.f;
  for (int64_t i = start + threadIdx.x; i < stop; i += blockDim.x) {
    const float v = (a[i] - off) * inv;
    int lo = 0, hi = 255;  // first index with code >= v
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if (s_code[mid] < v) lo = mid + 1; else hi = mid;
    }
    int best = lo;
    if (lo > 0 && fabsf(v - s_code[lo - 1]) <= fabsf(s_code[lo] - v)) best = lo - 1;
    q[i] = static_cast<uint8_t>(best);
  }
}

}  // namespace

extern "C" int qb_nf4_dequant(const uint8_t* packed, int64_t n_weights, const void* absmax,
                              int nested, const float* code2, const float* absmax2, float offset,
                              int blocksize, int blocksize2, const float* lut16, void* out,
                              int out_dtype, cudaStream_t stream) {
  if (n_weights < 0 || n_weights % 2) return qb::fail(QB_ERR_INVALID, "nf4_dequant: n_weights must be even and >= 0");
  if (blocksize <= 0 || blocksize % 2) return qb::fail(QB_ERR_INVALID, "nf4_dequant: blocksize must be even");
  if (nested && (blocksize2 <= 0 || blocksize2 % 2)) return qb::fail(QB_ERR_INVALID, "nf4_dequant: blocksize2 must be even");
  if (n_weights == 0) return QB_OK;
  if (!packed || !absmax || !lut16 || !out || (nested && (!code2 || !absmax2)))
    return qb::fail(QB_ERR_INVALID, "nf4_dequant: null pointer");
  QB_DISPATCH_FLOAT(out_dtype, T, {
    if (nested)
      return launch_dequant<T, true>(packed, n_weights, absmax, code2, absmax2, offset, blocksize,
                                     blocksize2, lut16, static_cast<T*>(out), stream);
    return launch_dequant<T, false>(packed, n_weights, absmax, code2, absmax2, offset, blocksize,
                                    1, lut16, static_cast<T*>(out), stream);
  });
}

extern "C" int qb_nf4_quantize(const void* w, int w_dtype, int64_t n_weights, int blocksize,
                               const float* lut16, uint8_t* packed, float* absmax,
                               cudaStream_t stream) {
  if (n_weights < 0 || n_weights % 2) return qb::fail(QB_ERR_INVALID, "nf4_quantize: n_weights must be even");
  if (blocksize <= 0 || blocksize % 2) return qb::fail(QB_ERR_INVALID, "nf4_quantize: blocksize must be even");
  if (n_weights == 0) return QB_OK;
  const int64_t n_blocks = (n_weights + blocksize - 1) / blocksize;
  const int warps = 8;
  const int64_t grid = (n_blocks + warps - 1) / warps;
  QB_DISPATCH_FLOAT(w_dtype, T, {
    nf4_quantize_kernel<T><<<static_cast<unsigned>(grid), warps * 32, 0, stream>>>(
        static_cast<const T*>(w), n_weights, blocksize, lut16, packed, absmax, n_blocks);
  });
  return qb::check_launch("nf4_quantize");
}

// ---------------------------------------------------------------------------------------------
// Double quant without any allocation, for callers that cannot allocate device memory.
//
// The partial sums live in this file-scope device array instead of a caller-provided workspace.
// Every GPU that loads the library holds these 4 KiB until the process exits. Host code must
// not pass `g_dq_scratch` to a kernel (on the host it names a stand-in, not device memory): the
// device address is looked up with cudaGetSymbolAddress on a device's first call and cached
// with the context it belongs to; a call under another context of that device (after
// cudaDeviceReset, which destroys the old one) looks it up again. The first call on a device
// makes that CUDA call, so it belongs before any stream capture. Every slot a
// call uses is written by its first kernel before its second kernel reads it, so nothing needs
// clearing between calls; calls whose kernels overlap on the GPU (different streams, or
// different host threads on one device) race on the array.
constexpr int kStaticPartials = 512;
static __device__ __align__(256) double g_dq_scratch[kStaticPartials];

namespace tc_host {
void* current_context_handle();   // tc_host.cu: this thread's current driver context
}

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_addr[kMaxDevices] = {};
void* g_scratch_ctx[kMaxDevices] = {};

int static_scratch(double** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return qb::fail(QB_ERR_CUDA, "nf4_double_quant_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return qb::fail(QB_ERR_UNSUPPORTED, "nf4_double_quant_noalloc: device %d", dev);
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  void* ctx = tc_host::current_context_handle();
  if (!g_scratch_addr[dev] || g_scratch_ctx[dev] != ctx) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_dq_scratch);
    if (e != cudaSuccess || !p)
      return qb::fail(QB_ERR_CUDA, "nf4_double_quant_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    g_scratch_addr[dev] = p;
    g_scratch_ctx[dev] = tc_host::current_context_handle();   // current now, if it was not
  }
  *out = static_cast<double*>(g_scratch_addr[dev]);
  return QB_OK;
}
}  // namespace

extern "C" int64_t qb_nf4_double_quant_noalloc_max_blocks(void) {
  return static_cast<int64_t>(kStaticPartials) * 4096;
}

extern "C" int qb_nf4_double_quant_noalloc(const float* absmax, int64_t n_blocks, int blocksize2,
                                           const float* code2, uint8_t* absmax_q, float* absmax2,
                                           float* offset_dev, cudaStream_t stream) {
  if (n_blocks <= 0) return qb::fail(QB_ERR_INVALID, "nf4_double_quant_noalloc: no blocks");
  if (blocksize2 <= 0 || blocksize2 % 2) return qb::fail(QB_ERR_INVALID, "nf4_double_quant_noalloc: blocksize2 must be even");
  const int64_t parts = (n_blocks + 4095) / 4096;  // the partition qb_nf4_double_quant uses
  if (parts > kStaticPartials)
    return qb::fail(QB_ERR_INVALID,
                    "nf4_double_quant_noalloc: %lld scale blocks exceed the static scratch "
                    "limit of %lld (use qb_nf4_double_quant with a workspace)",
                    (long long)n_blocks, (long long)kStaticPartials * 4096);
  double* partial = nullptr;
  if (int s = static_scratch(&partial)) return s;
  dq_partial_sum_kernel<<<static_cast<unsigned>(parts), kThreads, 0, stream>>>(absmax, n_blocks, partial);
  dq_mean_kernel<<<1, 32, 0, stream>>>(partial, static_cast<int>(parts), n_blocks, offset_dev);
  const int64_t grid = (n_blocks + blocksize2 - 1) / blocksize2;
  dq_quantize_kernel<<<static_cast<unsigned>(grid), 256, 0, stream>>>(
      absmax, n_blocks, blocksize2, code2, offset_dev, absmax_q, absmax2);
  return qb::check_launch("nf4_double_quant_noalloc");
}

extern "C" int64_t qb_nf4_double_quant_workspace(int64_t) {
  return static_cast<int64_t>(kPartials) * sizeof(double);
}

extern "C" int qb_nf4_double_quant(const float* absmax, int64_t n_blocks, int blocksize2,
                                   const float* code2, uint8_t* absmax_q, float* absmax2,
                                   float* offset_dev, void* workspace, cudaStream_t stream) {
  if (n_blocks <= 0) return qb::fail(QB_ERR_INVALID, "nf4_double_quant: no blocks");
  if (blocksize2 <= 0 || blocksize2 % 2) return qb::fail(QB_ERR_INVALID, "nf4_double_quant: blocksize2 must be even");
  if (!workspace) return qb::fail(QB_ERR_INVALID, "nf4_double_quant: workspace is required");
  auto* partial = static_cast<double*>(workspace);
  int parts = static_cast<int>((n_blocks + 4095) / 4096);
  if (parts > kPartials) parts = kPartials;
  if (parts < 1) parts = 1;
  dq_partial_sum_kernel<<<parts, kThreads, 0, stream>>>(absmax, n_blocks, partial);
  dq_mean_kernel<<<1, 32, 0, stream>>>(partial, parts, n_blocks, offset_dev);
  const int64_t grid = (n_blocks + blocksize2 - 1) / blocksize2;
  dq_quantize_kernel<<<static_cast<unsigned>(grid), 256, 0, stream>>>(
      absmax, n_blocks, blocksize2, code2, offset_dev, absmax_q, absmax2);
  return qb::check_launch("nf4_double_quant");
}
