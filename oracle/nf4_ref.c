/* NF4 + double-quant dequantisation in plain C — TEST INFRASTRUCTURE ONLY (the CPU baseline of
 * the standalone dequant sweep and a second checker beside oracle/nf4_ref.py).
 *
 * Follows solution/nf4.py:25-49: scale = code2[q] * absmax2[blk / blocksize2] (rounded), then
 * + offset (rounded; built with -ffp-contract=off so no fused multiply-add), w = lut[nibble] *
 * scale, rounded to nearest even into bf16. Byte i holds weights 2i (high nibble), 2i+1.
 * `threads` POSIX threads split the bytes into contiguous ranges.
 */
#include <pthread.h>
#include <stdint.h>
#include <string.h>

static inline uint16_t f32_to_bf16_rne(float f) {
  uint32_t b;
  memcpy(&b, &f, 4);
  if ((b & 0x7f800000u) == 0x7f800000u && (b & 0x007fffffu)) return 0x7fc0; /* NaN */
  b += 0x7fffu + ((b >> 16) & 1u);
  return (uint16_t)(b >> 16);
}

typedef struct {
  const uint8_t* packed;
  const uint8_t* absmax_q;
  const float* code2;
  const float* absmax2;
  const float* lut16;
  uint16_t* out;
  float offset;
  int blocksize, blocksize2;
  int64_t lo, hi; /* byte range */
} job_t;

static void* run(void* arg) {
  const job_t* j = (const job_t*)arg;
  for (int64_t i = j->lo; i < j->hi; ++i) {
    const int64_t blk = (2 * i) / j->blocksize;
    const float s = j->code2[j->absmax_q[blk]] * j->absmax2[blk / j->blocksize2];
    const float scale = s + j->offset;
    const uint8_t byte = j->packed[i];
    j->out[2 * i] = f32_to_bf16_rne(j->lut16[byte >> 4] * scale);
    j->out[2 * i + 1] = f32_to_bf16_rne(j->lut16[byte & 15] * scale);
  }
  return 0;
}

/* out: n_weights bf16 bit patterns. Returns 0, or -1 on a bad argument. */
int nf4_dequant_bf16(const uint8_t* packed, int64_t n_weights, const uint8_t* absmax_q,
                     const float* code2, const float* absmax2, float offset, int blocksize,
                     int blocksize2, const float* lut16, uint16_t* out, int threads) {
  if (n_weights < 0 || n_weights % 2 || blocksize <= 0 || blocksize % 2 || blocksize2 <= 0)
    return -1;
  if (threads < 1) threads = 1;
  if (threads > 256) threads = 256;
  const int64_t n_bytes = n_weights / 2;
  job_t jobs[256];
  pthread_t tid[256];
  for (int t = 0; t < threads; ++t) {
    job_t j = {packed, absmax_q, code2, absmax2, lut16, out, offset, blocksize, blocksize2,
               n_bytes * t / threads, n_bytes * (t + 1) / threads};
    jobs[t] = j;
  }
  for (int t = 1; t < threads; ++t) pthread_create(&tid[t], 0, run, &jobs[t]);
  run(&jobs[0]);
  for (int t = 1; t < threads; ++t) pthread_join(tid[t], 0);
  return 0;
}
