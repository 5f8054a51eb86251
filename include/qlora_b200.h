/* qlora_b200 — C-ABI of the B200 (sm_100a) kernel suite for the Qwen2.5 QLoRA training step.
 *
 * Every entry point takes plain device pointers, element counts, strides in elements, dtype
 * tags and a cudaStream_t, launches on that stream and returns a status (QB_OK = 0). A nonzero
 * status leaves a message for qb_last_error() on the calling thread. The caller owns all memory;
 * no entry point allocates device memory except where its comment says so. No entry point
 * synchronises the stream.
 *
 * Each declaration names the reference function (imoshka2009-lab/hackathon, `solution/`) whose
 * kernel it replaces, by file:line.
 */
#ifndef QLORA_B200_H
#define QLORA_B200_H

#include <stdint.h>
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define QB_OK 0
#define QB_ERR_INVALID 1     /* bad argument: shape, stride, dtype, alignment, null pointer */
#define QB_ERR_CUDA 2        /* a CUDA call or launch failed */
#define QB_ERR_UNSUPPORTED 3 /* valid input this build has no kernel for */
#define QB_ERR_TIMEOUT 4     /* a bounded device-side wait gave up */

/* dtype tags (the same numbers as solution/_common.py:19-25 round_mode) */
#define QB_F32 0
#define QB_F16 1
#define QB_BF16 2

/* Message of the last failed call on this thread ("" if none). */
const char* qb_last_error(void);
/* Version of this ABI; bumped when a signature changes. */
int qb_abi_version(void);

/* ---------------------------------------------------------------------------------------------
 * NF4 with double-quantised absmax (bitsandbytes layout)
 */

/* Dequantise n_weights NF4 weights into `out` (out_dtype F32/F16/BF16).
 * Replaces solution/nf4.py:25-49 (nf4_dequant_kernel) and :71-92 (dequantize_nf4).
 * packed: n_weights/2 bytes, weight 2i in the high nibble of byte i, 2i+1 in the low nibble.
 * nested=1: absmax is uint8 [ceil(n/blocksize)] codes into code2[256] (fp32), second-level
 *   scales absmax2 fp32 [ceil(nblocks/blocksize2)] and the fp32 `offset`:
 *   scale = code2[absmax[b]] * absmax2[b / blocksize2] + offset   (a rounded multiply, then a
 *   rounded add: no fused multiply-add), w = lut16[nibble] * scale, then rounded to out_dtype.
 * nested=0: absmax is fp32 [nblocks]; code2, absmax2 and offset are ignored.
 * blocksize (and blocksize2 when nested) must be even; n_weights must be even. */
int qb_nf4_dequant(const uint8_t* packed, int64_t n_weights, const void* absmax, int nested,
                   const float* code2, const float* absmax2, float offset, int blocksize,
                   int blocksize2, const float* lut16, void* out, int out_dtype,
                   cudaStream_t stream);

/* First-level NF4 quantisation of w (w_dtype F32/F16/BF16, n_weights even): per block of
 * `blocksize` weights absmax[b] = max|w|, each weight -> index of the nearest lut16 entry to
 * w/absmax, packed two per byte (high nibble first). The input producer of the format
 * qb_nf4_dequant reads (bitsandbytes quantize_4bit, used at solution/test_kernels.py:48-49). */
int qb_nf4_quantize(const void* w, int w_dtype, int64_t n_weights, int blocksize,
                    const float* lut16, uint8_t* packed, float* absmax, cudaStream_t stream);

/* Second-level (double) quantisation of the fp32 block scales: offset = mean(absmax) (written
 * to *offset_dev), then per block of blocksize2 scales absmax2[j] = max|absmax - offset| and
 * absmax_q[b] = index of the code2 entry nearest to (absmax[b] - offset) / absmax2[j].
 * code2 must be sorted ascending. `workspace` is caller-owned device memory of
 * qb_nf4_double_quant_workspace(n_blocks) bytes. */
int64_t qb_nf4_double_quant_workspace(int64_t n_blocks);
int qb_nf4_double_quant(const float* absmax, int64_t n_blocks, int blocksize2,
                        const float* code2, uint8_t* absmax_q, float* absmax2,
                        float* offset_dev, void* workspace, cudaStream_t stream);

/* qb_nf4_double_quant for callers that cannot allocate device memory — code running where
 * cudaMalloc is off limits (inside a caching allocator's own hooks, a plugin host that owns all
 * device memory, a process that has pinned its memory budget). No counterpart in the reference.
 * Same arguments and results as qb_nf4_double_quant, minus the workspace: the partial sums go
 * to a 4 KiB array compiled into the library (static device memory every GPU that loads the
 * library keeps until exit), so n_blocks is limited to qb_nf4_double_quant_noalloc_max_blocks()
 * (2,097,152 scale blocks = 134M weights at blocksize 64); larger inputs return QB_ERR_INVALID.
 * The first call on a device looks up the array's device address (cudaGetSymbolAddress): make
 * that first call before any stream capture. Calls share the array, so calls that overlap on the
 * GPU race; each call writes every slot it reads, so nothing needs clearing. */
int64_t qb_nf4_double_quant_noalloc_max_blocks(void);
int qb_nf4_double_quant_noalloc(const float* absmax, int64_t n_blocks, int blocksize2,
                                const float* code2, uint8_t* absmax_q, float* absmax2,
                                float* offset_dev, cudaStream_t stream);

/* ---------------------------------------------------------------------------------------------
 * RMSNorm (Qwen2RMSNorm), frozen weight
 */

/* y = w * round_x(x * rstd), rstd = 1/sqrt(mean(x^2) + eps) per row, stored to rstd[rows].
 * round_x rounds through x's dtype when x is F16/BF16 (no-op for F32). Row strides in elements;
 * the last dimension is contiguous. Replaces solution/rmsnorm.py:25-39 (rmsnorm_fwd_kernel). */
int qb_rmsnorm_fwd(const void* x, int x_dtype, int64_t x_row_stride, const void* w, int w_dtype,
                   void* y, int y_dtype, int64_t y_row_stride, float* rstd, int64_t rows,
                   int64_t cols, float eps, cudaStream_t stream);

/* dx = rstd * (g - x * rstd^2 * mean(g * x)), g = dy * w. No weight gradient (frozen).
 * Replaces solution/rmsnorm.py:43-55 (rmsnorm_bwd_kernel). */
int qb_rmsnorm_bwd(const void* dy, int dy_dtype, int64_t dy_row_stride, const void* x,
                   int x_dtype, int64_t x_row_stride, const void* w, int w_dtype,
                   const float* rstd, void* dx, int dx_dtype, int64_t dx_row_stride,
                   int64_t rows, int64_t cols, cudaStream_t stream);

/* ---------------------------------------------------------------------------------------------
 * RoPE on q and k in one launch
 */

/* Rotate-half RoPE. q [B,HQ,S,D] and k [B,HK,S,D] with arbitrary element strides
 * (q_strides = {b,h,s}; the last dimension is contiguous), cos/sin [B or broadcast, S, D] with
 * strides cs_stride_b (0 to broadcast) and cs_stride_s. Halves (x1,x2), (c1,c2), (s1,s2):
 *   forward : o1 = x1*c1 - x2*s1, o2 = x2*c2 + x1*s2
 *   backward: d1 = g1*c1 + g2*s2, d2 = g2*c2 - g1*s1
 * q/k share in_dtype, q_out/k_out share out_dtype; cos and sin share cs_dtype.
 * Replaces solution/rope.py:25-62 (rope_qk_kernel) and :65-75 (_launch). */
int qb_rope_qk(const void* q, const void* k, void* q_out, void* k_out, const void* cos_,
               const void* sin_, int in_dtype, int out_dtype, int cs_dtype, int64_t B,
               int64_t HQ, int64_t HK, int64_t S, int64_t D, const int64_t* q_strides,
               const int64_t* k_strides, const int64_t* qo_strides, const int64_t* ko_strides,
               int64_t cs_stride_b, int64_t cs_stride_s, int backward, cudaStream_t stream);

/* ---------------------------------------------------------------------------------------------
 * SwiGLU
 */

/* out = silu(gate) * up over n contiguous elements (fp32 math).
 * Replaces solution/swiglu.py:15-22 (example_swiglu_fwd_kernel). */
int qb_swiglu_fwd(const void* gate, const void* up, void* out, int dtype, int64_t n,
                  cudaStream_t stream);
/* dup = g*silu(gate); dgate = g*up*sig*(1 + gate*(1-sig)).
 * Replaces solution/swiglu.py:25-37 (example_swiglu_bwd_kernel). */
int qb_swiglu_bwd(const void* grad, const void* gate, const void* up, void* dgate, void* dup,
                  int dtype, int64_t n, cudaStream_t stream);

/* ---------------------------------------------------------------------------------------------
 * LoRA dropout + cast, scaled add
 */

/* out[r,c] = in[r,c] * keep * scale, keep = (u > p) with u the Philox-4x32-10 uniform of
 * (seed, int32(r*cols + c)) — the stream of Triton's tl.rand, so masks match the reference
 * bit for bit. With p <= 0: out = in * scale (a cast when scale = 1).
 * Replaces solution/lora.py:29-46 (lora_dropout_scale_kernel) and :74-81 (_dropout_scale). */
int qb_dropout_scale(const void* in, int in_dtype, int64_t in_row_stride, void* out,
                     int out_dtype, int64_t out_row_stride, int64_t rows, int64_t cols,
                     uint64_t seed, float p, float scale, cudaStream_t stream);

/* qb_dropout_scale that also records its mask: bits[r * words + c / 32] bit (c % 32) =
 * keep(r, c), words = ceil(cols / 32) (the same Philox stream, so the same mask). The recorded
 * mask lets the checkpoint recompute and the backward skip the random numbers (a variant of
 * solution/lora.py:29-46, which regenerates the mask from the seed each time). */
int qb_dropout_mask(const void* in, int in_dtype, int64_t in_row_stride, void* out,
                    int out_dtype, int64_t out_row_stride, uint32_t* bits, int64_t rows,
                    int64_t cols, uint64_t seed, float p, float scale, cudaStream_t stream);

/* The mask of qb_dropout_mask alone, no data read or written: bits[r * words + c / 32] bit
 * (c % 32) = keep(r, c), words = ceil(cols / 32), bits past a row's end 0. The mask depends only
 * on (seed, r, c), so it can be drawn ahead of the activations it will mask, e.g. on a side
 * stream beside the tensor-core GEMMs (the Philox rounds are integer-pipe work). ctas_per_sm:
 * 0 = as many 256-thread blocks as the work fills (up to 8 per SM); 1..8 = that many per SM at
 * most, a fixed grid that leaves room for a GEMM's CTA on every SM. Replaces the mask half of
 * solution/lora.py:29-46 (tl.rand(seed, offsets) > p). */
int qb_dropout_bits(uint32_t* bits, int64_t rows, int64_t cols, uint64_t seed, float p,
                    int ctas_per_sm, cudaStream_t stream);

/* The LoRA A product of a dropped-out input, from the input and the mask bits:
 *     U[M, R] = xd[M, K] A[R, K]^T,   xd[m, k] = bf16(x[m, k] * scale) if mask bit set, else 0
 * (bits: the words of qb_dropout_mask / qb_dropout_bits, row stride ldbits >= ceil(K / 32));
 * bits = NULL: xd = x (no dropout). xd is formed in shared memory only; xd != NULL (with bits)
 * also stores it ([M, K], row stride ldxd) for a backward that reads it. bf16 everywhere, fp32
 * accumulation (tcgen05, TMEM); R a multiple of 32 in 32..256; x, A, xd row strides multiples
 * of 8 elements, 16-byte-aligned bases; U rows 16-byte aligned (ldu a multiple of 8).
 * Replaces the DropoutCast -> F.linear(xd, lora_A) pair of solution/lora.py:84-93 and the
 * peft composition it serves (lora_A(dropout(x))). */
int qb_lora_xa(const void* x, int64_t ldx, const void* a, int64_t lda, const uint32_t* bits,
               int64_t ldbits, float scale, void* u, int64_t ldu, void* xd, int64_t ldxd,
               int64_t M, int64_t K, int64_t R, cudaStream_t stream);

/* out = in * bit * scale (accumulate = 0) or out += in * bit * scale (accumulate = 1) with the
 * bits of qb_dropout_mask; cols a multiple of 8, 16-byte-aligned rows. */
int qb_dropout_apply(const void* in, int in_dtype, int64_t in_row_stride, const uint32_t* bits,
                     void* out, int out_dtype, int64_t out_row_stride, int64_t rows,
                     int64_t cols, float scale, int accumulate, cudaStream_t stream);

/* qb_dropout_apply of one input with up to four masks at once: outs[j] = in * bit_j * scales[j]
 * (bits[j]: [rows, ceil(cols / 32)] words), `in` read once. Host arrays of n (1..4) entries;
 * cols a multiple of 8, 16-byte-aligned rows. The dropouts the reference draws one
 * DropoutCast at a time (solution/lora.py:84-93) on the q / k / v projections' common input and
 * on the gate / up pair's. */
int qb_dropout_apply_multi(const void* in, int in_dtype, int64_t in_row_stride, int n,
                           const uint32_t* const* bits, void* const* outs, int out_dtype,
                           const int64_t* out_row_strides, const float* scales, int64_t rows,
                           int64_t cols, cudaStream_t stream);

/* out = base + lo * scaling (fp32 math). Replaces solution/lora.py:49-60
 * (lora_scaled_add_kernel). */
int qb_scaled_add(const void* base, int base_dtype, int64_t base_row_stride, const void* lo,
                  int lo_dtype, int64_t lo_row_stride, void* out, int out_dtype,
                  int64_t out_row_stride, int64_t rows, int64_t cols, float scaling,
                  cudaStream_t stream);

/* One segment of qb_adapter_pack: rows x cols fp32 at src (row stride src_ld elements) ->
 * bf16 at dst (row stride dst_ld), each element multiplied by `scale` in fp32 and rounded to
 * nearest even - the bits of (src * scale).to(bfloat16). first_chunk: the segment's first
 * 2048-element chunk in the launch (the running sum of the earlier segments' chunks). */
typedef struct {
  const float* src;
  void* dst;
  int64_t src_ld, dst_ld;
  int32_t rows, cols;
  float scale;
  int32_t pad;
  int64_t first_chunk;
} qb_pack_segment;

/* sizeof(qb_pack_segment): the layout check of a binding that builds the table itself. */
int64_t qb_pack_segment_size(void);

/* The bf16 operands of every LoRA adapter of a model in one launch (the per-projection
 * casts autocast makes of lora_A / lora_B's fp32 weights at every call of solution/lora.py:172,
 * the scaling of :173 folded into B,
 * once per step instead of once per use): `segs` is a device array of nseg segments sorted by
 * first_chunk, total_chunks the sum of their chunks (ceil(rows * cols / 2048) each). */
int qb_adapter_pack(const qb_pack_segment* segs, int nseg, int64_t total_chunks,
                    cudaStream_t stream);

/* ---------------------------------------------------------------------------------------------
 * Cross-entropy over rows of materialised logits (the chunked path)
 */

/* Per row of logits [rows, vocab] (row_stride in elements): lse, loss = lse - z[label]
 * (0 when label == -100 or < 0), entropy = lse - sum(softmax*z), argmax (first index of the
 * max) into pred (int64, may be NULL) and correct (int32: argmax == label and labelled; may be
 * NULL). With write_grad the row is overwritten in place by (softmax - onehot) * grad_scale
 * for labelled rows and 0 for the others.
 * Replaces solution/cross_entropy.py:48-90 (fused_ce_kernel) and solution/fused_ce.py:42-96
 * (ce_row_kernel, grad_scale = 1). */
int qb_ce_rows(void* logits, int logits_dtype, int64_t row_stride, const int64_t* target,
               int64_t rows, int64_t vocab, float* loss, float* entropy, int64_t* pred,
               int32_t* correct, float grad_scale, int write_grad, cudaStream_t stream);

/* ---------------------------------------------------------------------------------------------
 * Tensor-core (tcgen05 / TMEM / TMA) GEMM
 */

/* C[M,N] = A[M,K] * B[N,K]^T (+ bias[N] fp32), bf16 operands, fp32 accumulation, C in F32 or
 * BF16 (row stride ldc). a_mn_major = 0: A is [M,K] with row stride lda; 1: A is stored [K,M]
 * (row stride lda). Same for B ([N,K] or stored [K,N]). Leading dimensions must make rows
 * 16-byte aligned. Replaces the cuBLAS calls of the reference's chunked CE
 * (solution/cross_entropy.py:117 logits = h @ W.T, :123 grad_h = dz @ W) and of its 4-bit
 * linear (solution/nf4.py:104 F.linear, :111 grad_out @ W). */
int qb_gemm_bf16(const void* A, int64_t lda, int a_mn_major, const void* B, int64_t ldb,
                 int b_mn_major, void* C, int64_t ldc, int c_dtype, const float* bias, int64_t M,
                 int64_t N, int64_t K, cudaStream_t stream);

/* C[M, N] = A0[M, K0] * B0[N, K0]^T + A1[M, K1] * B1[N, K1]^T (+ bias[N] fp32)
 * (+ residual[M, N], C's type, row stride ldr), fp32 accumulation in one pass (segment 1 is extra
 * K of the same accumulator), one rounding; C fp32 or bf16. K1 == 0 without a residual is
 * qb_gemm_bf16. Otherwise the A operands are K-major and the B operands are both K-major or both
 * MN-major (QB_ERR_UNSUPPORTED otherwise). This is the long-token path of a 4-bit projection with
 * its LoRA term on a transient bf16 copy of the weight (qb_nf4_dequant writes it): forward
 * y = h + [x | u] [W | s*B_lora]^T + bias (h: the residual stream the projection feeds), input
 * gradient dx = [dy | v] [W^T | A_lora^T]^T. Replaces solution/nf4.py:100-112 (F.linear /
 * grad_out @ W on the dequantised weight), the lora_B(...) + ScaledAdd of solution/lora.py:172-173
 * and the decoder layer's residual add (transformers Qwen2DecoderLayer). */
int qb_gemm2_bf16(const void* A0, int64_t lda0, int a0_mn_major, const void* B0, int64_t ldb0,
                  int b0_mn_major, int64_t K0, const void* A1, int64_t lda1, int a1_mn_major,
                  const void* B1, int64_t ldb1, int b1_mn_major, int64_t K1, void* C,
                  int64_t ldc, int c_dtype, const float* bias, const void* residual, int64_t ldr,
                  int64_t M, int64_t N, cudaStream_t stream);

/* A q or k projection with the rotate-half RoPE of its heads in the epilogue:
 *   C[M, N] = rope(bf16(A0 B0^T + A1 B1^T + bias))   (bf16; heads of head_dim = 128 along N)
 * row m is the token at position m % S (rows are batch-major tokens), rotated with
 * cos[m % S, :] / sin[m % S, :] (bf16 [S, 128], row stride cs_stride_s) in the arithmetic of
 * qb_rope_qk (forward). All operands K-major bf16; K1 = 0 for no LoRA term. Replaces the
 * projection + solution/rope.py:82-104 (TritonRoPE forward) pair. */
int qb_gemm2_rope_bf16(const void* A0, int64_t lda0, const void* B0, int64_t ldb0, int64_t K0,
                       const void* A1, int64_t lda1, const void* B1, int64_t ldb1, int64_t K1,
                       void* C, int64_t ldc, const float* bias, const void* cos_,
                       const void* sin_, int64_t cs_stride_s, int64_t S, int64_t head_dim,
                       int64_t M, int64_t N, cudaStream_t stream);

/* The gate and up projections of a SwiGLU MLP in one GEMM, with the SwiGLU in its epilogue:
 *   g = x w_gate^T + u1 b1_gate^T,  u = x w_up^T + u1 b1_up^T     (fp32 accumulation)
 *   h[M, I] = silu(bf16(g)) * bf16(u)   (bf16; the arithmetic of qb_swiglu_fwd)
 * and, when g_out / u_out are given (both or neither), bf16(g) and bf16(u) themselves ([M, I],
 * row stride ldgu) for the backward. x [M, K0], w_gate / w_up [I, K0] (row stride ldw), all
 * K-major bf16 with 16-byte-aligned rows. The LoRA terms ride as extra K (K1 = 2r, 0 for none):
 * u1 = [dropout_g(x) A_g^T | dropout_u(x) A_u^T] [M, 2r], b1_gate = [s B_g | 0] and
 * b1_up = [0 | s B_u] ([I, 2r], row stride ldb1). Each 256-wide output tile is 128 gate and the
 * same 128 up features, the B tile loaded by TMA from both weights. Replaces
 * solution/swiglu.py:68-81 (gate_proj, up_proj, then the SwiGLU kernel) with the weights the
 * 4-bit path dequantised (solution/nf4.py:100-104) and the LoRA branches of solution/lora.py:172. */
int qb_gemm_gateup_swiglu(const void* x, int64_t ldx, const void* w_gate, const void* w_up,
                          int64_t ldw, int64_t K0, const void* u1, int64_t ldu1,
                          const void* b1_gate, const void* b1_up, int64_t ldb1, int64_t K1,
                          void* h, int64_t ldh, void* g_out, void* u_out, int64_t ldgu, int64_t M,
                          int64_t I, cudaStream_t stream);

/* One dropout mask drawn as bits: words[r * ceil(cols / 32) + c / 32] bit (c & 31) is set when
 * element (r, c) is kept, the same words qb_dropout_bits writes for (rows, cols, seed, p). */
typedef struct qb_mask_job {
  uint32_t* bits;          /* device, 4-byte aligned, rows * ceil(cols / 32) words */
  int64_t rows, cols;
  uint64_t seed;
  float p;                 /* < 1 */
} qb_mask_job;

/* sizeof(qb_mask_job): the layout check of a binding that builds the array itself. */
int64_t qb_mask_job_size(void);

/* qb_gemm_gateup_swiglu, and in the same launch up to 8 dropout masks drawn as bits by warps the
 * GEMM adds beside its own (the Philox rounds run on the integer pipes while the tensor cores
 * run the product). `jobs` is a host array of njobs entries; the bits are complete when the
 * launch is. The model draws the next projections' masks here, which the projections then only
 * apply (solution/lora.py:29-46 draws each mask inside its own dropout pass). */
int qb_gemm_gateup_swiglu_masks(const void* x, int64_t ldx, const void* w_gate,
                                const void* w_up, int64_t ldw, int64_t K0, const void* u1,
                                int64_t ldu1, const void* b1_gate, const void* b1_up,
                                int64_t ldb1, int64_t K1, void* h, int64_t ldh, void* g_out,
                                void* u_out, int64_t ldgu, int64_t M, int64_t I,
                                const qb_mask_job* jobs, int njobs, cudaStream_t stream);

/* C[M, N] (bf16, in place) += scale * mask .* (A[M, K] * B[N, K]^T): fp32 product, one rounding
 * per element, A K-major, B K- or MN-major; mask bit (n & 31) of bits[m * ldbits + n / 32] (the
 * words qb_dropout_mask records). The input gradient of a dropped-out LoRA branch,
 * dx += s * mask .* ((dy s B) A), added to the base projection's dx without storing the [M, N]
 * product. Replaces the DropoutCast backward (solution/lora.py:90-93) on lora_A's input gradient
 * and the autograd sum of the two dx terms. */
int qb_gemm_bf16_mask_acc(const void* A, int64_t lda, const void* B, int64_t ldb, int b_mn_major,
                          const uint32_t* bits, int64_t ldbits, float scale, void* C, int64_t ldc,
                          int64_t M, int64_t N, int64_t K, cudaStream_t stream);

/* ---------------------------------------------------------------------------------------------
 * NF4 x LoRA projection on tcgen05, the NF4 weight rebuilt in registers inside the GEMM
 *
 * Weight: nested NF4 (blocksize 64, double-quantised scales) of shape [out_f, in_f], in the
 * layout qb_nf4_dequant reads; in_f a multiple of 64 (of 128 for the dgrad), packed 16-byte
 * aligned. Activations bf16 row-major with 16-byte-aligned rows.
 */

/* y[T, out_f] = x[T, in_f] * deq(W)^T (+ bias[out_f] bf16) (+ u[T, r] * lora_b_scaled[out_f, r]^T)
 * in bf16 (fp32 accumulation). With r > 0, u = dropout(x) * A_lora^T and lora_b_scaled =
 * scaling * B_lora (bf16): the LoRA term rides along as extra K, so the adapter's second GEMM and
 * the scaled add disappear. Replaces solution/nf4.py:100-104 (dequantize_nf4 + F.linear) and, with
 * r > 0, the lora_B(...) + ScaledAdd of solution/lora.py:172-173. */
int qb_nf4_linear_fwd(const void* x, int64_t ldx, const uint8_t* packed, const uint8_t* absmax_q,
                      const float* code2, const float* absmax2, float offset, int blocksize2,
                      const float* lut16, int64_t tokens, int64_t in_f, int64_t out_f,
                      const void* bias, const void* u, int64_t ldu, const void* lora_b_scaled,
                      int64_t ldlb, int64_t r, void* y, int64_t ldy, cudaStream_t stream);

/* dx[T, in_f] = dy[T, out_f] * deq(W) (+ v[T, r] * lora_a[r, in_f]) in bf16, W read transposed
 * from the same packed codes. With r > 0, v = scaling * dy * B_lora (no dropout on this path).
 * Replaces solution/nf4.py:107-112 (dequantize_nf4 + grad_out @ weight). */
int qb_nf4_linear_dgrad(const void* dy, int64_t lddy, const uint8_t* packed,
                        const uint8_t* absmax_q, const float* code2, const float* absmax2,
                        float offset, int blocksize2, const float* lut16, int64_t tokens,
                        int64_t in_f, int64_t out_f, const void* v, int64_t ldv,
                        const void* lora_a, int64_t ldla, int64_t r, void* dx, int64_t lddx,
                        cudaStream_t stream);

/* ---------------------------------------------------------------------------------------------
 * Fused linear cross-entropy on tcgen05 (logits only in TMEM)
 *
 * Replaces, for bf16 hidden states and head, the chunk loop of solution/cross_entropy.py:115-124
 * (cuBLAS logits, fused_ce_kernel, cuBLAS dz @ W) and of solution/fused_ce.py:132-144.
 * hidden [rows, hdim] bf16 (row stride ldh), weight [vocab, hdim] bf16 (row stride ldw),
 * target [rows] int64 (-100 or any value outside [0, vocab) = unlabelled).
 */

/* Number of 256-wide vocab tiles: partials hold vocab_tiles * rows float4 records. */
int64_t qb_linear_ce_vocab_tiles(int64_t vocab);

/* Pass 1: per (vocab tile, row) the tile's (max, sum exp(z - max), sum exp(z - max) * z, first
 * argmax) into `partials` (float4 [vocab_tiles, rows]), and z[label] into z_label[rows]. */
int qb_linear_ce_stats(const void* hidden, int64_t ldh, const void* weight, int64_t ldw,
                       const int64_t* target, int64_t rows, int64_t vocab, int64_t hdim,
                       void* partials, float* z_label, cudaStream_t stream);

/* qb_linear_ce_stats that also stores each tile's fp32 logits into `logits` ([rows, ldl],
 * ldl >= vocab): the gradient then comes from qb_ce_grad_from_logits, one streaming pass over
 * them, instead of a second GEMM (qb_linear_ce_grad). Costs rows * ldl * 4 bytes of caller scratch
 * per chunk. No counterpart in the reference (its chunk logits are a bf16 matmul output,
 * solution/cross_entropy.py:117). */
int qb_linear_ce_stats_logits(const void* hidden, int64_t ldh, const void* weight, int64_t ldw,
                              const int64_t* target, int64_t rows, int64_t vocab, int64_t hdim,
                              void* partials, float* z_label, float* logits, int64_t ldl,
                              cudaStream_t stream);

/* dz[rows, vocab] (bf16, row stride ldz) = (exp(z - lse) - onehot(label)) * scale from the fp32
 * logits qb_linear_ce_stats_logits stored: the same arithmetic on the same z as
 * qb_linear_ce_grad, so the same dz (solution/cross_entropy.py:83-90). */
int qb_ce_grad_from_logits(const float* logits, int64_t ldl, const int64_t* target, int64_t rows,
                           int64_t vocab, const float* lse, const float* scale_dev, void* dz,
                           int64_t ldz, cudaStream_t stream);

/* Merges the partials: lse, loss = lse - z[label] (0 if unlabelled), entropy = lse - sum(p*z),
 * pred = first argmax (int64, may be NULL), correct (int32, may be NULL), lse (may be NULL).
 * The per-row outputs of solution/cross_entropy.py:77-81 / fused_ce.py:81-87. */
int qb_ce_reduce(const void* partials, int64_t n_vtiles, int64_t rows, int64_t vocab,
                 const int64_t* target, const float* z_label, float* loss, float* entropy,
                 int64_t* pred, int32_t* correct, float* lse, cudaStream_t stream);

/* Pass 2: dz[rows, vocab] (bf16, row stride ldz) = (exp(z - lse) - onehot(label)) * scale, with
 * scale = *scale_dev (a device scalar, e.g. 1 / denominator) for labelled rows and 0
 * otherwise (solution/cross_entropy.py:83-90). dH = dz @ weight follows with qb_gemm_bf16. */
int qb_linear_ce_grad(const void* hidden, int64_t ldh, const void* weight, int64_t ldw,
                      const int64_t* target, int64_t rows, int64_t vocab, int64_t hdim,
                      const float* lse, const float* scale_dev, void* dz, int64_t ldz,
                      cudaStream_t stream);

/* Floats of workspace qb_gemm_bf16_acc_f32 needs for this shape on the current device (0: the
 * launch runs unsplit and needs none). */
int64_t qb_gemm_bf16_acc_f32_workspace(int64_t M, int64_t N, int64_t K);

/* C[M,N] (fp32, row stride ldc) = beta * C + alpha * A[M,K] * B[N,K]^T on the tcgen05 GEMM,
 * beta 0 (C is written without being read) or 1. When there are too few output tiles to fill
 * the SMs the k-blocks are split into ranges: each range's partial product goes to `workspace`
 * (at least qb_gemm_bf16_acc_f32_workspace floats, 16-byte aligned) and a second kernel adds
 * alpha * their sum, taken in range order - the same bits on every run. Operand layouts as
 * qb_gemm_bf16. The LoRA weight gradients of lora.py:172 (nn.Linear backward under autocast):
 * dA = V^T xd and dB = s g^T U, skinny outputs whose K is the token count. */
int qb_gemm_bf16_acc_f32(const void* A, int64_t lda, int a_mn_major, const void* B, int64_t ldb,
                         int b_mn_major, float alpha, float beta, float* C, int64_t ldc,
                         int64_t M, int64_t N, int64_t K, float* workspace,
                         int64_t workspace_floats, cudaStream_t stream);

/* Reads and clears this device's tensor-core error flag (synchronises `stream`): QB_OK, or
 * QB_ERR_TIMEOUT when a kernel gave up one of its bounded waits (its output is then invalid). */
int qb_device_error(cudaStream_t stream);

/* Report of this process's launch monitor for `device`, no counterpart in the reference. The
 * tensor-core kernels write pinned host memory mapped into the device: each CTA the launch
 * sequence number it started and, once it has released its tensor memory, finished; a bounded
 * wait that gives up writes its site, CTA and SM. This call formats that record into buf (at most
 * len bytes, NUL-terminated) from host memory alone - no CUDA call - so a watchdog thread can
 * read it while the device is stuck: the last launch issued, the last one whose CTAs all
 * finished, and each launch with CTAs that started and never finished. */
int qb_monitor_report(int device, char* buf, int64_t len);

/* Self-test of the failure path, no counterpart in the reference: launches one thread that waits
 * (bounded, limit_ns between 1 ms and 2 s) on an mbarrier nothing arrives on, so the wait gives up
 * and raises the device error flag as a stuck kernel would; qb_device_error then reports
 * QB_ERR_TIMEOUT and the context stays usable. */
int qb_selftest_bounded_wait(int64_t limit_ns, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* QLORA_B200_H */
