/*
 * ratchet_b200.h — C ABI of the B200 (sm_100a) ratchet-linear train-step library.
 *
 * Every entry point takes caller-owned device pointers, element strides and an explicit
 * cudaStream_t (passed as void*), allocates nothing, never synchronises the host and returns an
 * int status (RT_OK == 0).  On failure rt_last_error() returns a thread-local message.  Device-side
 * problems that are found while a kernel runs (non-finite gradients, a bounded wait that ran out)
 * are recorded in a sticky device status word read with rt_device_status().
 *
 * Reference interface each function replaces is cited as file:line inside the reference project
 * (LoomNode/local-ai-training, package src/local_ai_training).
 */
#ifndef RATCHET_B200_H
#define RATCHET_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define RT_ABI_VERSION 2

/* status codes */
#define RT_OK 0
#define RT_ERR_INVALID_ARGUMENT 1 /* shapes, strides, null pointers  -> ValueError   */
#define RT_ERR_DTYPE 2            /* unsupported element type        -> TypeError    */
#define RT_ERR_ALIGNMENT 3        /* pointer/stride alignment        -> ValueError   */
#define RT_ERR_CUDA 4             /* launch or driver failure        -> RuntimeError */
#define RT_ERR_UNSUPPORTED 5      /* valid request this build cannot serve           */

/* element types */
#define RT_F32 0
#define RT_BF16 1
#define RT_I8 2
#define RT_U8 3

/* bits of the sticky device status word */
#define RT_STATUS_NONFINITE_GRADIENT 0x1u /* ratchet gradient held NaN/Inf (row left unchanged) */
#define RT_STATUS_WAIT_TIMEOUT 0x2u       /* a bounded pipeline wait gave up                     */
#define RT_STATUS_CODE_RANGE 0x4u         /* validate: code escaped [-max_code, max_code]        */
#define RT_STATUS_PRESSURE_RANGE 0x8u     /* validate: |pressure| > 7                            */
#define RT_STATUS_SCALE_INVALID 0x10u     /* validate: a row scale is <= 0 or non-finite         */
#define RT_STATUS_INDEX_RANGE 0x20u       /* a token id / window outside its table (zeros used)  */

int rt_abi_version(void);
const char *rt_last_error(void);

/* Reads the sticky device status word into *out (host memory) after the work queued on `stream`
 * so far; optionally clears it.  This call synchronises `stream` (eval-cadence use only). */
int rt_device_status(uint32_t *out, int clear, void *stream);

/* Number of SMs of the current device (cached per device). */
int rt_sm_count(int *out);

/* ---------------------------------------------------------------------------------------------
 * Row quantisation.  Replaces int8_matmul.py:_quantize_rows_kernel (106-150) through
 * quantize_rows (251-259) and quantize_rows_colscaled (262-277).
 *   v[m,k]   = float(x[m,k]) * col_scale[k]          (col_scale optional)
 *   scale[m] = max(max_k |v[m,k]| / 127, FLT_MIN)
 *   RN: q = clamp(rint(v / scale), -127, 127)
 *   SR: q = clamp(floor(v / scale + u), -127, 127), u = (h + 1/2)·2^-16 from 16-bit half
 *       (e & 1) of word (e & 7)/2 of Philox4x32-10 keyed by (seed, layer) with counter
 *       (element index e / 8, step)  [own mapping, not Triton's tl.rand]
 * x_bf16_out (optional) receives bf16(x) (unscaled) — the grad_weight GEMM operand of
 * ratchet.py:162 — so the gradient is read from HBM once.
 * round_input_bf16 (fp32 input): each value is first rounded to bf16, the cast autograd applies
 * to the gradient of a bf16 layer output whose consumer was fused into an fp32 residual add.
 * step_dev (optional): two device uint32s.  step_dev[0] is read in place of `step` and the call
 * advances it by one once every CTA has read it; step_dev[1] is the call's arrival count and must
 * be zero between calls (calls leave it zero).  Consecutive calls, and the replays of a captured
 * CUDA graph, thus draw fresh streams without host work.  Calls sharing a step_dev must not
 * overlap on the GPU.
 * ------------------------------------------------------------------------------------------- */
int rt_quantize_rows(const void *x, int x_dtype, int64_t rows, int64_t cols, int64_t stride_row,
                     int64_t stride_col, const float *col_scale, int stochastic,
                     int round_input_bf16, uint64_t seed, uint32_t step, uint32_t layer,
                     uint32_t *step_dev, int8_t *q,
                     int64_t ldq, float *row_scale, void *x_bf16_out, int64_t ld_xbf16,
                     void *stream);

/* ---------------------------------------------------------------------------------------------
 * Scaled int8 GEMM.  Replaces int8_matmul.py:scaled_int8_mm (289-343) / _scaled_int8_kernel
 * (26-79).  out[m,n] = bf16((float(sum_k lhs[m,k]*rhs[k,n]) * lhs_scale[m]) * rhs_scale[n]);
 * rhs_scale may be NULL (== 1.0, the grad_input call of ratchet.py:133-134).  Operands are
 * addressed by element strides exactly like the reference kernel: lhs (M,K), rhs (K,N).
 * out_dtype RT_BF16 stores the bf16 value, RT_F32 stores the same bf16-rounded value widened to
 * fp32 (the `.to(inputs.dtype)` of ratchet.py:67 fused into the epilogue).
 * 16-byte-aligned unit-stride operands run the tcgen05 kind::i8 TMA kernel; anything else runs a
 * SIMT kernel with identical arithmetic.
 * rhs_abs_max: a bound the caller guarantees on |rhs| (ratchet codes: 7), or 0 when unknown; it
 * only selects a cheaper exact int32 -> fp32 conversion when K·128·bound < 2^22 (results are the
 * same either way as long as the bound holds).
 * residual (optional, fp32 out only, M x N with row stride ld_residual; may be `out` itself):
 * out = residual + (the fp32-widened bf16 value), the residual add of the transformer block
 * (model.py TransformerBlock.forward: `inputs + attention(...)`, `inputs + feed_forward(...)`) in
 * the epilogue instead of a separate pass over the residual stream.
 * ------------------------------------------------------------------------------------------- */
int rt_scaled_int8_mm(const int8_t *lhs, int64_t lhs_stride_m, int64_t lhs_stride_k,
                      const int8_t *rhs, int64_t rhs_stride_k, int64_t rhs_stride_n,
                      const float *lhs_scale, const float *rhs_scale, void *out, int out_dtype,
                      int64_t ldo, int64_t M, int64_t N, int64_t K, int rhs_abs_max,
                      const float *residual, int64_t ld_residual, void *stream);

/* ---------------------------------------------------------------------------------------------
 * grad_weight GEMM.  Replaces the per-tile cuBLAS BF16 GEMM of ratchet.py:148-163:
 *   gw[n,k] (+)= sum_m g[m,n] * x[m,k]     (bf16 operands, fp32 accumulation)
 * g is (M_tok, N) and x is (M_tok, K), both row-major with unit column stride.  out_dtype RT_F32
 * (`accumulate` adds into out) or RT_BF16 (`accumulate` must be 0).  The bf16 rounding the
 * reference applies to the GEMM output is applied by rt_ratchet_update(round_bf16=1), not here.
 * Small outputs split the token dimension across SMs: each split writes an fp32 partial tile to
 * `workspace` and a second launch sums the partials in split order (deterministic, no CTA waits
 * for another).  workspace: 256-byte aligned, no initial contents needed; NULL disables
 * splitting.  Calls sharing a workspace must not overlap on the GPU.
 * ------------------------------------------------------------------------------------------- */
int rt_grad_weight_bf16(const void *g, int64_t ldg, const void *x, int64_t ldx, void *out,
                        int out_dtype, int64_t ldo, int64_t M_tok, int64_t N, int64_t K,
                        int accumulate, void *workspace, int64_t workspace_bytes, void *stream);
/* Workspace bytes rt_grad_weight_bf16 can use for this shape on the current device (0: none). */
int64_t rt_grad_weight_workspace_bytes(int64_t M_tok, int64_t N, int64_t K);

/* grad_weight GEMM and ratchet update in one call: the fused-update path of ratchet.py:148-163
 * (per-tile bf16 GEMM, `.float()` of its bf16 result) -> _capture_weight_gradient -> the update of
 * rt_ratchet_update(normalize=1, round_bf16=1) with grad[n,k] = sum_m g[m,n] * x[m,k].  grad_W is
 * never stored: the GEMM leaves fp32 partial tiles in `workspace` (at least
 * rt_grad_weight_update_workspace_bytes, 256-byte aligned) and the update sums them in split order
 * as it reads each row, giving the values rt_grad_weight_bf16 + rt_ratchet_update would use.
 * g (M_tok, rows) and x (M_tok, cols) bf16 with 16-byte rows, cols % 8 == 0, else
 * RT_ERR_UNSUPPORTED.  Remaining arguments as rt_ratchet_update. */
int rt_grad_weight_ratchet_update(const void *g, int64_t ldg, const void *x, int64_t ldx,
                                  int64_t M_tok, int64_t rows, int64_t cols, void *workspace,
                                  int64_t workspace_bytes, uint8_t *packed, int64_t ldp,
                                  int8_t *code_out, int64_t ldc, float *rms_ema, double ema_beta,
                                  int max_code, int threshold, double bucket_low,
                                  double bucket_high, double eps, int64_t *counts, float *row_rms,
                                  float *rms_sum, float *grad_scale, void *stream);
int64_t rt_grad_weight_update_workspace_bytes(int64_t M_tok, int64_t rows, int64_t cols);

/* rt_grad_weight_bf16 that allocates nothing and takes no workspace (no counterpart in the
 * reference, whose grad_weight GEMM is a cuBLAS call).  For callers that bind the C ABI without
 * a device allocator of their own (an FFI host with no caching allocator, where cudaMalloc would
 * synchronise the device in the middle of a step) or that have budgeted all HBM to resident
 * state.  The split-K partial tiles live in a 20 MiB device array of this library (one copy per
 * device); shapes whose workspace (rt_grad_weight_workspace_bytes) exceeds it fail with
 * RT_ERR_UNSUPPORTED (on B200, 148 SMs, no shape needs more than 18.5 MiB, so this only happens on
 * parts with more than 160 SMs).  The array's address belongs to one CUDA context: the first call
 * in each context (a device's primary context, a context created after cudaDeviceReset, or any
 * other context the host makes current) looks it up with that context current and caches it
 * under the context's unique id; make that first call before any stream capture.  Nothing in the
 * array needs to start at zero (every partial tile is written before it is read, within a call).
 * All calls on one device share the array: calls that overlap on the GPU
 * (different streams, no ordering between them) race and give wrong results.  Results equal
 * rt_grad_weight_bf16 with a workspace of rt_grad_weight_workspace_bytes bytes. */
int rt_grad_weight_bf16_noalloc(const void *g, int64_t ldg, const void *x, int64_t ldx, void *out,
                                int out_dtype, int64_t ldo, int64_t M_tok, int64_t N, int64_t K,
                                int accumulate, void *stream);

/* out[M,N] = A[M,K] @ B[K,N]: bf16 operands, row-major (row strides lda / ldb elements, 16-byte
 * aligned rows), fp32 accumulation, bf16 (RN) or float32 output.  Replaces the bf16 grad_input
 * matmul of ratchet.py:135-141 (`grad_output.to(bf16) @ (code.to(bf16) * scale.to(bf16))`, the
 * non-int8-backward branch and the self-quantising lm_head) with the tcgen05 kind::f16 GEMM. */
int rt_matmul_bf16(const void *a, int64_t lda, const void *b, int64_t ldb, void *out,
                   int out_dtype, int64_t ldo, int64_t M, int64_t N, int64_t K, void *stream);

/* rt_grad_weight_bf16 adding a float32 matrix: out[n,k] = round(addend[n,k] + sum_m g[m,n]*x[m,k])
 * in out_dtype (float32 or bfloat16), addend row stride ld_addend; addend may be `out` itself
 * when out is float32.  For gradient accumulation over micro-batches (no counterpart in the
 * reference, which takes one batch per update): earlier micro-batches accumulate their grad_W
 * in float32, and the last one writes the bf16-rounded total straight into the buffer that is
 * reduce-scattered or updated -- the reference's bf16 rounding of the GEMM output
 * (ratchet.py:162-163) then happens once, on the accumulated sum. */
int rt_grad_weight_bf16_add(const void *g, int64_t ldg, const void *x, int64_t ldx,
                            const float *addend, int64_t ld_addend, void *out, int out_dtype,
                            int64_t ldo, int64_t M_tok, int64_t N, int64_t K, void *workspace,
                            int64_t workspace_bytes, void *stream);

/* Dequantises saved int8 activations: out[m,k] = bf16(bf16(q[m,k]) * bf16(s[m]))
 * (ratchet.py:73-76). */
int rt_dequant_rows_bf16(const int8_t *q, int64_t ldq, const float *row_scale, void *out,
                         int64_t ldo, int64_t rows, int64_t cols, void *stream);

/* ---------------------------------------------------------------------------------------------
 * Ratchet update, one HBM pass per weight.  Replaces ratchet.py:_capture_weight_gradient
 * (487-537) -> _normalize (539-556) -> _ratchet_update_core (265-301) -> pack (185-192), and
 * apply_normalized_gradient (582-611) when normalize == 0.
 *   grad: (rows, cols) fp32 or bf16; round_bf16 rounds fp32 input to bf16 first (the
 *         `grad_weight_tile.float()` of ratchet.py:162-163).
 *   packed: uint8 code|pressure nibbles, updated in place; code_out (optional) receives the new
 *         int8 codes (the GEMM operand), code_out may alias nothing else.
 *   rms_ema (optional, rows): per-row second-moment EMA (ratchet.py:543-553), beta in (0,1).
 *   counts (int64[4], accumulated): positive, negative, blocked positive, blocked negative moves.
 *   row_rms (optional, rows): sqrt(mean(g^2)) of each row (ratchet.py:534-537 statistics).
 *   rms_sum (optional, one float, accumulated): the sum of those row values.
 *   grad_scale (optional, rows): sum_k g[r,k] * code_before[r,k] (ratchet.py:167-169).
 * Rows holding NaN/Inf are left unchanged and set RT_STATUS_NONFINITE_GRADIENT.
 * The row mean-square uses a fixed reduction order (documented in the kernel) mirrored by the
 * CPU oracle, so results are bit-reproducible.
 * ------------------------------------------------------------------------------------------- */
int rt_ratchet_update(const void *grad, int grad_dtype, int round_bf16, int64_t ldg, int64_t rows,
                      int64_t cols, uint8_t *packed, int64_t ldp, int8_t *code_out, int64_t ldc,
                      int normalize, float *rms_ema, double ema_beta, int max_code, int threshold,
                      double bucket_low, double bucket_high, double eps, int64_t *counts,
                      float *row_rms, float *rms_sum, float *grad_scale, void *stream);

/* One layer of a grouped update (rt_ratchet_update_grouped). */
typedef struct rt_update_layer {
  const void *grad;   /* (rows, cols) gradient in the group's dtype, row stride ldg elements */
  int64_t ldg;
  int64_t rows;
  uint8_t *packed;    /* updated in place, row stride ldp */
  int64_t ldp;
  int8_t *code_out;   /* optional: receives the new int8 codes, row stride ldc */
  int64_t ldc;
  float *rms_ema;     /* optional (rows), used when ema_beta > 0 */
  int64_t *counts;    /* int64[4] move counters of the layer, accumulated */
  float *rms_sum;     /* optional: += sum of the layer's row rms values */
  float grad_mul;     /* gradient multiplier applied after the optional bf16 rounding (1: none) */
} rt_update_layer;

/* rt_ratchet_update over many layers in as few launches as possible (one per 64 layers).
 * Replaces the reference's per-layer update inside backward (ratchet.py:_capture_weight_gradient
 * 487-537 called once per 256-row tile from _RatchetMatmul.backward, ratchet.py:150-169) after
 * the whole backward: rows are independent, so updating every layer after backward gives the
 * same state as updating each inside its own backward (each layer's grad_input has already
 * read its codes).  All layers share cols, dtype and the ratchet parameters; per layer the
 * result equals rt_ratchet_update on grad * grad_mul (normalize, round_bf16 as there; row_rms and
 * grad_scale are not produced).  `layers` is host memory, read during the call. */
int rt_ratchet_update_grouped(const rt_update_layer *layers, int n_layers, int grad_dtype,
                              int round_bf16, int64_t cols, int normalize, double ema_beta,
                              int max_code, int threshold, double bucket_low, double bucket_high,
                              double eps, void *stream);

/* Pressure leak: every nonzero pressure moves one unit toward zero (ratchet.py:613-625).
 * code_out, when given, is refreshed with the (unchanged) codes. */
int rt_ratchet_leak(uint8_t *packed, int64_t ldp, int64_t rows, int64_t cols, int max_code,
                    void *stream);

/* Unpacks nibbles (ratchet.py:195-199); code or pressure may be NULL. */
int rt_unpack_code_pressure(const uint8_t *packed, int64_t ldp, int64_t rows, int64_t cols,
                            int max_code, int8_t *code, int64_t ldc, int8_t *pressure,
                            int64_t ldpr, void *stream);

/* State validation (ratchet.py:672-679) into the sticky device status word: code range,
 * pressure nibble range and, when scale != NULL, positive finite row scales. */
int rt_ratchet_validate(const uint8_t *packed, int64_t ldp, int64_t rows, int64_t cols,
                        int max_code, const float *scale, void *stream);

/* ---------------------------------------------------------------------------------------------
 * Fused producers of pre-quantised layer inputs (int8_fused.py / int8_backward.py).
 * dq_out (optional, rows x cols bf16, row stride ld_dq): also receives bf16(bf16(q) * bf16(s)),
 * the grad_weight operand the layer's backward would otherwise dequantise from the saved int8
 * rows (ratchet.py:73-76, rt_dequant_rows_bf16) -- written from registers by the producer.
 * ------------------------------------------------------------------------------------------- */
/* y = x * rsqrt(mean(x^2) + eps) * w, then RN row quant (int8_fused.py:14-56). */
int rt_rmsnorm_quantize(const void *x, int x_dtype, int64_t ldx, const float *weight, double eps,
                        int64_t rows, int64_t cols, int8_t *q, int64_t ldq, float *row_scale,
                        void *dq_out, int64_t ld_dq, void *stream);
/* tanh-GELU then RN row quant (int8_fused.py:58-101). */
int rt_gelu_quantize(const void *x, int x_dtype, int64_t ldx, int64_t rows, int64_t cols,
                     int8_t *q, int64_t ldq, float *row_scale, void *dq_out, int64_t ld_dq,
                     void *stream);
/* [B,H,T,D] (any strides) -> rows b*T+t of H*D channels, RN row quant (int8_fused.py:103-151). */
int rt_transpose_quantize(const void *x, int x_dtype, int64_t batch, int64_t heads, int64_t seq,
                          int64_t head_dim, int64_t stride_b, int64_t stride_h, int64_t stride_s,
                          int64_t stride_d, int8_t *q, int64_t ldq, float *row_scale,
                          void *dq_out, int64_t ld_dq, void *stream);
/* RMSNorm backward (int8_backward.py:7-51): dx written in dx_dtype (through bf16, as the
 * reference stores it); dw (optional, cols floats, accumulated) += sum over rows of gy*x*rsqrt,
 * summed in a fixed order (per-CTA partial rows, then the partials in CTA order), so the result
 * is the same on every call, as the reference's torch reduction is.  dw_work: with dw, a device
 * workspace of rt_rmsnorm_backward_workspace_bytes(rows, cols) bytes (16-byte aligned), used
 * within the call.  dx_add (optional, fp32 dx only, may equal dx): the residual branch's
 * gradient, added to dx the way autograd accumulates the two branches of the residual stream. */
int rt_rmsnorm_backward(const void *grad_y, int gy_dtype, const void *x, int x_dtype,
                        const float *weight, double eps, int64_t rows, int64_t cols, void *dx,
                        int dx_dtype, float *dw, const float *dx_add, float *dw_work,
                        int64_t dw_work_bytes, void *stream);
int64_t rt_rmsnorm_backward_workspace_bytes(int64_t rows, int64_t cols);
/* tanh-GELU backward (int8_backward.py:53-89); dx written in dx_dtype. */
int rt_gelu_backward(const void *grad_y, int gy_dtype, const void *x, int x_dtype, int64_t rows,
                     int64_t cols, void *dx, int dx_dtype, void *stream);

/* ---------------------------------------------------------------------------------------------
 * Gradient producers fused with the consuming layer's stochastic-rounding quantisation.  Each
 * computes the output gradient G of a ratchet layer (the gradient the layer's backward receives)
 * and, in the same pass, quantises G exactly as rt_quantize_rows(G, col_scale, stochastic=1,
 * round_input_bf16, seed, step, layer, step_dev, q, ldq, row_scale, x_bf16_out) would: the
 * ratchet.py:117-134 fold of the layer's row scales into the gradient and its per-token
 * stochastic rounding, with the same Philox stream and step_dev advance.  They replace the
 * reference's two passes (the producer's backward, then the layer's quantisation) over G.
 * Rows must allow 16-byte chunks (RT_ERR_UNSUPPORTED otherwise; the caller then runs the two
 * passes).
 *
 * rt_rmsnorm_backward_sr: rt_rmsnorm_backward (int8_backward.py:7-51) whose dx is G.
 * rt_gelu_backward_sr: tanh-GELU backward (int8_backward.py:53-89) of contiguous rows whose
 *   dx (dtype of grad_y and x) is G.
 * rt_heads_gather_sr: G[b·T+t, p·H·D + h·D + d] = src_p[b, h, t, d] for p = 0, 1, 2 — the
 *   gradient of a q|k|v projection output split into three [B, H, T, D] head views
 *   (model.py:61-70, `.chunk(3)` and the head transposes), written to `out` (row stride ldo).
 *   strides holds (b, h, t, d) element strides of src_0, src_1, src_2; d strides must be 1.
 * ------------------------------------------------------------------------------------------- */
int rt_rmsnorm_backward_sr(const void *grad_y, int gy_dtype, const void *x, int x_dtype,
                           const float *weight, double eps, int64_t rows, int64_t cols, void *dx,
                           int dx_dtype, float *dw, const float *dx_add, const float *col_scale,
                           int round_input_bf16, uint64_t seed, uint32_t step, uint32_t layer,
                           uint32_t *step_dev, int8_t *q, int64_t ldq, float *row_scale,
                           void *x_bf16_out, int64_t ld_xbf16, float *dw_work,
                           int64_t dw_work_bytes, void *stream);
int rt_gelu_backward_sr(const void *grad_y, const void *x, int dtype, int64_t rows, int64_t cols,
                        void *dx, const float *col_scale, uint64_t seed, uint32_t step,
                        uint32_t layer, uint32_t *step_dev, int8_t *q, int64_t ldq,
                        float *row_scale, void *x_bf16_out, int64_t ld_xbf16, void *stream);
int rt_heads_gather_sr(const void *const *src, const int64_t *strides, int dtype, int64_t batch,
                       int64_t heads, int64_t seq, int64_t head_dim, void *out, int64_t ldo,
                       const float *col_scale, uint64_t seed, uint32_t step, uint32_t layer,
                       uint32_t *step_dev, int8_t *q, int64_t ldq, float *row_scale,
                       void *x_bf16_out, int64_t ld_xbf16, void *stream);

/* ---------------------------------------------------------------------------------------------
 * Token cross-entropy over the lm_head logits.  Replaces F.cross_entropy(logits, targets) of
 * model.py:244-249 (mean over targets != ignore_index) and the bf16 cast of its gradient before
 * the lm_head grad GEMMs (ratchet.py:139-141, 161).  Forward, per row: row_max, row_logsum =
 * log(sum exp(x - max)), row_loss = -((x_t - max) - logsum) (0 for ignored rows).  Backward
 * writes grad_bf16[r, j] = bf16(RN(exp((x - max) - logsum) * w) - [j == t] * w (+ extra_grad)),
 * w = grad_loss / count read from device memory (no host sync; capturable).  An out-of-range
 * target sets RT_STATUS_CODE_RANGE and its row is treated as ignored.
 * ------------------------------------------------------------------------------------------- */
int rt_cross_entropy_fwd(const void *logits, int dtype, int64_t ld, int64_t rows, int64_t cols,
                         const int64_t *targets, int64_t ignore_index, float *row_max,
                         float *row_logsum, float *row_loss, void *stream);
int rt_cross_entropy_bwd(const void *logits, int dtype, int64_t ld, int64_t rows, int64_t cols,
                         const int64_t *targets, int64_t ignore_index, const float *row_max,
                         const float *row_logsum, const float *grad_loss, const float *count,
                         const float *extra_grad, int64_t ld_extra, void *grad_bf16, int64_t ldo,
                         void *stream);

/* ---------------------------------------------------------------------------------------------
 * Ratchet embedding (ratchet.py:688-749, RatchetEmbedding: rows are tokens) and device-resident
 * uint16 token shards (data.py:238-287).
 *
 * rt_embedding_forward: out[t, :] = float(code(packed[tok[t], :])) * scale[tok[t]], the
 *   reference's F.embedding(tokens, code.float() * scale[:, None]) without materialising the
 *   [rows, dim] effective weight.  Tokens outside [0, rows) give zero rows and set
 *   RT_STATUS_INDEX_RANGE.
 * rt_embedding_ratchet_update: the embedding's update from its output gradient grad [n_tok, dim]
 *   (fp32) without a [rows, dim] gradient: sorted_tokens / order are the token ids sorted stably
 *   and their positions; each distinct token's gradient row is the sum of its positions' rows in
 *   position order from +0 (the reference's CPU embedding backward), then that row is updated
 *   exactly as rt_ratchet_update(normalize=1) would; rows of absent tokens have a zero gradient
 *   in the reference and stay unchanged there, so they are not visited.  workspace:
 *   rt_embedding_update_workspace_bytes(n_tok, dim) bytes, 256-byte aligned.  counts and rms_sum
 *   accumulate over the visited rows (the absent rows' rms is zero).
 * rt_token_windows: inputs[b, t] = data[starts[b] + t], targets[b, t] = data[starts[b] + t + 1]
 *   (uint16 ids widened to int64), the reference's batch_from_starts; windows past the data give
 *   zeros and set RT_STATUS_INDEX_RANGE.
 * ------------------------------------------------------------------------------------------- */
int rt_embedding_forward(const uint8_t *packed, int64_t ldp, const float *scale, int max_code,
                         const int64_t *tokens, int64_t n_tok, int64_t rows, int64_t dim,
                         float *out, int64_t ldo, void *stream);
int64_t rt_embedding_update_workspace_bytes(int64_t n_tok, int64_t dim);
int rt_embedding_ratchet_update(const float *grad, int64_t ldg, const int64_t *sorted_tokens,
                                const int64_t *order, int64_t n_tok, int64_t rows, int64_t dim,
                                void *workspace, int64_t workspace_bytes, uint8_t *packed,
                                int64_t ldp, int8_t *code_out, int64_t ldc, float *rms_ema,
                                double ema_beta, int max_code, int threshold, double bucket_low,
                                double bucket_high, double eps, int64_t *counts, float *rms_sum,
                                void *stream);
int rt_token_windows(const uint16_t *data, int64_t n, const int64_t *starts, int64_t batch,
                     int64_t block, int64_t *inputs, int64_t *targets, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* RATCHET_B200_H */
