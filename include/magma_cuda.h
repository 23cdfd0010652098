/*
 * magma_cuda.h — C ABI of libmagma_cuda.so, the sm_100a (B200) execution
 * backend for the fused ops that Magma's LazyTensor graph emits for a
 * training step: LayerNorm fwd/bwd, causal attention fwd/bwd, the Linear
 * contraction (GEMM), the generic Adam update, and the glue ops on the same
 * graphs (embedding, softmax cross-entropy, GELU/ReLU, bias gradient,
 * dtype conversion).
 *
 * Conventions follow Magma's PJRT C shim
 * (Sources/CXLARuntime/include/PJRTSimpleWrapper.h):
 *   - every entry point returns a status code whose values are those of
 *     SW_PJRT_Error_Code (PJRTSimpleWrapper.h:32-50);
 *   - dtypes use the values of SW_PJRT_Buffer_Type (PJRTSimpleWrapper.h:52-71),
 *     so F32 = 10 and BF16 = 12 on both sides of the boundary;
 *   - a failing call records a message in thread-local storage, read with
 *     magma_get_last_error_message() and cleared with
 *     magma_clear_last_error_message() (PJRTSimpleWrapper.h:86-99);
 *   - buffers are plain device pointers owned by the caller, who allocates
 *     and frees them (as with PJRT_CreateBuffer / PJRT_DestroyBuffer,
 *     PJRTSimpleWrapper.h:174-232). Outputs are written into caller-provided
 *     buffers. Ops that need scratch memory take a caller-provided workspace
 *     and export a *_workspace_size query; the library never allocates device
 *     memory on an op path;
 *   - every op is asynchronous on the `stream` argument (a cudaStream_t passed
 *     as void*; NULL is the legacy default stream). Calls on distinct streams
 *     from distinct threads are independent.
 *
 * Layouts are row-major. Integer sizes are int64_t; strides are in elements.
 */
#ifndef MAGMA_CUDA_H_
#define MAGMA_CUDA_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define MAGMA_API __attribute__((visibility("default")))
#else
#define MAGMA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes: values of SW_PJRT_Error_Code (PJRTSimpleWrapper.h:32-50) */
typedef int32_t magma_status_t;
#define MAGMA_OK 0
#define MAGMA_CANCELLED 1
#define MAGMA_UNKNOWN 2
#define MAGMA_INVALID_ARGUMENT 3
#define MAGMA_DEADLINE_EXCEEDED 4
#define MAGMA_NOT_FOUND 5
#define MAGMA_RESOURCE_EXHAUSTED 8
#define MAGMA_FAILED_PRECONDITION 9
#define MAGMA_OUT_OF_RANGE 11
#define MAGMA_UNIMPLEMENTED 12
#define MAGMA_INTERNAL 13
#define MAGMA_UNAVAILABLE 14

/* ---- dtypes: values of SW_PJRT_Buffer_Type (PJRTSimpleWrapper.h:52-71) */
typedef int32_t magma_dtype_t;
#define MAGMA_DTYPE_S32 3
#define MAGMA_DTYPE_S64 4
#define MAGMA_DTYPE_F32 10
#define MAGMA_DTYPE_BF16 12

/* ---- GEMM epilogues (fused into the contraction's store) */
#define MAGMA_EPI_NONE 0          /* c = acc                                   */
#define MAGMA_EPI_BIAS 1          /* c = acc + bias[col]                       */
#define MAGMA_EPI_BIAS_GELU 2     /* aux_out = acc + bias; c = gelu(aux_out)   */
#define MAGMA_EPI_BIAS_RESIDUAL 3 /* c = aux_in + (acc + bias[col]); aux_in f32 */
#define MAGMA_EPI_DGELU 4         /* c = acc * gelu'(aux_in)                   */
#define MAGMA_EPI_ACCUMULATE 5    /* c = c + acc  (c must be f32)              */
#define MAGMA_EPI_BIAS_RELU 6     /* aux_out = acc + bias; c = relu(aux_out)   */
#define MAGMA_EPI_DRELU 7         /* c = acc * (aux_in > 0)                    */
#define MAGMA_EPI_ROWSTATS 8      /* c = acc; aux_out: softmax partials (below) */
/* MAGMA_EPI_ROWSTATS (BF16 operands, tensor-core path, no K split): besides
 * storing c, writes for every row r and every 64-column chunk j of c the pair
 * (max_j, sum over the chunk of exp(c - max_j)), computed from c as stored
 * (rounded to c's dtype), to aux_out as float2 [ceil(n / 64)][m] (chunk-major).
 * magma_cross_entropy_fwd_bwd_rowstats consumes them: the lm-head GEMM and the
 * softmax cross-entropy then read the logits once instead of twice. */

/* ---- errors (PJRTSimpleWrapper.h:86-99) ------------------------------------ */

/* Message of the most recent failure on the calling thread, or NULL. */
MAGMA_API const char* magma_get_last_error_message(void);
/* Clears the calling thread's last error message. */
MAGMA_API void magma_clear_last_error_message(void);
/* ABI version of this header (major*10000 + minor*100 + patch). */
MAGMA_API int32_t magma_abi_version(void);

/* ---- runtime: device, streams, memory (the PJRTClient/PJRTBuffer surface of
 *      Sources/XLARuntime/XLARuntime.swift:407-923, without XLA) ------------- */

MAGMA_API magma_status_t magma_device_count(int32_t* count);
/* Makes `device_ordinal` current on the calling thread and checks that it is an
 * sm_100 device; records the device's SM count for grid sizing. */
MAGMA_API magma_status_t magma_init(int32_t device_ordinal);
MAGMA_API magma_status_t magma_stream_create(void** stream);
MAGMA_API magma_status_t magma_stream_destroy(void* stream);
MAGMA_API magma_status_t magma_stream_synchronize(void* stream);
MAGMA_API magma_status_t magma_malloc(void** ptr, size_t bytes);
MAGMA_API magma_status_t magma_free(void* ptr);
/* Asynchronous copies on `stream`; synchronize the stream before reading. */
MAGMA_API magma_status_t magma_memcpy_h2d(void* dst, const void* src, size_t bytes, void* stream);
MAGMA_API magma_status_t magma_memcpy_d2h(void* dst, const void* src, size_t bytes, void* stream);
MAGMA_API magma_status_t magma_memset(void* dst, int32_t value, size_t bytes, void* stream);
/* Synchronizes `stream`, then reads and clears the device-side error word
 * that kernels with bounded waits set when a wait times out. Returns
 * MAGMA_DEADLINE_EXCEEDED (and the kernel's code in *code) if one did. */
MAGMA_API magma_status_t magma_device_error_check(void* stream, int32_t* code);

/* ---- LayerNorm ---------------------------------------------------------------
 * Replaces nn.LayerNorm.forward (Sources/Core/Module.swift:2754-2791) and the
 * GPT block's layerNorm (Benchmarks/GPT2Shakespeare/Sources/main.swift:364-375):
 *   mean = sum(x)/D; var = sum((x-mean)^2)/D; std = sqrt(var + eps);
 *   y = ((x - mean) / std) * gamma + beta.
 * x [rows, dim] in x_dtype (F32|BF16); y in y_dtype (F32|BF16); gamma, beta,
 * mean[rows], rstd[rows] = 1/std are F32. */
MAGMA_API magma_status_t magma_layernorm_fwd(const void* x, const float* gamma, const float* beta,
                                   void* y, float* mean, float* rstd,
                                   int64_t rows, int64_t dim, float eps,
                                   magma_dtype_t x_dtype, magma_dtype_t y_dtype,
                                   void* stream);

/* Bytes of workspace magma_layernorm_bwd needs for (rows, dim). */
MAGMA_API size_t magma_layernorm_bwd_workspace_size(int64_t rows, int64_t dim);

/* Replaces the autodiff chain of the LayerNorm above (vjpDivide, vjpSqrt,
 * vjpMeanDims, vjpMultiply/vjpAdd with sumAlongBroadcastDims:
 * Sources/Core/Autodiff.swift:57-94,221-257,351-370, Optimizer.swift:627-633):
 *   dx = rstd * (g - mean(g) - xhat * mean(g * xhat)), g = dy*gamma;
 *   dgamma = sum_rows dy*xhat; dbeta = sum_rows dy (fixed summation order).
 * accumulate_dx != 0 adds into dx (dx must then be F32); accumulate_params != 0
 * adds into dgamma/dbeta. */
MAGMA_API magma_status_t magma_layernorm_bwd(const void* dy, const void* x, const float* gamma,
                                   const float* mean, const float* rstd,
                                   void* dx, float* dgamma, float* dbeta,
                                   int64_t rows, int64_t dim,
                                   magma_dtype_t dy_dtype, magma_dtype_t x_dtype,
                                   magma_dtype_t dx_dtype,
                                   int32_t accumulate_dx, int32_t accumulate_params,
                                   void* workspace, size_t workspace_bytes, void* stream);

/* Allocation-free variant of magma_layernorm_bwd (no counterpart in the
 * reference: Magma's own runtime always hands XLA a buffer pool).
 *
 * For callers that cannot allocate device memory for the per-CTA dgamma/dbeta
 * partial sums: a plugin whose host framework owns all device memory and has no
 * allocation hook for it, code running inside an existing stream capture or a
 * real-time step loop where a cudaMalloc would synchronise the device, or a
 * caller working inside a fixed memory budget. Same arguments and results as
 * magma_layernorm_bwd, without the workspace: the partial sums go to a
 * scratch array compiled into the library (2.3 MiB on every GPU that loads the
 * library, held until the process exits). Limits: dim <= 1024 (larger dims
 * return MAGMA_INVALID_ARGUMENT; use magma_layernorm_bwd with a workspace).
 * The first call on a device looks up the scratch array's device address
 * (cudaGetSymbolAddress) — make that first call before any stream capture.
 * Every call on a device shares the one scratch array: calls that overlap on
 * the GPU (on different streams without ordering) race and give wrong sums;
 * order them on one stream. Each call writes every scratch entry it later
 * reads, so nothing carried over from the previous call is used. Calls no
 * cudaMalloc, cudaFree or allocating library routine. */
MAGMA_API magma_status_t magma_layernorm_bwd_noalloc(const void* dy, const void* x,
                                   const float* gamma, const float* mean, const float* rstd,
                                   void* dx, float* dgamma, float* dbeta,
                                   int64_t rows, int64_t dim,
                                   magma_dtype_t dy_dtype, magma_dtype_t x_dtype,
                                   magma_dtype_t dx_dtype,
                                   int32_t accumulate_dx, int32_t accumulate_params,
                                   void* stream);

/* LayerNorm backward into a pre-LN residual stream (no single counterpart in
 * the reference; it fuses three of the ops its traced GPT step emits after the
 * LayerNorm VJP: the gradient add into the residual branch, the BF16 cast of
 * that gradient for the next matmuls, and the bias-gradient column sum of the
 * Linear whose output the residual stream receives, Autodiff.swift:221-257).
 * As magma_layernorm_bwd with x and dx F32, plus:
 *   dx_bf16 (optional, [rows, dim] BF16): a copy of the final dx;
 *   dcol (optional, [dim] F32): column sums of the final dx over the rows,
 *   written or (accumulate_params) added like dgamma and dbeta.
 * dim % 8 == 0, dim <= 1024, 16-byte aligned dy, x, gamma, dx, dx_bf16.
 * Workspace: magma_layernorm_bwd_residual_workspace_size(rows, dim). */
MAGMA_API size_t magma_layernorm_bwd_residual_workspace_size(int64_t rows, int64_t dim);
MAGMA_API magma_status_t magma_layernorm_bwd_residual(const void* dy, const float* x,
                                   const float* gamma, const float* mean, const float* rstd,
                                   float* dx, void* dx_bf16, float* dgamma, float* dbeta,
                                   float* dcol, int64_t rows, int64_t dim,
                                   magma_dtype_t dy_dtype, int32_t accumulate_dx,
                                   int32_t accumulate_params, void* workspace,
                                   size_t workspace_bytes, void* stream);

/* ---- Linear contraction (GEMM) ------------------------------------------------
 * Replaces Tensor.matmul -> stablehlo.dot (Sources/Core/Tensor.swift:1102-1121,
 * Sources/StableHLO/Builder/MLIRBuilder.swift:372-378) as used by value Linear
 * (ValueLayers.swift:38-41, x.W + b), nn.Linear (Module.swift:266-300,
 * x.W^T + b), the GPT linear (main.swift:353-362), and their VJPs
 * (Autodiff.swift:177-191): c[m,n] = sum_k opA[m,k] * opB[k,n], then the
 * epilogue.
 *   trans_a = 0: A stored [m, k] (lda >= k); 1: A stored [k, m] (lda >= m).
 *   trans_b = 0: B stored [k, n] (ldb >= n); 1: B stored [n, k] (ldb >= k).
 *   c stored [m, n] (ldc >= n). ab_dtype F32 or BF16; BF16 runs on the tcgen05
 *   tensor cores with F32 accumulation; F32 runs on the same tensor cores
 *   through a three-term BF16 split of both operands when m*n*k >= 2^27 and
 *   the workspace holds the split (else, and for ROWSTATS, an F32 FFMA kernel).
 *   c_dtype F32 or BF16. bias is F32 [n]. aux_in / aux_out are [m, n] with
 *   leading dimension ldc: aux_in F32 for BIAS_RESIDUAL, else c_dtype-typed
 *   pre-activations; aux_out has c_dtype.
 * BF16 operands need 16-byte aligned base pointers and leading dimensions that
 * are multiples of 8 elements (TMA). */
MAGMA_API size_t magma_gemm_workspace_size(int64_t m, int64_t n, int64_t k, magma_dtype_t ab_dtype);
MAGMA_API magma_status_t magma_gemm(const void* a, const void* b, void* c,
                          int64_t m, int64_t n, int64_t k,
                          int64_t lda, int64_t ldb, int64_t ldc,
                          int32_t trans_a, int32_t trans_b,
                          magma_dtype_t ab_dtype, magma_dtype_t c_dtype,
                          int32_t epilogue, const float* bias,
                          const void* aux_in, void* aux_out,
                          void* workspace, size_t workspace_bytes, void* stream);

/* ---- causal scaled-dot-product attention -----------------------------------
 * Replaces nn.scaledDotProductAttention (Module.swift:2408-2441) and the GPT
 * block's attention (main.swift:467-481): S = (Q K^T) * scale, masked entries
 * (key > query when causal) set to -1e9 (main.swift:793-801), P = softmax(S),
 * O = P V. Q, K, V, O have logical shape [batch, heads, seq, head_dim]; element
 * (b, h, s, d) lives at base + b*strides[0] + h*strides[1] + s*strides[2] + d.
 * qkv_strides applies to Q, K and V; o_strides to O and dO (and dQ/dK/dV use
 * qkv_strides). lse [batch, heads, seq] F32 receives the row log-sum-exp of the
 * scaled, masked scores. dtype F32 or BF16; head_dim 64 (BF16) or <= 128 (F32). */
MAGMA_API magma_status_t magma_attention_fwd(const void* q, const void* k, const void* v,
                                   void* o, float* lse,
                                   int64_t batch, int64_t heads, int64_t seq, int64_t head_dim,
                                   const int64_t* qkv_strides, const int64_t* o_strides,
                                   float scale, int32_t causal, magma_dtype_t dtype,
                                   void* stream);

MAGMA_API size_t magma_attention_bwd_workspace_size(int64_t batch, int64_t heads, int64_t seq,
                                          int64_t head_dim, magma_dtype_t dtype);

/* Replaces the attention VJP chain (vjpBatchedMatmul Autodiff.swift:309-317,
 * vjpSoftmax :379-386, the scale multiply VJP :76-82, mask add VJP): with
 * P recomputed from lse, dV = P^T dO; dP = dO V^T; dS = P * (dP - rowsum(dO*O));
 * dQ = scale * dS K; dK = scale * dS^T Q. */
MAGMA_API magma_status_t magma_attention_bwd(const void* q, const void* k, const void* v,
                                   const void* o, const void* d_o, const float* lse,
                                   void* dq, void* dk, void* dv,
                                   int64_t batch, int64_t heads, int64_t seq, int64_t head_dim,
                                   const int64_t* qkv_strides, const int64_t* o_strides,
                                   float scale, int32_t causal, magma_dtype_t dtype,
                                   void* workspace, size_t workspace_bytes, void* stream);

/* ---- Adam -----------------------------------------------------------------
 * Replaces optim.Adam.step (Sources/Core/Optimizer.swift:354-412) and the value
 * Adam.update (Sources/Core/TangentOptimizer.swift:99-135), element-wise over a
 * flat F32 arena, in the reference's op order:
 *   g = grad * grad_scale;
 *   if weight_decay: p = p - p * (lr*weight_decay);
 *   m = m*beta1 + g*(1-beta1);  v = v*beta2 + (g*g)*(1-beta2);
 *   p = p - (m/bc1) / (sqrt(v/bc2) + eps) * lr,  bc_i = 1 - beta_i^step (F32).
 * step counts from 1. If shadow_bf16 is non-NULL the updated parameters are
 * also written there rounded to BF16 (round-to-nearest-even). */
MAGMA_API magma_status_t magma_adam_step(float* params, const float* grads, float* m, float* v,
                               void* shadow_bf16, int64_t n,
                               float lr, float beta1, float beta2, float eps,
                               float weight_decay, int64_t step, float grad_scale,
                               void* stream);

/* Same update over `count` separate tensors in one launch (multi-tensor apply);
 * the pointer and size arrays are host arrays. */
MAGMA_API magma_status_t magma_adam_step_multi(float* const* params, const float* const* grads,
                                     float* const* m, float* const* v,
                                     const int64_t* sizes, int32_t count,
                                     float lr, float beta1, float beta2, float eps,
                                     float weight_decay, int64_t step, float grad_scale,
                                     void* stream);

/* Global L2 norm of a gradient arena, as optim.clipGradNorm forms it
 * (Sources/Core/Optimizer.swift:1229-1247; applied by the GPT trainer before
 * every Adam step, Benchmarks/GPT2Shakespeare/Sources/main.swift:857):
 * norm[0] = sqrt(sum_i (grads[i] * grad_scale)^2), grad_scale being the 1/n of
 * a data-parallel mean. norm is a device F32 scalar. workspace holds per-block
 * partial sums: at least magma_grad_norm_workspace_size(n) bytes, 4-byte
 * aligned, on the device. The sum is taken in a fixed order, so the result is
 * the same on every run on the same GPU model. */
MAGMA_API int64_t magma_grad_norm_workspace_size(int64_t n);
MAGMA_API magma_status_t magma_grad_norm(const float* grads, int64_t n, float grad_scale,
                                         float* norm, void* workspace, int64_t workspace_bytes,
                                         void* stream);

/* The pieces of magma_grad_norm for a gradient sharded over ranks: each rank
 * writes the sum of squares of its (scaled) part to a device scalar
 * (magma_grad_sumsq, same workspace as magma_grad_norm), the ranks gather
 * those scalars (magma_all_gather), and magma_grad_norm_combine adds `count`
 * of them in index order and takes the square root, so every rank computes the
 * same norm. */
MAGMA_API magma_status_t magma_grad_sumsq(const float* grads, int64_t n, float grad_scale,
                                          float* sumsq, void* workspace, int64_t workspace_bytes,
                                          void* stream);
MAGMA_API magma_status_t magma_grad_norm_combine(const float* sumsq, int64_t count, float* norm,
                                                 void* stream);

/* Adam with global-norm clipping fused in front (clipGradNorm's scaling,
 * Optimizer.swift:1249-1267, then optim.Adam.step, :354-412): with
 * c = max_norm / (norm + 1e-6) if that is below 1, else 1 (also 1 for a NaN
 * norm), the gradient is g = (grad * grad_scale) * c, then the update of
 * magma_adam_step. grad_norm is the device scalar magma_grad_norm wrote; it is
 * read on the device, so no host synchronisation sits between the two calls. */
MAGMA_API magma_status_t magma_adam_step_clipped(float* params, const float* grads, float* m,
                                                 float* v, void* shadow_bf16, int64_t n,
                                                 float lr, float beta1, float beta2, float eps,
                                                 float weight_decay, int64_t step,
                                                 float grad_scale, const float* grad_norm,
                                                 float max_norm, void* stream);

/* Learning rate of optim.WarmupCosineScheduler (Optimizer.swift:766-803) at
 * scheduler step `step` (0 for the first training step; clamped to
 * total_steps as the scheduler's step() clamps): linear warmup
 * base_lr * (step + 1) / warmup_steps, then min_lr + (base_lr - min_lr) *
 * (1 + cos(pi * progress)) / 2. F32 arithmetic in the reference's order; host
 * only (no device work). Requires 0 <= warmup_steps < total_steps. */
MAGMA_API magma_status_t magma_lr_warmup_cosine(float base_lr, float min_lr, int64_t warmup_steps,
                                                int64_t total_steps, int64_t step, float* lr);

/* ---- glue ops on the same graphs ------------------------------------------ */

/* Token + position embedding gather (Sources/Core/Data.swift:856-886, GPT
 * main.swift:454-458): out[b*seq+s, :] = wte[tokens[b*seq+s], :] + wpe[s, :].
 * wte [vocab, dim], wpe [>=seq, dim], out [batch*seq, dim]; all F32.
 * Out-of-range token ids are an error recorded in the device error word. */
MAGMA_API magma_status_t magma_embedding_fwd(const int32_t* tokens, const float* wte, const float* wpe,
                                   float* out, int64_t batch, int64_t seq, int64_t dim,
                                   int64_t vocab, void* stream);

/* Embedding VJP (the one-hot matmul of Data.swift:890-907, as a scatter-add):
 * dwte[tokens[r], :] += dout[r, :]; dwpe[s, :] += sum_b dout[b*seq+s, :].
 * Both accumulate into their outputs (F32). dwpe may be NULL. */
MAGMA_API magma_status_t magma_embedding_bwd(const int32_t* tokens, const float* dout,
                                   float* dwte, float* dwpe,
                                   int64_t batch, int64_t seq, int64_t dim, int64_t vocab,
                                   void* stream);

/* The same VJP with a fixed summation order: each token row of dwte gets the
 * rows that hold that token added one at a time in increasing row order
 * (dwte accumulates; dwpe, if not NULL, is added to when accumulate_dwpe != 0
 * and written otherwise), so
 * the result is identical on every run (the one-hot matmul of
 * Data.swift:890-907 reduces in an order the compiler picks; this order is the
 * plain sequential one). The rows are put in (token, row) order (1024-row
 * chunks sorted in shared memory, then ranked across chunks), and one warp per
 * token adds the token's rows. workspace:
 * magma_embedding_bwd_workspace_size(batch, seq) bytes of device memory (12
 * bytes per row, rows rounded up to a multiple of 1024), 16-byte aligned.
 * vocab must be below 4194303. */
MAGMA_API int64_t magma_embedding_bwd_workspace_size(int64_t batch, int64_t seq);
MAGMA_API magma_status_t magma_embedding_bwd_deterministic(const int32_t* tokens,
                                                           const float* dout, float* dwte,
                                                           float* dwpe, int64_t batch,
                                                           int64_t seq, int64_t dim, int64_t vocab,
                                                           int32_t accumulate_dwpe,
                                                           void* workspace,
                                                           int64_t workspace_bytes, void* stream);

/* Softmax cross-entropy with class-index targets, forward and backward in one
 * pass (main.swift:412-433, Loss.swift:627-699): for each row r of logits
 * [rows, classes] (leading dimension ld), losses[r] = logsumexp(row) -
 * row[targets[r]], and the row is overwritten in place with
 * grad_scale * (softmax(row) - onehot(targets[r])); columns in [classes, ld)
 * are set to zero. dtype F32 or BF16 (F32 math). */
MAGMA_API magma_status_t magma_cross_entropy_fwd_bwd(void* logits, const int32_t* targets, float* losses,
                                           int64_t rows, int64_t classes, int64_t ld,
                                           float grad_scale, magma_dtype_t dtype, void* stream);

/* As magma_cross_entropy_fwd_bwd for logits written by a MAGMA_EPI_ROWSTATS
 * GEMM with n = classes: row maxima and sums come from the GEMM's softmax
 * partials `stats` (float2 [ceil(classes / 64)][rows]), so each row is read
 * once (and written once with the gradient). Same outputs, BF16 logits. */
MAGMA_API magma_status_t magma_cross_entropy_fwd_bwd_rowstats(void* logits, const void* stats,
                                   const int32_t* targets, float* losses, int64_t rows,
                                   int64_t classes, int64_t ld, float grad_scale,
                                   magma_dtype_t dtype, void* stream);

/* Deterministic sum of n F32 values into out[0] (e.g. the mean loss with
 * scale = 1/n). */
MAGMA_API magma_status_t magma_reduce_sum(const float* x, float* out, int64_t n, float scale, void* stream);

/* Mean-squared error as the reference's value-layer example writes it
 * (Examples/ValueLayers/main.swift: r = pred - target; loss = sum(r*r) / n)
 * and its VJP (Autodiff.swift: divide, sum and multiply pullbacks):
 * loss[0] = sum_i (pred_i - target_i)^2 / divisor and, if dpred is not NULL,
 * dpred_i = v*r_i + v*r_i with v = 1/divisor. F32, n elements. */
MAGMA_API magma_status_t magma_mse_fwd_bwd(const float* pred, const float* target, float* dpred,
                                           float* loss, int64_t n, float divisor, void* stream);

/* GELU (tanh form, StableHLOEmitter.swift:804-816) and its VJP
 * (Autodiff.swift:401-418), element-wise; dtype F32 or BF16. */
MAGMA_API magma_status_t magma_gelu_fwd(const void* x, void* y, int64_t n, magma_dtype_t dtype, void* stream);
MAGMA_API magma_status_t magma_gelu_bwd(const void* x, const void* dy, void* dx, int64_t n,
                              magma_dtype_t dtype, void* stream);
/* ReLU (Tensor.swift:1386) and its VJP (Autodiff.swift:119-135). */
MAGMA_API magma_status_t magma_relu_fwd(const void* x, void* y, int64_t n, magma_dtype_t dtype, void* stream);
MAGMA_API magma_status_t magma_relu_bwd(const void* x, const void* dy, void* dx, int64_t n,
                              magma_dtype_t dtype, void* stream);

/* Bias gradient: dbias[c] (+)= sum_r dy[r, c] over dy [rows, cols] (leading
 * dimension ld) in a fixed order (sumAlongBroadcastDims, Autodiff.swift:221-257).
 * dy F32 or BF16; dbias F32. */
MAGMA_API size_t magma_bias_grad_workspace_size(int64_t rows, int64_t cols);
MAGMA_API magma_status_t magma_bias_grad(const void* dy, float* dbias, int64_t rows, int64_t cols,
                               int64_t ld, magma_dtype_t dtype, int32_t accumulate,
                               void* workspace, size_t workspace_bytes, void* stream);

/* dtype conversion (Tensor.swift:2069-2130; F32 -> BF16 rounds to nearest even
 * as LazyTensor.swift:1511-1516 does). */
MAGMA_API magma_status_t magma_convert(const void* src, void* dst, int64_t n,
                             magma_dtype_t src_dtype, magma_dtype_t dst_dtype, void* stream);

/* y = y * alpha (F32), e.g. the 1/n of allReduceMean (MLIRBuilder.swift:923-929)
 * applied after a sum all-reduce. */
MAGMA_API magma_status_t magma_scale(float* y, int64_t n, float alpha, void* stream);

/* ---- collectives (data-parallel exchange) -----------------------------------
 * The reference's replicated step crosses its C shim at PJRT_ExecuteMultiDevice
 * (Sources/CXLARuntime/PJRTSimpleWrapper.c:1412), with the gradient mean traced
 * as crossReplicaMean (Sources/Core/Distributed.swift:59-64) and lowered to
 * all_reduce(add) then a multiply by 1/n (MLIRBuilder.swift:923-929). These
 * entry points are that exchange over NCCL: one communicator per GPU, the
 * collective enqueued on the caller's stream. NCCL is opened at run time
 * (libnccl.so.2); without it every call returns MAGMA_UNAVAILABLE.
 * Communicators are non-blocking: initialisation and each enqueue wait at most
 * a bounded time for the other ranks (timeout_ms, or 120 s), then abort the
 * communicator and return MAGMA_DEADLINE_EXCEEDED. */
#define MAGMA_COMM_ID_BYTES 128
#define MAGMA_REDUCE_SUM 0
#define MAGMA_REDUCE_MAX 1
#define MAGMA_REDUCE_MIN 2
#define MAGMA_REDUCE_AVG 3

/* A new communicator id (rank 0 makes it; the caller hands the bytes to the
 * other ranks over its own channel). id: at least MAGMA_COMM_ID_BYTES bytes. */
MAGMA_API magma_status_t magma_comm_unique_id(uint8_t* id, size_t bytes);
/* Joins rank `rank` of `nranks` on the current device (one process or thread
 * per GPU). timeout_ms <= 0 means 120 s. */
MAGMA_API magma_status_t magma_comm_init_rank(void** comm, int32_t nranks, int32_t rank,
                                              const uint8_t* id, int64_t timeout_ms);
/* One communicator per listed device, all in this process (devices may be
 * NULL for 0..ndev-1); comms receives ndev handles. */
MAGMA_API magma_status_t magma_comm_init_all(int32_t ndev, const int32_t* devices, void** comms);
MAGMA_API magma_status_t magma_comm_destroy(void* comm);
/* Ends a communicator without waiting for its peers (after a failure). */
MAGMA_API magma_status_t magma_comm_abort(void* comm);
MAGMA_API magma_status_t magma_comm_size(void* comm, int32_t* nranks);
MAGMA_API magma_status_t magma_comm_rank(void* comm, int32_t* rank);
/* MAGMA_OK while the communicator is healthy; an error status (with the NCCL
 * reason in the last-error message) once it has failed, e.g. after a peer
 * died. Host-side; does not wait. */
MAGMA_API magma_status_t magma_comm_check(void* comm);
/* recv = reduce over ranks of send, count elements (in place when send ==
 * recv). op: MAGMA_REDUCE_*. dtype F32, BF16, S32 or S64. */
MAGMA_API magma_status_t magma_allreduce(const void* send, void* recv, int64_t count,
                                         magma_dtype_t dtype, int32_t op, void* comm,
                                         void* stream);
/* recv (recv_count elements) = this rank's block of the reduction of send
 * (nranks * recv_count elements, rank r owning [r*recv_count, (r+1)*recv_count)). */
MAGMA_API magma_status_t magma_reduce_scatter(const void* send, void* recv, int64_t recv_count,
                                              magma_dtype_t dtype, int32_t op, void* comm,
                                              void* stream);
/* recv (nranks * send_count elements) = every rank's send, in rank order. */
MAGMA_API magma_status_t magma_all_gather(const void* send, void* recv, int64_t send_count,
                                          magma_dtype_t dtype, void* comm, void* stream);
/* Brackets several collectives (e.g. one per device of magma_comm_init_all
 * from one thread) so that they are issued together. */
MAGMA_API magma_status_t magma_group_start(void);
MAGMA_API magma_status_t magma_group_end(void);

/* ---- events (ordering between streams, device timing) ---------------------- */
MAGMA_API magma_status_t magma_event_create(void** event, int32_t enable_timing);
MAGMA_API magma_status_t magma_event_destroy(void* event);
MAGMA_API magma_status_t magma_event_record(void* event, void* stream);
/* Work queued on `stream` after this call waits for the event. */
MAGMA_API magma_status_t magma_stream_wait_event(void* stream, void* event);
MAGMA_API magma_status_t magma_event_synchronize(void* event);
/* *done = 1 once the work before the event has finished, else 0. */
MAGMA_API magma_status_t magma_event_query(void* event, int32_t* done);
MAGMA_API magma_status_t magma_event_elapsed_ms(void* start, void* end, float* ms);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* MAGMA_CUDA_H_ */
