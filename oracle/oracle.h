/*
 * oracle.h — CPU restatement of the op sequences Magma's LazyTensor graph runs
 * for the training-step hot path (LayerNorm, attention, Linear, Adam and the
 * glue ops). TEST INFRASTRUCTURE ONLY: the checker that the sm_100a kernels in
 * libmagma_cuda.so are compared against, and the timed CPU baseline. Nothing in
 * the product path links, loads or calls this library.
 *
 * Every function follows the reference's op order with F32 intermediates
 * materialised the way the emitted StableHLO program has them; each cites the
 * reference file:line it restates (paths within pedronahum/Magma). Pinned
 * against the reference's own known-answer tests (see tests/test_oracle.py).
 * LayerNorm backward and attention backward have no known-answer test in the
 * reference: for those two the restatement of the autodiff chain is the only
 * oracle (parity unpinned by reference fixtures).
 */
#ifndef MAGMA_ORACLE_H_
#define MAGMA_ORACLE_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

void oracle_set_threads(int n);
int oracle_get_threads(void);

/* c[m,n] = sum_k opA[m,k] opB[k,n]; trans flags as in magma_gemm. */
void oracle_matmul(const float* a, const float* b, float* c, int64_t m, int64_t n, int64_t k,
                   int trans_a, int trans_b);

void oracle_layernorm_fwd(const float* x, const float* gamma, const float* beta, float* y,
                          float* mean, float* rstd, int64_t rows, int64_t dim, float eps);
void oracle_layernorm_bwd(const float* dy, const float* x, const float* gamma, float* dx,
                          float* dgamma, float* dbeta, int64_t rows, int64_t dim, float eps);

/* nn.LayerNorm's backward chain (variance through vjpVariance). */
void oracle_layernorm_module_bwd(const float* dy, const float* x, const float* gamma, float* dx,
                                 float* dgamma, float* dbeta, int64_t rows, int64_t dim,
                                 float eps);

/* Primitives of those chains on [rows, cols]; axis 0: over rows, 1: over
 * columns, 2: over both. */
void oracle_variance_fwd(const float* x, float* out, int64_t rows, int64_t cols, int axis,
                         int unbiased);
void oracle_variance_vjp(const float* x, const float* v, float* dx, int64_t rows, int64_t cols,
                         int axis, int unbiased);
void oracle_softmax_fwd(const float* x, float* s, int64_t rows, int64_t cols, int axis);
void oracle_softmax_vjp(const float* s, const float* v, float* dx, int64_t rows, int64_t cols,
                        int axis);
void oracle_masked_fill_fwd(const float* x, const float* mask, const float* value, float* out,
                            int64_t n);
void oracle_masked_fill_vjp(const float* mask, const float* v, float* dx, float* dvalue,
                            int64_t n);

/* Q,K,V,O contiguous [batch, heads, seq, hd]. probs (optional) receives the
 * softmax [batch, heads, seq, seq]; lse (optional) the row log-sum-exp. */
void oracle_attention_fwd(const float* q, const float* k, const float* v, float* o, float* probs,
                          float* lse, int64_t batch, int64_t heads, int64_t seq, int64_t hd,
                          float scale, int causal);
void oracle_attention_bwd(const float* q, const float* k, const float* v, const float* d_o,
                          float* dq, float* dk, float* dv, int64_t batch, int64_t heads,
                          int64_t seq, int64_t hd, float scale, int causal);

/* The same chain with the probabilities and the softmax cotangent rounded to
 * BF16 before their contractions and the row term taken from the stored
 * output o (all inputs BF16 values carried as F32). */
void oracle_attention_bwd_bf16(const float* q, const float* k, const float* v, const float* o,
                               const float* d_o, float* dq, float* dk, float* dv, int64_t batch,
                               int64_t heads, int64_t seq, int64_t hd, float scale, int causal);

void oracle_adam(float* p, const float* g, float* m, float* v, int64_t n, float lr, float beta1,
                 float beta2, float eps, float weight_decay, int64_t step, float grad_scale);
/* Global gradient norm, clipped Adam and warmup-cosine LR (Optimizer.swift:
 * 1229-1267, 766-803). */
float oracle_grad_norm(const float* g, int64_t n, float grad_scale);
void oracle_adam_clipped(float* p, const float* g, float* m, float* v, int64_t n, float lr,
                         float beta1, float beta2, float eps, float weight_decay, int64_t step,
                         float grad_scale, float norm, float max_norm);
float oracle_lr_warmup_cosine(float base_lr, float min_lr, int64_t warmup, int64_t total,
                              int64_t step);

void oracle_gelu_fwd(const float* x, float* y, int64_t n);
void oracle_gelu_bwd(const float* x, const float* dy, float* dx, int64_t n);

/* Mean softmax cross-entropy over rows; dlogits (optional) = d loss / d logits. */
float oracle_cross_entropy(const float* logits, const int32_t* targets, float* dlogits,
                           int64_t rows, int64_t classes);

/* allReduceMean over `replicas` buffers of `count` floats into out. */
void oracle_allreduce_mean(const float* const* bufs, int replicas, int64_t count, float* out);

/* ---- GPT (pre-LN decoder, main.swift:437-498) ---------------------------- */
typedef struct {
  int64_t vocab, vocab_padded, seq, layers, heads, dim;
  int32_t tied; /* 1: lm-head weight is wte */
} oracle_gpt_config;

/* Number of floats in the parameter arena and the offset of tensor `idx`
 * (order: wte, wpe, per layer [ln1_w, ln1_b, qkv_w, qkv_b, proj_w, proj_b,
 * ln2_w, ln2_b, fc_w, fc_b, fcproj_w, fcproj_b], lnf_w, lnf_b, [lm_head]);
 * every offset is a multiple of 64 floats. */
int64_t oracle_gpt_param_count(const oracle_gpt_config* cfg);
int64_t oracle_gpt_num_tensors(const oracle_gpt_config* cfg);
int64_t oracle_gpt_param_offset(const oracle_gpt_config* cfg, int64_t idx);

/* Forward + backward of one batch: returns the mean loss, writes the gradient
 * arena (same layout as params). tokens/targets [batch*seq]. */
float oracle_gpt_fwd_bwd(const oracle_gpt_config* cfg, const float* params, float* grads,
                         const int32_t* tokens, const int32_t* targets, int64_t batch);

/* ---- MLP classifier (784-128-10, ReLU, softmax CE) -------------------------
 * params: w1 [in,hid], b1 [hid], w2 [hid,out], b2 [out] (value Linear x.W+b,
 * ValueLayers.swift:38-41). Returns the mean loss, writes grads. */
float oracle_mlp_fwd_bwd(const float* params, float* grads, const float* x, const int32_t* labels,
                         int64_t batch, int64_t in, int64_t hid, int64_t out);

/* The reference's Examples/ValueLayers program: 1->16->1 ReLU MLP fitting
 * y = x^2 on 9 points with value Adam (lr 0.05). losses[i] is the loss after
 * i updates, for i in [0, steps]. */
void oracle_value_layers_example(int steps, float* losses);

#ifdef __cplusplus
}
#endif

#endif /* MAGMA_ORACLE_H_ */
