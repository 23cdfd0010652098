/*
 * oracle.c — CPU restatement of the reference's hot-path op sequences.
 *
 * TEST INFRASTRUCTURE ONLY (the checker and the timed CPU baseline); the
 * product path never links or calls it. F32 throughout, intermediates
 * materialised in the order the reference's lazy graph emits them, no FMA
 * contraction (-ffp-contract=off), OpenMP over independent rows/heads.
 * Each function names the reference file:line (pedronahum/Magma) it follows.
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

static int g_threads = 0;

void oracle_set_threads(int n) {
  g_threads = n;
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#endif
}

int oracle_get_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

static void* xmalloc(size_t n) {
  void* p = calloc(n ? n : 1, 1);
  if (!p) abort();
  return p;
}

/* c[i,:] += av * brow — the inner loop of every contraction. */
__attribute__((target_clones("avx2", "default")))
static void axpy_row(float* __restrict c, const float* __restrict b, float av, int64_t n) {
  for (int64_t j = 0; j < n; ++j) c[j] += av * b[j];
}

/* stablehlo.dot semantics (MLIRBuilder.swift:372-378): F32 products summed
 * over k in increasing order per output element. */
void oracle_matmul(const float* a, const float* b, float* c, int64_t m, int64_t n, int64_t k,
                   int trans_a, int trans_b) {
  const float* bk = b; /* [k, n] */
  float* bt = NULL;
  if (trans_b) {
    bt = (float*)xmalloc((size_t)k * n * sizeof(float));
#pragma omp parallel for schedule(static)
    for (int64_t p = 0; p < k; ++p)
      for (int64_t j = 0; j < n; ++j) bt[p * n + j] = b[j * k + p];
    bk = bt;
  }
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < m; ++i) {
    float* crow = c + i * n;
    memset(crow, 0, (size_t)n * sizeof(float));
    for (int64_t p = 0; p < k; ++p) {
      float av = trans_a ? a[p * m + i] : a[i * k + p];
      if (av != 0.0f) axpy_row(crow, bk + p * n, av, n);
    }
  }
  free(bt);
}

/* ---- LayerNorm ------------------------------------------------------------
 * Forward: main.swift:364-375 (== nn.LayerNorm.forward, Module.swift:2774-2784):
 *   mean = reduceMean(x) (sum / D, StableHLOEmitter.swift:781-788);
 *   centered = x - mean; variance = mean(centered*centered);
 *   std = sqrt(variance + eps); normalized = centered / std;
 *   y = normalized * w + b. */
void oracle_layernorm_fwd(const float* x, const float* gamma, const float* beta, float* y,
                          float* mean_out, float* rstd_out, int64_t rows, int64_t dim, float eps) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    const float* xr = x + r * dim;
    float s = 0.f;
    for (int64_t i = 0; i < dim; ++i) s += xr[i];
    const float mean = s / (float)dim;
    float ss = 0.f;
    for (int64_t i = 0; i < dim; ++i) {
      float c = xr[i] - mean;
      ss += c * c;
    }
    const float var = ss / (float)dim;
    const float stdv = sqrtf(var + eps);
    for (int64_t i = 0; i < dim; ++i) {
      float normalized = (xr[i] - mean) / stdv;
      y[r * dim + i] = normalized * gamma[i] + beta[i];
    }
    if (mean_out) mean_out[r] = mean;
    if (rstd_out) rstd_out[r] = 1.0f / stdv;
  }
}

/* Backward: the autodiff chain through the forward above —
 *   y = scaled + b          vjpAdd + sumAlongBroadcastDims (Autodiff.swift:57-63,221-257)
 *   scaled = normalized * w vjpMultiply (:76-82)
 *   normalized = centered / std   vjpDivide (:85-94): dc1 = v/std, dstd = sum(-v*result/std)
 *   std = sqrt(vpe)         vjpSqrt (Optimizer.swift:627-633): v*0.5/result
 *   variance = mean(sq)     vjpMeanDims (Autodiff.swift:351-370): v/D broadcast
 *   sq = centered*centered  vjpMultiply: v*centered + v*centered
 *   centered = x - mean     vjpSubtract (:66-73): dx1 = v, dmean = -sum(v)
 *   mean = mean(x)          vjpMeanDims: dmean/D broadcast. */
void oracle_layernorm_bwd(const float* dy, const float* x, const float* gamma, float* dx,
                          float* dgamma, float* dbeta, int64_t rows, int64_t dim, float eps) {
  float* pg = (float*)xmalloc((size_t)rows * dim * sizeof(float)); /* dy*normalized per row */
#pragma omp parallel
  {
    float* centered = (float*)xmalloc((size_t)dim * sizeof(float));
    float* normalized = (float*)xmalloc((size_t)dim * sizeof(float));
    float* dcent = (float*)xmalloc((size_t)dim * sizeof(float));
#pragma omp for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
      const float* xr = x + r * dim;
      const float* dyr = dy + r * dim;
      float s = 0.f;
      for (int64_t i = 0; i < dim; ++i) s += xr[i];
      const float mean = s / (float)dim;
      float ss = 0.f;
      for (int64_t i = 0; i < dim; ++i) {
        centered[i] = xr[i] - mean;
        ss += centered[i] * centered[i];
      }
      const float variance = ss / (float)dim;
      const float stdv = sqrtf(variance + eps);
      for (int64_t i = 0; i < dim; ++i) normalized[i] = centered[i] / stdv;
      /* normalized = centered / std */
      float dstd = 0.f;
      for (int64_t i = 0; i < dim; ++i) {
        float dnorm = dyr[i] * gamma[i];
        dcent[i] = dnorm / stdv;
        dstd += (-dnorm) * normalized[i] / stdv;
        pg[r * dim + i] = dyr[i] * normalized[i];
      }
      const float dvpe = dstd * 0.5f / stdv;
      const float dsq = dvpe / (float)dim;
      float dmean = 0.f;
      for (int64_t i = 0; i < dim; ++i) {
        dcent[i] = dcent[i] + dsq * centered[i] + dsq * centered[i];
        dmean += -dcent[i];
      }
      const float dmb = dmean / (float)dim;
      for (int64_t i = 0; i < dim; ++i) dx[r * dim + i] = dcent[i] + dmb;
    }
    free(centered);
    free(normalized);
    free(dcent);
  }
  /* dgamma / dbeta: sums over the broadcast (row) dimension. */
  if (dgamma || dbeta) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < dim; ++i) {
      float sg = 0.f, sb = 0.f;
      for (int64_t r = 0; r < rows; ++r) {
        sg += pg[r * dim + i];
        sb += dy[r * dim + i];
      }
      if (dgamma) dgamma[i] = sg;
      if (dbeta) dbeta[i] = sb;
    }
  }
  free(pg);
}

/* nn.LayerNorm's backward (Module.swift:2774-2784): the module takes the
 * variance through Tensor.variance(dims:unbiased:false), whose custom VJP
 * (vjpVariance, Autodiff.swift:576-592) returns v * centered * (2/N) without
 * a path through the mean, while the GPT block's layerNorm (main.swift:
 * 364-375, oracle_layernorm_bwd above) forms it as mean(centered*centered).
 * The two agree up to rounding (sum(centered) = 0). Chain per row:
 *   normalized = centered / std  vjpDivide: dcent = v/std, dstd = sum(-v*result/std)
 *   std = sqrt(var + eps)        vjpSqrt: v*0.5/result
 *   var = x.variance(...)        vjpVariance: dvar * centered * (2/N)
 *   centered = x - mean          vjpSubtract: dx += dcent, dmean = -sum(dcent)
 *   mean = x.mean(...)           vjpMeanDims: dmean / N broadcast. */
void oracle_layernorm_module_bwd(const float* dy, const float* x, const float* gamma, float* dx,
                                 float* dgamma, float* dbeta, int64_t rows, int64_t dim,
                                 float eps) {
  const float two_n = 2.0f / (float)dim;
  float* row_mean = (float*)xmalloc((size_t)rows * sizeof(float));
  float* row_std = (float*)xmalloc((size_t)rows * sizeof(float));
#pragma omp parallel
  {
    float* centered = (float*)xmalloc((size_t)dim * sizeof(float));
    float* dcent = (float*)xmalloc((size_t)dim * sizeof(float));
#pragma omp for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
      const float* xr = x + r * dim;
      const float* dyr = dy + r * dim;
      float s = 0.f;
      for (int64_t i = 0; i < dim; ++i) s += xr[i];
      const float mean = s / (float)dim;
      float ss = 0.f;
      for (int64_t i = 0; i < dim; ++i) {
        centered[i] = xr[i] - mean;
        ss += centered[i] * centered[i];
      }
      const float stdv = sqrtf(ss / (float)dim + eps);
      row_mean[r] = mean;
      row_std[r] = stdv;
      float dstd = 0.f;
      for (int64_t i = 0; i < dim; ++i) {
        const float normalized = centered[i] / stdv;
        const float dnorm = dyr[i] * gamma[i];
        dcent[i] = dnorm / stdv;
        dstd += (-dnorm) * normalized / stdv;
      }
      const float dvar = dstd * 0.5f / stdv;
      float dmean = 0.f;
      for (int64_t i = 0; i < dim; ++i) dmean += -dcent[i];
      const float dmb = dmean / (float)dim;
      for (int64_t i = 0; i < dim; ++i) dx[r * dim + i] = dcent[i] + dmb + dvar * centered[i] * two_n;
    }
    free(centered);
    free(dcent);
  }
  if (dgamma || dbeta) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < dim; ++i) {
      float sg = 0.f, sb = 0.f;
      for (int64_t r = 0; r < rows; ++r) {
        sg += dy[r * dim + i] * ((x[r * dim + i] - row_mean[r]) / row_std[r]);
        sb += dy[r * dim + i];
      }
      if (dgamma) dgamma[i] = sg;
      if (dbeta) dbeta[i] = sb;
    }
  }
  free(row_mean);
  free(row_std);
}

/* ---- reduction, softmax and masking primitives (2-D, row-major [rows, cols])
 * The pieces the LayerNorm and attention chains are made of, exported so that
 * the reference's own gradient checks of these primitives
 * (Tests/CoreTests/CrossModuleDifferentiabilityTests.swift) can be run on the
 * oracle. axis 0 reduces over rows (one result per column), axis 1 over
 * columns (one per row); axis 2 reduces over both (one result). */
static void reduce_geometry(int64_t rows, int64_t cols, int axis, int64_t* outer, int64_t* count,
                            int64_t* stride_out, int64_t* stride_in) {
  if (axis == 1) { *outer = rows; *count = cols; *stride_out = cols; *stride_in = 1; }
  else if (axis == 0) { *outer = cols; *count = rows; *stride_out = 1; *stride_in = cols; }
  else { *outer = 1; *count = rows * cols; *stride_out = 0; *stride_in = 1; }
}

/* Tensor.variance(dims:unbiased:) (Tensor.swift:2014-2043): meanVal = mean;
 * centered = x - meanVal; mean(centered*centered); times count/(count-1)
 * when unbiased and count > 1. out has one entry per reduced group. */
void oracle_variance_fwd(const float* x, float* out, int64_t rows, int64_t cols, int axis,
                         int unbiased) {
  int64_t outer, count, so, si;
  reduce_geometry(rows, cols, axis, &outer, &count, &so, &si);
  for (int64_t o = 0; o < outer; ++o) {
    const float* base = x + o * so;
    float s = 0.f;
    for (int64_t i = 0; i < count; ++i) s += base[i * si];
    const float mean = s / (float)count;
    float ss = 0.f;
    for (int64_t i = 0; i < count; ++i) {
      const float c = base[i * si] - mean;
      ss += c * c;
    }
    float var = ss / (float)count;
    if (unbiased && count > 1) var = var * ((float)count / (float)(count - 1));
    out[o] = var;
  }
}

/* vjpVariance (Autodiff.swift:576-592): dx = v * centered * (2/d), d = N-1
 * when unbiased and N > 1, else N; v has one entry per reduced group. */
void oracle_variance_vjp(const float* x, const float* v, float* dx, int64_t rows, int64_t cols,
                         int axis, int unbiased) {
  int64_t outer, count, so, si;
  reduce_geometry(rows, cols, axis, &outer, &count, &so, &si);
  const int64_t den = unbiased && count > 1 ? count - 1 : count;
  const float scale = 2.0f / (float)den;
  for (int64_t o = 0; o < outer; ++o) {
    const float* base = x + o * so;
    float s = 0.f;
    for (int64_t i = 0; i < count; ++i) s += base[i * si];
    const float mean = s / (float)count;
    for (int64_t i = 0; i < count; ++i) {
      const float c = base[i * si] - mean;
      dx[o * so + i * si] = v[o] * c * scale;
    }
  }
}

/* Softmax composite (StableHLOEmitter.swift:795-803: max, subtract, exp, sum,
 * divide) along axis 0 or 1 of a [rows, cols] tensor. */
void oracle_softmax_fwd(const float* x, float* s, int64_t rows, int64_t cols, int axis) {
  int64_t outer, count, so, si;
  reduce_geometry(rows, cols, axis, &outer, &count, &so, &si);
  for (int64_t o = 0; o < outer; ++o) {
    const float* xb = x + o * so;
    float* sb = s + o * so;
    float mx = -INFINITY;
    for (int64_t i = 0; i < count; ++i) mx = xb[i * si] > mx ? xb[i * si] : mx;
    float sum = 0.f;
    for (int64_t i = 0; i < count; ++i) {
      sb[i * si] = expf(xb[i * si] - mx);
      sum += sb[i * si];
    }
    for (int64_t i = 0; i < count; ++i) sb[i * si] = sb[i * si] / sum;
  }
}

/* vjpSoftmax (Autodiff.swift:379-386) along axis 0 or 1, given the softmax
 * output s and the cotangent v; the per-row form is what the attention
 * backward applies to its probabilities. */
void oracle_softmax_vjp(const float* s, const float* v, float* dx, int64_t rows, int64_t cols,
                        int axis) {
  int64_t outer, count, so, si;
  reduce_geometry(rows, cols, axis, &outer, &count, &so, &si);
  for (int64_t o = 0; o < outer; ++o) {
    float sumvs = 0.f;
    for (int64_t i = 0; i < count; ++i) sumvs += v[o * so + i * si] * s[o * so + i * si];
    for (int64_t i = 0; i < count; ++i) {
      const int64_t e = o * so + i * si;
      dx[e] = s[e] * (v[e] - sumvs);
    }
  }
}

/* maskedFill (Tensor.swift:1251-1262): out = mask != 0 ? value : x, and its
 * VJP (vjpMaskedFill, Autodiff.swift:601-613): dx = v * (1 - selected),
 * dvalue = v * selected (value of the same shape). The attention chains use
 * it as the causal mask (value -1e9; its cotangent is discarded). */
void oracle_masked_fill_fwd(const float* x, const float* mask, const float* value, float* out,
                            int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = mask[i] != 0.0f ? value[i] : x[i];
}
void oracle_masked_fill_vjp(const float* mask, const float* v, float* dx, float* dvalue,
                            int64_t n) {
  for (int64_t i = 0; i < n; ++i) {
    const float selected = mask[i] != 0.0f ? 1.0f : 0.0f;
    if (dx) dx[i] = v[i] * (1.0f - selected);
    if (dvalue) dvalue[i] = v[i] * selected;
  }
}

/* ---- attention ------------------------------------------------------------
 * main.swift:467-481 / Module.swift:2408-2441: scores = (q . k^T) * scale;
 * masked = scores + mask (0 or -1e9, main.swift:793-801); softmax composite
 * (StableHLOEmitter.swift:795-803): max, subtract, exp, sum, divide;
 * out = probs . v. lse (not a reference output) = max + log(sum). */
static void attention_probs_head(const float* q, const float* k, float* p, float* lse,
                                 int64_t seq, int64_t hd, float scale, int causal) {
  for (int64_t i = 0; i < seq; ++i) {
    float* pr = p + i * seq;
    float mx = -INFINITY;
    for (int64_t j = 0; j < seq; ++j) {
      float s = 0.f;
      for (int64_t d = 0; d < hd; ++d) s += q[i * hd + d] * k[j * hd + d];
      s = s * scale;
      s = s + ((causal && j > i) ? -1e9f : 0.0f);
      pr[j] = s;
      if (s > mx) mx = s;
    }
    float sum = 0.f;
    for (int64_t j = 0; j < seq; ++j) {
      pr[j] = expf(pr[j] - mx);
      sum += pr[j];
    }
    for (int64_t j = 0; j < seq; ++j) pr[j] = pr[j] / sum;
    if (lse) lse[i] = mx + logf(sum);
  }
}

void oracle_attention_fwd(const float* q, const float* k, const float* v, float* o, float* probs,
                          float* lse, int64_t batch, int64_t heads, int64_t seq, int64_t hd,
                          float scale, int causal) {
  const int64_t bh = batch * heads;
#pragma omp parallel
  {
    float* p = probs ? NULL : (float*)xmalloc((size_t)seq * seq * sizeof(float));
#pragma omp for schedule(dynamic)
    for (int64_t h = 0; h < bh; ++h) {
      const float* qh = q + h * seq * hd;
      const float* kh = k + h * seq * hd;
      const float* vh = v + h * seq * hd;
      float* ph = probs ? probs + h * seq * seq : p;
      attention_probs_head(qh, kh, ph, lse ? lse + h * seq : NULL, seq, hd, scale, causal);
      float* oh = o + h * seq * hd;
      for (int64_t i = 0; i < seq; ++i) {
        for (int64_t d = 0; d < hd; ++d) oh[i * hd + d] = 0.f;
        for (int64_t j = 0; j < seq; ++j) {
          float pv = ph[i * seq + j];
          for (int64_t d = 0; d < hd; ++d) oh[i * hd + d] += pv * vh[j * hd + d];
        }
      }
    }
    free(p);
  }
}

/* vjpSoftmax (Autodiff.swift:379-386) on one row of n entries:
 * dx = s * (v - sum(v * s)), the sum over the row in increasing order. */
static void softmax_vjp_row(const float* s, const float* v, float* dx, int64_t n) {
  float sumvs = 0.f;
  for (int64_t j = 0; j < n; ++j) sumvs += v[j] * s[j];
  for (int64_t j = 0; j < n; ++j) dx[j] = s[j] * (v[j] - sumvs);
}

/* VJP chain: vjpBatchedMatmul (Autodiff.swift:309-317): dP = dO.V^T, dV = P^T.dO;
 * vjpSoftmax (:379-386): dS = P*(dP - sum(dP*P)); mask add passes dS; scale
 * multiply (:76-82): dQK = dS*scale; dQ = dQK.K, dK = dQK^T.Q. Every output
 * element is a sum over its contraction index in increasing order; the loops
 * that accumulate whole rows keep that order per element. */
void oracle_attention_bwd(const float* q, const float* k, const float* v, const float* d_o,
                          float* dq, float* dk, float* dv, int64_t batch, int64_t heads,
                          int64_t seq, int64_t hd, float scale, int causal) {
  const int64_t bh = batch * heads;
#pragma omp parallel
  {
    float* p = (float*)xmalloc((size_t)seq * seq * sizeof(float));
    float* dp = (float*)xmalloc((size_t)seq * seq * sizeof(float));
#pragma omp for schedule(dynamic)
    for (int64_t h = 0; h < bh; ++h) {
      const float* qh = q + h * seq * hd;
      const float* kh = k + h * seq * hd;
      const float* vh = v + h * seq * hd;
      const float* doh = d_o + h * seq * hd;
      float* dqh = dq + h * seq * hd;
      float* dkh = dk + h * seq * hd;
      float* dvh = dv + h * seq * hd;
      attention_probs_head(qh, kh, p, NULL, seq, hd, scale, causal);
      for (int64_t i = 0; i < seq; ++i)
        for (int64_t j = 0; j < seq; ++j) {
          float s = 0.f;
          for (int64_t d = 0; d < hd; ++d) s += doh[i * hd + d] * vh[j * hd + d];
          dp[i * seq + j] = s;
        }
      /* dV[j, :] = sum_i P[i, j] dO[i, :] */
      memset(dvh, 0, (size_t)seq * hd * sizeof(float));
      for (int64_t i = 0; i < seq; ++i)
        for (int64_t j = 0; j < seq; ++j) axpy_row(dvh + j * hd, doh + i * hd, p[i * seq + j], hd);
      for (int64_t i = 0; i < seq; ++i) {
        softmax_vjp_row(p + i * seq, dp + i * seq, dp + i * seq, seq);
        for (int64_t j = 0; j < seq; ++j) dp[i * seq + j] = dp[i * seq + j] * scale;
      }
      /* dQ[i, :] = sum_j dQK[i, j] K[j, :];  dK[j, :] = sum_i dQK[i, j] Q[i, :] */
      memset(dqh, 0, (size_t)seq * hd * sizeof(float));
      memset(dkh, 0, (size_t)seq * hd * sizeof(float));
      for (int64_t i = 0; i < seq; ++i)
        for (int64_t j = 0; j < seq; ++j) axpy_row(dqh + i * hd, kh + j * hd, dp[i * seq + j], hd);
      for (int64_t i = 0; i < seq; ++i)
        for (int64_t j = 0; j < seq; ++j) axpy_row(dkh + j * hd, qh + i * hd, dp[i * seq + j], hd);
    }
    free(p);
    free(dp);
  }
}

/* BF16 round-to-nearest-even of an F32 value (LazyTensor.swift:1511-1516),
 * returned as F32. NaN stays NaN. */
static inline float bf16_round(float x) {
  uint32_t u;
  memcpy(&u, &x, 4);
  if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) return x;
  u = (u + 0x7fffu + ((u >> 16) & 1u)) & 0xffff0000u;
  float r;
  memcpy(&r, &u, 4);
  return r;
}

/* The attention VJP chain as a BF16 program runs it: the probabilities and the
 * softmax cotangent are materialised as BF16 tensors before the contractions
 * that consume them (a BF16 graph of the reference stores every intermediate
 * in BF16, rounding to nearest even, LazyTensor.swift:1511-1516), and the
 * row term of the softmax VJP is formed from the stored (BF16) output:
 * sum_j dP_ij P_ij = sum_d dO_id O_id. Everything else as
 * oracle_attention_bwd, in F32: dP = dO.V^T; dS = P*(dP - delta);
 * dV = bf16(P)^T.dO; dQ = (bf16(dS).K)*scale; dK = (bf16(dS)^T.Q)*scale.
 * Inputs are the BF16 values as F32; o is the forward output as stored. */
void oracle_attention_bwd_bf16(const float* q, const float* k, const float* v, const float* o,
                               const float* d_o, float* dq, float* dk, float* dv, int64_t batch,
                               int64_t heads, int64_t seq, int64_t hd, float scale, int causal) {
  const int64_t bh = batch * heads;
#pragma omp parallel
  {
    float* p = (float*)xmalloc((size_t)seq * seq * sizeof(float));
    float* dp = (float*)xmalloc((size_t)seq * seq * sizeof(float));
#pragma omp for schedule(dynamic)
    for (int64_t h = 0; h < bh; ++h) {
      const float* qh = q + h * seq * hd;
      const float* kh = k + h * seq * hd;
      const float* vh = v + h * seq * hd;
      const float* oh = o + h * seq * hd;
      const float* doh = d_o + h * seq * hd;
      float* dqh = dq + h * seq * hd;
      float* dkh = dk + h * seq * hd;
      float* dvh = dv + h * seq * hd;
      attention_probs_head(qh, kh, p, NULL, seq, hd, scale, causal);
      for (int64_t i = 0; i < seq; ++i) {
        float delta = 0.f;
        for (int64_t d = 0; d < hd; ++d) delta += doh[i * hd + d] * oh[i * hd + d];
        for (int64_t j = 0; j < seq; ++j) {
          float s = 0.f;
          for (int64_t d = 0; d < hd; ++d) s += doh[i * hd + d] * vh[j * hd + d];
          const float pij = p[i * seq + j];
          dp[i * seq + j] = bf16_round(pij * (s - delta));
          p[i * seq + j] = bf16_round(pij);
        }
      }
      memset(dvh, 0, (size_t)seq * hd * sizeof(float));
      memset(dqh, 0, (size_t)seq * hd * sizeof(float));
      memset(dkh, 0, (size_t)seq * hd * sizeof(float));
      for (int64_t i = 0; i < seq; ++i)
        for (int64_t j = 0; j < seq; ++j) {
          axpy_row(dvh + j * hd, doh + i * hd, p[i * seq + j], hd);
          axpy_row(dqh + i * hd, kh + j * hd, dp[i * seq + j], hd);
          axpy_row(dkh + j * hd, qh + i * hd, dp[i * seq + j], hd);
        }
      for (int64_t e = 0; e < seq * hd; ++e) {
        dqh[e] = dqh[e] * scale;
        dkh[e] = dkh[e] * scale;
      }
    }
    free(p);
    free(dp);
  }
}

/* ---- Adam -----------------------------------------------------------------
 * optim.Adam.step (Optimizer.swift:354-412) / value Adam.update
 * (TangentOptimizer.swift:99-135): scalars formed in F32 once per step. */
void oracle_adam(float* p, const float* g, float* m, float* v, int64_t n, float lr, float beta1,
                 float beta2, float eps, float weight_decay, int64_t step, float grad_scale) {
  const float omb1 = 1.0f - beta1, omb2 = 1.0f - beta2;
  const float bc1 = 1.0f - powf(beta1, (float)step);
  const float bc2 = 1.0f - powf(beta2, (float)step);
  const float lrwd = lr * weight_decay;
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    float gi = g[i] * grad_scale;
    float pi = p[i];
    if (weight_decay != 0.0f) pi = pi - pi * lrwd;
    float mi = m[i] * beta1 + gi * omb1;
    float vi = v[i] * beta2 + (gi * gi) * omb2;
    float mhat = mi / bc1;
    float vhat = vi / bc2;
    float upd = mhat / (sqrtf(vhat) + eps);
    p[i] = pi - upd * lr;
    m[i] = mi;
    v[i] = vi;
  }
}

/* ---- global-norm clipping (Optimizer.swift:1229-1267) and the warmup-cosine
 * schedule (Optimizer.swift:766-803) ------------------------------------------ */
/* sqrt(sum_i (g[i]*grad_scale)^2): the products rounded to F32 as the
 * reference's (grad * grad).sum() of the scaled gradient; the sum in double,
 * so the oracle has no summation-order error of its own. */
float oracle_grad_norm(const float* g, int64_t n, float grad_scale) {
  double acc = 0.0;
  for (int64_t i = 0; i < n; ++i) {
    const float a = g[i] * grad_scale;
    acc += (double)a * (double)a;
  }
  return (float)sqrt(acc);
}

/* clipCoeff = maxNorm / (totalNorm + 1e-6), clamped to 1 (:1253-1262), the
 * gradient scaled by it (:1265-1267), then the oracle_adam update. */
void oracle_adam_clipped(float* p, const float* g, float* m, float* v, int64_t n, float lr,
                         float beta1, float beta2, float eps, float weight_decay, int64_t step,
                         float grad_scale, float norm, float max_norm) {
  const float raw = max_norm / (norm + 1e-6f);
  const float coeff = raw < 1.0f ? raw : 1.0f;
  float* gc = (float*)malloc((size_t)(n > 0 ? n : 1) * sizeof(float));
  for (int64_t i = 0; i < n; ++i) gc[i] = (g[i] * grad_scale) * coeff;
  oracle_adam(p, gc, m, v, n, lr, beta1, beta2, eps, weight_decay, step, 1.0f);
  free(gc);
}

/* WarmupCosineScheduler.currentLR (:774-783) at scheduler step `step`. */
float oracle_lr_warmup_cosine(float base_lr, float min_lr, int64_t warmup, int64_t total,
                              int64_t step) {
  if (step > total) step = total;
  if (step < warmup) return base_lr * (float)(step + 1) / (float)warmup;
  const float progress = (float)(step - warmup) / (float)(total - warmup);
  return min_lr + (base_lr - min_lr) * (1.0f + cosf(3.14159265358979323846f * progress)) / 2.0f;
}

/* ---- GELU (StableHLOEmitter.swift:804-816) and VJP (Autodiff.swift:401-418) */
static inline float gelu1(float x) {
  float x3 = x * (x * x);
  float inner = x + 0.044715f * x3;
  float t = tanhf(0.7978845608f * inner);
  return 0.5f * (x * (1.0f + t));
}
static inline float gelu_grad1(float x) {
  const float c = 0.7978845608f, a = 0.044715f;
  float x2 = x * x;
  float u = c * (x + a * (x2 * x));
  float t = tanhf(u);
  float up = c * (1.0f + (3.0f * a) * x2);
  return 0.5f * (1.0f + t) + ((0.5f * x) * (1.0f - t * t)) * up;
}
void oracle_gelu_fwd(const float* x, float* y, int64_t n) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) y[i] = gelu1(x[i]);
}
void oracle_gelu_bwd(const float* x, const float* dy, float* dx, int64_t n) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) dx[i] = dy[i] * gelu_grad1(x[i]);
}

/* ---- cross-entropy (main.swift:412-433; Loss.swift:627-699) ---------------
 * shifted = x - max; lse = log(sum(exp(shifted))); logp = shifted - lse;
 * loss = mean(-(logp . onehot)). Gradient through that chain:
 * dlogits = exp(shifted) * ((1/R)/sumExp) - onehot/R. */
float oracle_cross_entropy(const float* logits, const int32_t* targets, float* dlogits,
                           int64_t rows, int64_t classes) {
  float* per = (float*)xmalloc((size_t)rows * sizeof(float));
  const float inv_r = 1.0f / (float)rows;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    const float* x = logits + r * classes;
    float mx = -INFINITY;
    for (int64_t c = 0; c < classes; ++c) mx = x[c] > mx ? x[c] : mx;
    float sum = 0.f;
    for (int64_t c = 0; c < classes; ++c) sum += expf(x[c] - mx);
    const float lse = logf(sum);
    const int32_t t = targets[r];
    per[r] = -((x[t] - mx) - lse);
    if (dlogits) {
      const float coef = inv_r / sum;
      for (int64_t c = 0; c < classes; ++c)
        dlogits[r * classes + c] = expf(x[c] - mx) * coef - (c == t ? inv_r : 0.0f);
    }
  }
  float s = 0.f;
  for (int64_t r = 0; r < rows; ++r) s += per[r];
  free(per);
  return s / (float)rows;
}

/* allReduceMean (MLIRBuilder.swift:923-929): all_reduce add, then * (1/n). */
void oracle_allreduce_mean(const float* const* bufs, int replicas, int64_t count, float* out) {
  const float inv = 1.0f / (float)replicas;
  for (int64_t i = 0; i < count; ++i) {
    float s = 0.f;
    for (int r = 0; r < replicas; ++r) s += bufs[r][i];
    out[i] = s * inv;
  }
}

/* ---- GPT ------------------------------------------------------------------ */
enum { T_LN1W, T_LN1B, T_QKVW, T_QKVB, T_PROJW, T_PROJB, T_LN2W, T_LN2B, T_FCW, T_FCB,
       T_FCPW, T_FCPB, T_PER_LAYER };

static int64_t tensor_size(const oracle_gpt_config* c, int64_t idx) {
  const int64_t D = c->dim, L = c->layers;
  if (idx == 0) return c->vocab_padded * D;
  if (idx == 1) return c->seq * D;
  int64_t j = idx - 2;
  if (j < L * T_PER_LAYER) {
    switch (j % T_PER_LAYER) {
      case T_LN1W: case T_LN1B: case T_LN2W: case T_LN2B: case T_PROJB: case T_FCPB: return D;
      case T_QKVW: return 3 * D * D;
      case T_QKVB: return 3 * D;
      case T_PROJW: return D * D;
      case T_FCW: return 4 * D * D;
      case T_FCB: return 4 * D;
      case T_FCPW: return 4 * D * D;
    }
  }
  j -= L * T_PER_LAYER;
  if (j == 0 || j == 1) return D;
  return c->vocab_padded * D; /* untied lm-head */
}

int64_t oracle_gpt_num_tensors(const oracle_gpt_config* c) {
  return 2 + c->layers * T_PER_LAYER + 2 + (c->tied ? 0 : 1);
}

int64_t oracle_gpt_param_offset(const oracle_gpt_config* c, int64_t idx) {
  int64_t off = 0;
  for (int64_t i = 0; i < idx; ++i) off += (tensor_size(c, i) + 63) / 64 * 64;
  return off;
}

int64_t oracle_gpt_param_count(const oracle_gpt_config* c) {
  return oracle_gpt_param_offset(c, oracle_gpt_num_tensors(c));
}

/* y[t, :] = x[t, :] . w^T + b (the GPT linear, main.swift:353-362). */
static void linear_fwd(const float* x, const float* w, const float* b, float* y, int64_t T,
                       int64_t in, int64_t out) {
  oracle_matmul(x, w, y, T, out, in, 0, 1);
  if (b) {
#pragma omp parallel for schedule(static)
    for (int64_t t = 0; t < T; ++t)
      for (int64_t o = 0; o < out; ++o) y[t * out + o] = y[t * out + o] + b[o];
  }
}

/* dx (+)= dy . w; dw += dy^T . x; db += sum_t dy (Autodiff.swift:177-191,221-257). */
static void linear_bwd(const float* dy, const float* x, const float* w, float* dx, float* dw,
                       float* db, int64_t T, int64_t in, int64_t out, float* scratch) {
  if (dx) oracle_matmul(dy, w, dx, T, in, out, 0, 0);
  oracle_matmul(dy, x, scratch, out, in, T, 1, 0);
  for (int64_t i = 0; i < out * in; ++i) dw[i] += scratch[i];
  if (db) {
    for (int64_t o = 0; o < out; ++o) {
      float s = 0.f;
      for (int64_t t = 0; t < T; ++t) s += dy[t * out + o];
      db[o] += s;
    }
  }
}

/* [B,S,3,H,hd] slice `which` of qkv -> [B,H,S,hd] (the reshape + transpose(1,2)
 * of main.swift:460-465). */
static void split_heads(const float* qkv, float* dst, int which, int64_t B, int64_t S, int64_t H,
                        int64_t hd) {
  const int64_t D = H * hd;
  for (int64_t b = 0; b < B; ++b)
    for (int64_t h = 0; h < H; ++h)
      for (int64_t s = 0; s < S; ++s)
        memcpy(dst + ((b * H + h) * S + s) * hd, qkv + (b * S + s) * 3 * D + which * D + h * hd,
               (size_t)hd * sizeof(float));
}
static void merge_heads_add(const float* src, float* qkv_like, int64_t ld, int64_t col0, int64_t B,
                            int64_t S, int64_t H, int64_t hd, int accumulate) {
  for (int64_t b = 0; b < B; ++b)
    for (int64_t h = 0; h < H; ++h)
      for (int64_t s = 0; s < S; ++s) {
        const float* sp = src + ((b * H + h) * S + s) * hd;
        float* dp = qkv_like + (b * S + s) * ld + col0 + h * hd;
        for (int64_t d = 0; d < hd; ++d) dp[d] = accumulate ? dp[d] + sp[d] : sp[d];
      }
}

float oracle_gpt_fwd_bwd(const oracle_gpt_config* c, const float* params, float* grads,
                         const int32_t* tokens, const int32_t* targets, int64_t B) {
  const int64_t D = c->dim, L = c->layers, S = c->seq, H = c->heads, hd = D / H;
  const int64_t T = B * S, V = c->vocab;
  const float eps = 1e-5f, scale = 1.0f / sqrtf((float)hd);
#define P(i) (params + oracle_gpt_param_offset(c, (i)))
#define G(i) (grads + oracle_gpt_param_offset(c, (i)))
#define LT(l, t) (2 + (l) * T_PER_LAYER + (t))
  const int64_t idx_lnf = 2 + L * T_PER_LAYER;
  const float* wte = P(0);
  const float* lm_w = c->tied ? wte : P(idx_lnf + 2);
  float* g_lm = c->tied ? G(0) : G(idx_lnf + 2);
  memset(grads, 0, (size_t)oracle_gpt_param_count(c) * sizeof(float));

  size_t TD = (size_t)T * D * sizeof(float);
  float* xs = (float*)xmalloc(TD * (L + 1)); /* residual stream entering each block + final */
  float* hs = (float*)xmalloc(TD * L);       /* after attention residual */
  float* ln1 = (float*)xmalloc(TD * L);
  float* ln2 = (float*)xmalloc(TD * L);
  float* qkv = (float*)xmalloc(TD * 3 * L);
  float* att = (float*)xmalloc(TD * L);      /* attention output merged [T, D] */
  float* fc = (float*)xmalloc(TD * 4 * L);   /* pre-GELU */
  float* gl = (float*)xmalloc(TD * 4 * L);   /* post-GELU */
  float* lnf = (float*)xmalloc(TD);
  float* logits = (float*)xmalloc((size_t)T * V * sizeof(float));
  float* qh = (float*)xmalloc(TD), *kh = (float*)xmalloc(TD), *vh = (float*)xmalloc(TD);
  float* oh = (float*)xmalloc(TD);
  float* tmp = (float*)xmalloc(TD * 4);
  size_t scratch_n = (size_t)4 * D * D;
  if ((size_t)c->vocab_padded * D > scratch_n) scratch_n = (size_t)c->vocab_padded * D;
  float* scratch = (float*)xmalloc(scratch_n * sizeof(float));

  /* embeddings (main.swift:454-458) */
  for (int64_t t = 0; t < T; ++t)
    for (int64_t d = 0; d < D; ++d)
      xs[t * D + d] = wte[(int64_t)tokens[t] * D + d] + P(1)[(t % S) * D + d];
  for (int64_t l = 0; l < L; ++l) {
    float* x = xs + l * T * D;
    float* h = hs + l * T * D;
    float* a1 = ln1 + l * T * D;
    float* a2 = ln2 + l * T * D;
    float* q3 = qkv + l * T * 3 * D;
    float* ao = att + l * T * D;
    float* f = fc + l * T * 4 * D;
    float* g = gl + l * T * 4 * D;
    oracle_layernorm_fwd(x, P(LT(l, T_LN1W)), P(LT(l, T_LN1B)), a1, NULL, NULL, T, D, eps);
    linear_fwd(a1, P(LT(l, T_QKVW)), P(LT(l, T_QKVB)), q3, T, D, 3 * D);
    split_heads(q3, qh, 0, B, S, H, hd);
    split_heads(q3, kh, 1, B, S, H, hd);
    split_heads(q3, vh, 2, B, S, H, hd);
    oracle_attention_fwd(qh, kh, vh, oh, NULL, NULL, B, H, S, hd, scale, 1);
    merge_heads_add(oh, ao, D, 0, B, S, H, hd, 0);
    linear_fwd(ao, P(LT(l, T_PROJW)), P(LT(l, T_PROJB)), tmp, T, D, D);
    for (int64_t i = 0; i < T * D; ++i) h[i] = x[i] + tmp[i];
    oracle_layernorm_fwd(h, P(LT(l, T_LN2W)), P(LT(l, T_LN2B)), a2, NULL, NULL, T, D, eps);
    linear_fwd(a2, P(LT(l, T_FCW)), P(LT(l, T_FCB)), f, T, D, 4 * D);
    oracle_gelu_fwd(f, g, T * 4 * D);
    linear_fwd(g, P(LT(l, T_FCPW)), P(LT(l, T_FCPB)), tmp, T, 4 * D, D);
    float* xn = xs + (l + 1) * T * D;
    for (int64_t i = 0; i < T * D; ++i) xn[i] = h[i] + tmp[i];
  }
  float* xf = xs + L * T * D;
  oracle_layernorm_fwd(xf, P(idx_lnf), P(idx_lnf + 1), lnf, NULL, NULL, T, D, eps);
  linear_fwd(lnf, lm_w, NULL, logits, T, D, V); /* first V rows of the (padded) head */
  float* dlogits = (float*)xmalloc((size_t)T * V * sizeof(float));
  const float loss = oracle_cross_entropy(logits, targets, dlogits, T, V);

  /* ---- backward ---- */
  float* dx = (float*)xmalloc(TD);
  float* dtmp = (float*)xmalloc(TD * 4);
  float* dtmp2 = (float*)xmalloc(TD * 4);
  linear_bwd(dlogits, lnf, lm_w, dtmp, g_lm, NULL, T, D, V, scratch);
  oracle_layernorm_bwd(dtmp, xf, P(idx_lnf), dx, scratch, scratch + D, T, D, eps);
  for (int64_t i = 0; i < D; ++i) {
    G(idx_lnf)[i] += scratch[i];
    G(idx_lnf + 1)[i] += scratch[D + i];
  }
  for (int64_t l = L - 1; l >= 0; --l) {
    float* x = xs + l * T * D;
    float* h = hs + l * T * D;
    float* a1 = ln1 + l * T * D;
    float* a2 = ln2 + l * T * D;
    float* q3 = qkv + l * T * 3 * D;
    float* ao = att + l * T * D;
    float* f = fc + l * T * 4 * D;
    float* g = gl + l * T * 4 * D;
    /* x_{l+1} = h + mlp: dh = dx; dmlp = dx */
    linear_bwd(dx, g, P(LT(l, T_FCPW)), dtmp, G(LT(l, T_FCPW)), G(LT(l, T_FCPB)), T, 4 * D, D,
               scratch);
    oracle_gelu_bwd(f, dtmp, dtmp2, T * 4 * D);
    linear_bwd(dtmp2, a2, P(LT(l, T_FCW)), dtmp, G(LT(l, T_FCW)), G(LT(l, T_FCB)), T, D, 4 * D,
               scratch);
    float* dln = dtmp2;
    oracle_layernorm_bwd(dtmp, h, P(LT(l, T_LN2W)), dln, scratch, scratch + D, T, D, eps);
    for (int64_t i = 0; i < D; ++i) {
      G(LT(l, T_LN2W))[i] += scratch[i];
      G(LT(l, T_LN2B))[i] += scratch[D + i];
    }
    for (int64_t i = 0; i < T * D; ++i) dx[i] += dln[i]; /* dh */
    /* h = x + proj(att) */
    linear_bwd(dx, ao, P(LT(l, T_PROJW)), dtmp, G(LT(l, T_PROJW)), G(LT(l, T_PROJB)), T, D, D,
               scratch);
    split_heads(q3, qh, 0, B, S, H, hd);
    split_heads(q3, kh, 1, B, S, H, hd);
    split_heads(q3, vh, 2, B, S, H, hd);
    /* dO in head layout */
    for (int64_t b = 0; b < B; ++b)
      for (int64_t hh = 0; hh < H; ++hh)
        for (int64_t s = 0; s < S; ++s)
          memcpy(oh + ((b * H + hh) * S + s) * hd, dtmp + (b * S + s) * D + hh * hd,
                 (size_t)hd * sizeof(float));
    float* dq = dtmp2;
    float* dk = dtmp2 + T * D;
    float* dv = dtmp2 + 2 * T * D;
    oracle_attention_bwd(qh, kh, vh, oh, dq, dk, dv, B, H, S, hd, scale, 1);
    float* dqkv = dtmp; /* [T, 3D] */
    merge_heads_add(dq, dqkv, 3 * D, 0, B, S, H, hd, 0);
    merge_heads_add(dk, dqkv, 3 * D, D, B, S, H, hd, 0);
    merge_heads_add(dv, dqkv, 3 * D, 2 * D, B, S, H, hd, 0);
    float* dln1 = dtmp2;
    linear_bwd(dqkv, a1, P(LT(l, T_QKVW)), dln1, G(LT(l, T_QKVW)), G(LT(l, T_QKVB)), T, D, 3 * D,
               scratch);
    float* dxa = dtmp2 + 3 * T * D;
    oracle_layernorm_bwd(dln1, x, P(LT(l, T_LN1W)), dxa, scratch, scratch + D, T, D, eps);
    for (int64_t i = 0; i < D; ++i) {
      G(LT(l, T_LN1W))[i] += scratch[i];
      G(LT(l, T_LN1B))[i] += scratch[D + i];
    }
    for (int64_t i = 0; i < T * D; ++i) dx[i] += dxa[i];
  }
  /* embedding VJP (Data.swift:890-907: one-hot^T . v, i.e. a scatter-add) */
  for (int64_t t = 0; t < T; ++t)
    for (int64_t d = 0; d < D; ++d) {
      G(0)[(int64_t)tokens[t] * D + d] += dx[t * D + d];
      G(1)[(t % S) * D + d] += dx[t * D + d];
    }
#undef P
#undef G
#undef LT
  free(xs); free(hs); free(ln1); free(ln2); free(qkv); free(att); free(fc); free(gl);
  free(lnf); free(logits); free(qh); free(kh); free(vh); free(oh); free(tmp); free(scratch);
  free(dlogits); free(dx); free(dtmp); free(dtmp2);
  return loss;
}

/* ---- MLP classifier (value Linear x.W+b, ValueLayers.swift:38-41) ---------- */
float oracle_mlp_fwd_bwd(const float* params, float* grads, const float* x, const int32_t* labels,
                         int64_t B, int64_t in, int64_t hid, int64_t out) {
  const float* w1 = params;
  const float* b1 = w1 + in * hid;
  const float* w2 = b1 + hid;
  const float* b2 = w2 + hid * out;
  float* gw1 = grads;
  float* gb1 = gw1 + in * hid;
  float* gw2 = gb1 + hid;
  float* gb2 = gw2 + hid * out;
  float* z = (float*)xmalloc((size_t)B * hid * sizeof(float));
  float* h = (float*)xmalloc((size_t)B * hid * sizeof(float));
  float* logits = (float*)xmalloc((size_t)B * out * sizeof(float));
  float* dlog = (float*)xmalloc((size_t)B * out * sizeof(float));
  float* dh = (float*)xmalloc((size_t)B * hid * sizeof(float));
  oracle_matmul(x, w1, z, B, hid, in, 0, 0);
  for (int64_t i = 0; i < B; ++i)
    for (int64_t j = 0; j < hid; ++j) {
      z[i * hid + j] = z[i * hid + j] + b1[j];
      h[i * hid + j] = z[i * hid + j] > 0.f ? z[i * hid + j] : 0.f;
    }
  oracle_matmul(h, w2, logits, B, out, hid, 0, 0);
  for (int64_t i = 0; i < B; ++i)
    for (int64_t j = 0; j < out; ++j) logits[i * out + j] = logits[i * out + j] + b2[j];
  const float loss = oracle_cross_entropy(logits, labels, dlog, B, out);
  oracle_matmul(h, dlog, gw2, hid, out, B, 1, 0);
  for (int64_t j = 0; j < out; ++j) {
    float s = 0.f;
    for (int64_t i = 0; i < B; ++i) s += dlog[i * out + j];
    gb2[j] = s;
  }
  oracle_matmul(dlog, w2, dh, B, hid, out, 0, 1);
  for (int64_t i = 0; i < B * hid; ++i) dh[i] = h[i] > 0.f ? dh[i] : 0.f;
  oracle_matmul(x, dh, gw1, in, hid, B, 1, 0);
  for (int64_t j = 0; j < hid; ++j) {
    float s = 0.f;
    for (int64_t i = 0; i < B; ++i) s += dh[i * hid + j];
    gb1[j] = s;
  }
  free(z); free(h); free(logits); free(dlog); free(dh);
  return loss;
}

/* ---- Examples/ValueLayers/main.swift ---------------------------------------
 * Model (makeMLP): Linear(w1 = ones [1,16], b1 = -knee_i, knee_i = i/15*4-2),
 * ReLU, Linear(w2_i = (i%3)*0.1 - 0.1 [16,1], b2 = 0). Data: x in -2..2 step
 * 0.5 (9 points), y = x^2. Loss: sum((pred-y)^2)/n. Optimizer: value Adam,
 * lr 0.05 (TangentOptimizer.swift:99-135). */
static float value_layers_loss(const float* p, const float* xs, const float* ys, int n,
                               float* grad) {
  const float* w1 = p;
  const float* b1 = p + 16;
  const float* w2 = p + 32;
  const float b2 = p[48];
  float loss = 0.f;
  float z[9][16], h[9][16], pred[9];
  for (int i = 0; i < n; ++i) {
    float s = 0.f;
    for (int j = 0; j < 16; ++j) {
      z[i][j] = xs[i] * w1[j] + b1[j];
      h[i][j] = z[i][j] > 0.f ? z[i][j] : 0.f;
      s += h[i][j] * w2[j];
    }
    pred[i] = s + b2;
    float r = pred[i] - ys[i];
    loss += r * r;
  }
  loss = loss / (float)n;
  if (grad) {
    memset(grad, 0, 49 * sizeof(float));
    for (int i = 0; i < n; ++i) {
      float r = pred[i] - ys[i];
      float dp = r * (1.0f / (float)n) + r * (1.0f / (float)n);
      grad[48] += dp;
      for (int j = 0; j < 16; ++j) {
        grad[32 + j] += h[i][j] * dp;
        float dz = z[i][j] > 0.f ? dp * w2[j] : 0.f;
        grad[j] += xs[i] * dz;
        grad[16 + j] += dz;
      }
    }
  }
  return loss;
}

void oracle_value_layers_example(int steps, float* losses) {
  float p[49], g[49], m[49], v[49];
  float xs[9], ys[9];
  for (int i = 0; i < 9; ++i) {
    xs[i] = -2.0f + 0.5f * (float)i;
    ys[i] = xs[i] * xs[i];
  }
  for (int j = 0; j < 16; ++j) {
    p[j] = 1.0f;
    p[16 + j] = -((float)j / 15.0f * 4.0f - 2.0f);
    p[32 + j] = (float)(j % 3) * 0.1f - 0.1f;
  }
  p[48] = 0.f;
  memset(m, 0, sizeof(m));
  memset(v, 0, sizeof(v));
  losses[0] = value_layers_loss(p, xs, ys, 9, NULL);
  for (int s = 1; s <= steps; ++s) {
    value_layers_loss(p, xs, ys, 9, g);
    oracle_adam(p, g, m, v, 49, 0.05f, 0.9f, 0.999f, 1e-8f, 0.0f, s, 1.0f);
    losses[s] = value_layers_loss(p, xs, ys, 9, NULL);
  }
}
