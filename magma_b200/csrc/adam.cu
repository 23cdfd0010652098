// Adam update over flat F32 parameter arenas.
//
// Restates optim.Adam.step (Sources/Core/Optimizer.swift:354-412) and the value
// Adam.update (Sources/Core/TangentOptimizer.swift:99-135) element-wise, in the
// reference's op order and without contraction into FMAs (each op rounds, as
// the reference's separate StableHLO ops do):
//   g  = grad * grad_scale                 (grad_scale = 1/n folds allReduceMean)
//   p  = p - p * lrwd                      (decoupled decay, Optimizer.swift:384-386)
//   m  = m*b1 + g*(1-b1)                   (:389-393)
//   v  = v*b2 + (g*g)*(1-b2)               (:396-401)
//   p  = p - ((m/bc1) / (sqrt(v/bc2) + eps)) * lr   (:404-410)
// The scalars b1, 1-b1, b2, 1-b2, bc1 = 1-b1^t, bc2 = 1-b2^t, lr*wd are formed
// on the host in F32 as the reference does (:370-379).
//
// HBM-bound: 16 B read of p, g, m, v and 12 B written per element (+2 B for the
// optional BF16 shadow copy), float4-vectorised with a grid sized to the SMs.
//
// Global-norm clipping (optim.clipGradNorm, Optimizer.swift:1229-1267, as the
// GPT trainer applies it before every Adam step, main.swift:857) is split in
// two: grad_sumsq_partial + grad_norm_finish write the norm of the scaled
// gradient to a device scalar (per-block sums in a fixed order, so the result
// does not depend on scheduling), and the clipped Adam kernels read that
// scalar and scale g by the clip coefficient before the update, so no host
// synchronisation sits between the two.
#include <cmath>

#include "common.cuh"

namespace magma {
namespace {

struct AdamScalars {
  float b1, omb1, b2, omb2, bc1, bc2, eps, lr, lrwd, grad_scale;
  int has_wd;
  const float* norm;  // clipped update: device scalar with the global gradient norm
  float max_norm;
};

// Clip coefficient of clipGradNorm (Optimizer.swift:1253-1262): maxNorm /
// (norm + 1e-6) where that is below 1, else 1 (also 1 for a NaN norm, as the
// reference's lessThan mask is then false).
__device__ __forceinline__ float clip_coeff(const AdamScalars& s) {
  if (s.norm == nullptr) return 1.f;
  const float raw = __fdiv_rn(s.max_norm, __fadd_rn(*s.norm, 1e-6f));
  return raw < 1.f ? raw : 1.f;
}

__device__ __forceinline__ void adam_elem(float& p, float g, float& m, float& v,
                                          const AdamScalars& s, float coeff = 1.f) {
  g = __fmul_rn(g, s.grad_scale);
  if (s.norm != nullptr) g = __fmul_rn(g, coeff);  // clipped gradient
  if (s.has_wd) p = __fsub_rn(p, __fmul_rn(p, s.lrwd));
  m = __fadd_rn(__fmul_rn(m, s.b1), __fmul_rn(g, s.omb1));
  v = __fadd_rn(__fmul_rn(v, s.b2), __fmul_rn(__fmul_rn(g, g), s.omb2));
  float mhat = __fdiv_rn(m, s.bc1);
  float vhat = __fdiv_rn(v, s.bc2);
  float upd = __fdiv_rn(mhat, __fadd_rn(__fsqrt_rn(vhat), s.eps));
  p = __fsub_rn(p, __fmul_rn(upd, s.lr));
}

__global__ void __launch_bounds__(256)
adam_vec4(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
          float* __restrict__ v, __nv_bfloat16* __restrict__ shadow, int64_t n, AdamScalars s) {
  const float coeff = clip_coeff(s);
  const int64_t n4 = n >> 2;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
    float4 pv = reinterpret_cast<float4*>(p)[i];
    float4 gv = __ldcs(reinterpret_cast<const float4*>(g) + i);
    float4 mv = reinterpret_cast<float4*>(m)[i];
    float4 vv = reinterpret_cast<float4*>(v)[i];
    adam_elem(pv.x, gv.x, mv.x, vv.x, s, coeff);
    adam_elem(pv.y, gv.y, mv.y, vv.y, s, coeff);
    adam_elem(pv.z, gv.z, mv.z, vv.z, s, coeff);
    adam_elem(pv.w, gv.w, mv.w, vv.w, s, coeff);
    reinterpret_cast<float4*>(p)[i] = pv;
    __stcs(reinterpret_cast<float4*>(m) + i, mv);
    __stcs(reinterpret_cast<float4*>(v) + i, vv);
    if (shadow != nullptr) {
      __nv_bfloat162 lo = __floats2bfloat162_rn(pv.x, pv.y);
      __nv_bfloat162 hi = __floats2bfloat162_rn(pv.z, pv.w);
      uint2 u;
      u.x = *reinterpret_cast<uint32_t*>(&lo);
      u.y = *reinterpret_cast<uint32_t*>(&hi);
      reinterpret_cast<uint2*>(shadow)[i] = u;
    }
  }
  // tail (n % 4 elements) handled by the first threads of block 0
  if (blockIdx.x == 0 && threadIdx.x < (n & 3)) {
    int64_t i = (n4 << 2) + threadIdx.x;
    float pp = p[i], mm = m[i], vv = v[i];
    adam_elem(pp, g[i], mm, vv, s, coeff);
    p[i] = pp;
    m[i] = mm;
    v[i] = vv;
    if (shadow != nullptr) shadow[i] = __float2bfloat16_rn(pp);
  }
}

__global__ void __launch_bounds__(256)
adam_scalar(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
            float* __restrict__ v, __nv_bfloat16* __restrict__ shadow, int64_t n, AdamScalars s) {
  const float coeff = clip_coeff(s);
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    float pp = p[i], mm = m[i], vv = v[i];
    adam_elem(pp, g[i], mm, vv, s, coeff);
    p[i] = pp;
    m[i] = mm;
    v[i] = vv;
    if (shadow != nullptr) shadow[i] = __float2bfloat16_rn(pp);
  }
}

// Multi-tensor apply: up to kMaxTensors tensors per launch, passed by value in
// the kernel parameter space. Block b walks every tensor with stride gridDim.
constexpr int kMaxTensors = 96;
struct TensorList {
  float* p[kMaxTensors];
  const float* g[kMaxTensors];
  float* m[kMaxTensors];
  float* v[kMaxTensors];
  int64_t n[kMaxTensors];
  int count;
};

__global__ void __launch_bounds__(256) adam_multi(TensorList t, AdamScalars s) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int k = 0; k < t.count; ++k) {
    float* p = t.p[k];
    const float* g = t.g[k];
    float* m = t.m[k];
    float* v = t.v[k];
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < t.n[k]; i += stride) {
      float pp = p[i], mm = m[i], vv = v[i];
      adam_elem(pp, g[i], mm, vv, s);
      p[i] = pp;
      m[i] = mm;
      v[i] = vv;
    }
  }
}

magma_status_t make_scalars(float lr, float beta1, float beta2, float eps, float wd, int64_t step,
                            float grad_scale, AdamScalars* s) {
  if (!(lr > 0.f)) return fail(MAGMA_INVALID_ARGUMENT, "adam: learning rate must be positive");
  if (!(beta1 >= 0.f && beta1 < 1.f)) return fail(MAGMA_INVALID_ARGUMENT, "adam: beta1 must be in [0, 1)");
  if (!(beta2 >= 0.f && beta2 < 1.f)) return fail(MAGMA_INVALID_ARGUMENT, "adam: beta2 must be in [0, 1)");
  if (step < 1) return fail(MAGMA_INVALID_ARGUMENT, "adam: step counts from 1 (got %lld)", (long long)step);
  s->b1 = beta1;
  s->omb1 = 1.0f - beta1;
  s->b2 = beta2;
  s->omb2 = 1.0f - beta2;
  s->bc1 = 1.0f - powf(beta1, (float)step);
  s->bc2 = 1.0f - powf(beta2, (float)step);
  s->eps = eps;
  s->lr = lr;
  s->lrwd = lr * wd;
  s->has_wd = wd != 0.f;
  s->grad_scale = grad_scale;
  s->norm = nullptr;
  s->max_norm = 0.f;
  return MAGMA_OK;
}

// ---- global gradient norm ----------------------------------------------------
constexpr int kNormThreads = 256;

__device__ __forceinline__ float block_sum(float x, float* red) {
  x = warp_sum(x);  // butterfly: the same order on every run
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[w] = x;
  __syncthreads();
  float t = 0.f;
  if (threadIdx.x == 0)
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t += red[i];
  return t;  // valid in thread 0
}

// partial[b] = sum over this block's grid-stride elements of (g * scale)^2.
__global__ void __launch_bounds__(kNormThreads)
grad_sumsq_partial(const float* __restrict__ g, int64_t n, float scale, int vec,
                   float* __restrict__ partial) {
  __shared__ float red[kNormThreads / 32];
  float acc = 0.f;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t i0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (vec) {
    const int64_t n4 = n >> 2;
    for (int64_t i = i0; i < n4; i += stride) {
      const float4 t = __ldcs(reinterpret_cast<const float4*>(g) + i);
      const float a = __fmul_rn(t.x, scale), b = __fmul_rn(t.y, scale);
      const float c = __fmul_rn(t.z, scale), d = __fmul_rn(t.w, scale);
      acc = fmaf(a, a, acc);
      acc = fmaf(b, b, acc);
      acc = fmaf(c, c, acc);
      acc = fmaf(d, d, acc);
    }
    if (blockIdx.x == 0 && threadIdx.x < (n & 3)) {
      const float a = __fmul_rn(g[(n4 << 2) + threadIdx.x], scale);
      acc = fmaf(a, a, acc);
    }
  } else {
    for (int64_t i = i0; i < n; i += stride) {
      const float a = __fmul_rn(g[i], scale);
      acc = fmaf(a, a, acc);
    }
  }
  const float t = block_sum(acc, red);
  if (threadIdx.x == 0) partial[blockIdx.x] = t;
}

// norm[0] = sqrt(sum of the partials) (or the sum itself without SQRT),
// summed in block order.
template <bool SQRT>
__global__ void __launch_bounds__(kNormThreads)
grad_norm_finish(const float* __restrict__ partial, int nb, float* __restrict__ norm) {
  __shared__ float red[kNormThreads / 32];
  float acc = 0.f;
  for (int i = threadIdx.x; i < nb; i += blockDim.x) acc += partial[i];
  const float t = block_sum(acc, red);
  if (threadIdx.x == 0) norm[0] = SQRT ? __fsqrt_rn(t) : t;
}

// norm[0] = sqrt(sumsq[0] + sumsq[1] + ...), added in index order by one thread.
__global__ void grad_norm_combine(const float* __restrict__ sumsq, int64_t count,
                                  float* __restrict__ norm) {
  float t = 0.f;
  for (int64_t i = 0; i < count; ++i) t += sumsq[i];
  norm[0] = __fsqrt_rn(t);
}

int64_t norm_blocks(int64_t n) {
  int64_t b = ceil_div((n >> 2) > 0 ? (n >> 2) : 1, kNormThreads);
  const int64_t cap = 4LL * num_sms();
  return b > cap ? cap : b;
}

magma_status_t launch_adam(float* params, const float* grads, float* m, float* v,
                           void* shadow_bf16, int64_t n, const AdamScalars& s, cudaStream_t cs) {
  int threads = 256;
  bool vec = aligned16(params) && aligned16(grads) && aligned16(m) && aligned16(v) &&
             (shadow_bf16 == nullptr || (reinterpret_cast<uintptr_t>(shadow_bf16) & 7u) == 0);
  int64_t work = vec ? (n >> 2) : n;
  int64_t blocks = ceil_div(work > 0 ? work : 1, threads);
  int64_t cap = 8LL * num_sms();
  if (blocks > cap) blocks = cap;
  if (vec)
    adam_vec4<<<(int)blocks, threads, 0, cs>>>(params, grads, m, v, (__nv_bfloat16*)shadow_bf16,
                                               n, s);
  else
    adam_scalar<<<(int)blocks, threads, 0, cs>>>(params, grads, m, v,
                                                 (__nv_bfloat16*)shadow_bf16, n, s);
  return check_launch("adam_step");
}

template <bool SQRT>
magma_status_t grad_norm_impl(const char* fn, const float* grads, int64_t n, float grad_scale,
                              float* norm, void* workspace, int64_t workspace_bytes,
                              void* stream) {
  MAGMA_REQUIRE(n >= 0, "%s: negative size", fn);
  MAGMA_REQUIRE(norm != nullptr, "%s: NULL output", fn);
  cudaStream_t cs = (cudaStream_t)stream;
  if (n == 0) return cuda_status(cudaMemsetAsync(norm, 0, sizeof(float), cs), "grad_norm memset");
  MAGMA_REQUIRE(grads != nullptr, "%s: NULL grads", fn);
  const int64_t nb = norm_blocks(n);
  MAGMA_REQUIRE(workspace != nullptr && workspace_bytes >= 4 * nb,
                "%s: workspace of %lld bytes needed (magma_grad_norm_workspace_size)", fn,
                (long long)(4 * nb));
  MAGMA_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 3u) == 0,
                "%s: workspace must be 4-byte aligned", fn);
  float* partial = static_cast<float*>(workspace);
  grad_sumsq_partial<<<(int)nb, kNormThreads, 0, cs>>>(grads, n, grad_scale,
                                                       aligned16(grads) ? 1 : 0, partial);
  if (magma_status_t st = check_launch("grad_sumsq_partial")) return st;
  grad_norm_finish<SQRT><<<1, kNormThreads, 0, cs>>>(partial, (int)nb, norm);
  return check_launch("grad_norm_finish");
}

}  // namespace
}  // namespace magma

using namespace magma;

extern "C" {

magma_status_t magma_adam_step(float* params, const float* grads, float* m, float* v,
                               void* shadow_bf16, int64_t n, float lr, float beta1, float beta2,
                               float eps, float weight_decay, int64_t step, float grad_scale,
                               void* stream) {
  MAGMA_REQUIRE(n >= 0, "magma_adam_step: negative size");
  AdamScalars s;
  if (magma_status_t st = make_scalars(lr, beta1, beta2, eps, weight_decay, step, grad_scale, &s))
    return st;
  if (n == 0) return MAGMA_OK;
  MAGMA_REQUIRE(params && grads && m && v, "magma_adam_step: NULL pointer");
  return launch_adam(params, grads, m, v, shadow_bf16, n, s, (cudaStream_t)stream);
}

int64_t magma_grad_norm_workspace_size(int64_t n) {
  return n > 0 ? 4 * norm_blocks(n) : 0;
}

magma_status_t magma_grad_norm(const float* grads, int64_t n, float grad_scale, float* norm,
                               void* workspace, int64_t workspace_bytes, void* stream) {
  return grad_norm_impl<true>("magma_grad_norm", grads, n, grad_scale, norm, workspace,
                              workspace_bytes, stream);
}

magma_status_t magma_grad_sumsq(const float* grads, int64_t n, float grad_scale, float* sumsq,
                                void* workspace, int64_t workspace_bytes, void* stream) {
  return grad_norm_impl<false>("magma_grad_sumsq", grads, n, grad_scale, sumsq, workspace,
                               workspace_bytes, stream);
}

magma_status_t magma_grad_norm_combine(const float* sumsq, int64_t count, float* norm,
                                       void* stream) {
  MAGMA_REQUIRE(count >= 1 && sumsq != nullptr && norm != nullptr,
                "magma_grad_norm_combine: bad arguments");
  grad_norm_combine<<<1, 1, 0, (cudaStream_t)stream>>>(sumsq, count, norm);
  return check_launch("grad_norm_combine");
}

magma_status_t magma_adam_step_clipped(float* params, const float* grads, float* m, float* v,
                                       void* shadow_bf16, int64_t n, float lr, float beta1,
                                       float beta2, float eps, float weight_decay, int64_t step,
                                       float grad_scale, const float* grad_norm, float max_norm,
                                       void* stream) {
  MAGMA_REQUIRE(n >= 0, "magma_adam_step_clipped: negative size");
  MAGMA_REQUIRE(grad_norm != nullptr, "magma_adam_step_clipped: NULL grad_norm");
  MAGMA_REQUIRE(max_norm > 0.f, "magma_adam_step_clipped: max_norm must be positive");
  AdamScalars s;
  if (magma_status_t st = make_scalars(lr, beta1, beta2, eps, weight_decay, step, grad_scale, &s))
    return st;
  s.norm = grad_norm;
  s.max_norm = max_norm;
  if (n == 0) return MAGMA_OK;
  MAGMA_REQUIRE(params && grads && m && v, "magma_adam_step_clipped: NULL pointer");
  return launch_adam(params, grads, m, v, shadow_bf16, n, s, (cudaStream_t)stream);
}

magma_status_t magma_lr_warmup_cosine(float base_lr, float min_lr, int64_t warmup_steps,
                                      int64_t total_steps, int64_t step, float* lr) {
  MAGMA_REQUIRE(lr != nullptr, "magma_lr_warmup_cosine: NULL output");
  MAGMA_REQUIRE(warmup_steps >= 0, "magma_lr_warmup_cosine: warmup_steps must be non-negative");
  MAGMA_REQUIRE(total_steps > warmup_steps,
                "magma_lr_warmup_cosine: total_steps (%lld) must exceed warmup_steps (%lld)",
                (long long)total_steps, (long long)warmup_steps);
  MAGMA_REQUIRE(step >= 0, "magma_lr_warmup_cosine: negative step");
  if (step > total_steps) step = total_steps;  // the scheduler stops counting there
  if (step < warmup_steps) {
    *lr = base_lr * (float)(step + 1) / (float)warmup_steps;
    return MAGMA_OK;
  }
  const float progress = (float)(step - warmup_steps) / (float)(total_steps - warmup_steps);
  const float pi = 3.14159265358979323846f;
  *lr = min_lr + (base_lr - min_lr) * (1.0f + cosf(pi * progress)) / 2.0f;
  return MAGMA_OK;
}

magma_status_t magma_adam_step_multi(float* const* params, const float* const* grads,
                                     float* const* m, float* const* v, const int64_t* sizes,
                                     int32_t count, float lr, float beta1, float beta2, float eps,
                                     float weight_decay, int64_t step, float grad_scale,
                                     void* stream) {
  MAGMA_REQUIRE(count >= 0, "magma_adam_step_multi: negative count");
  AdamScalars s;
  if (magma_status_t st = make_scalars(lr, beta1, beta2, eps, weight_decay, step, grad_scale, &s))
    return st;
  if (count == 0) return MAGMA_OK;
  MAGMA_REQUIRE(params && grads && m && v && sizes, "magma_adam_step_multi: NULL array");
  cudaStream_t cs = (cudaStream_t)stream;
  int32_t k = 0;
  while (k < count) {
    TensorList t;
    t.count = 0;
    int64_t maxn = 0;
    for (; k < count && t.count < kMaxTensors; ++k) {
      MAGMA_REQUIRE(sizes[k] >= 0, "magma_adam_step_multi: negative size at %d", k);
      if (sizes[k] == 0) continue;
      MAGMA_REQUIRE(params[k] && grads[k] && m[k] && v[k],
                    "magma_adam_step_multi: NULL tensor at %d", k);
      t.p[t.count] = params[k];
      t.g[t.count] = grads[k];
      t.m[t.count] = m[k];
      t.v[t.count] = v[k];
      t.n[t.count] = sizes[k];
      if (sizes[k] > maxn) maxn = sizes[k];
      ++t.count;
    }
    if (t.count == 0) continue;
    int64_t blocks = ceil_div(maxn, 256);
    int64_t cap = 8LL * num_sms();
    if (blocks > cap) blocks = cap;
    adam_multi<<<(int)blocks, 256, 0, cs>>>(t, s);
    if (magma_status_t st = check_launch("adam_step_multi")) return st;
  }
  return MAGMA_OK;
}

}  // extern "C"
