// Glue ops on the training graphs: embedding gather and its scatter-add VJP,
// fused softmax cross-entropy forward+backward, GELU/ReLU and their VJPs,
// bias gradient, deterministic sum, dtype conversion, scaling. All are
// HBM-bound element/row kernels with 128-bit accesses where alignment allows.
#include <cmath>

#include "common.cuh"
#include "sm100.cuh"

namespace magma {
namespace {

int grid_for(int64_t work, int threads, int per_sm = 8) {
  int64_t b = ceil_div(work > 0 ? work : 1, threads);
  int64_t cap = (int64_t)per_sm * num_sms();
  return (int)(b > cap ? cap : b);
}

// ---- embedding ---------------------------------------------------------------
// Data.swift:856-886 (gather along axis 0) + GPT main.swift:454-458 (tok + pos).
__global__ void embedding_fwd_kernel(const int32_t* __restrict__ tokens,
                                     const float* __restrict__ wte, const float* __restrict__ wpe,
                                     float* __restrict__ out, int64_t rows, int64_t seq, int dim,
                                     int64_t vocab, int* err) {
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  for (int64_t r = (int64_t)blockIdx.x * warps + (threadIdx.x >> 5); r < rows;
       r += (int64_t)gridDim.x * warps) {
    int32_t t = tokens[r];
    if (t < 0 || t >= vocab) {
      if (lane == 0) set_device_error(err, kDevErrBadIndex);
      t = 0;
    }
    const float* te = wte + (int64_t)t * dim;
    const float* pe = wpe ? wpe + (r % seq) * dim : nullptr;
    float* o = out + r * dim;
    for (int i = lane; i < dim; i += 32) o[i] = pe ? __fadd_rn(te[i], pe[i]) : te[i];
  }
}

// Scatter-add of token rows: dwte[tokens[r]] += dout[r] (fp32 atomics; the sum
// over rows sharing a token is order-independent up to rounding).
__global__ void embedding_bwd_tok_kernel(const int32_t* __restrict__ tokens,
                                         const float* __restrict__ dout, float* __restrict__ dwte,
                                         int64_t rows, int dim, int64_t vocab, int* err) {
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  for (int64_t r = (int64_t)blockIdx.x * warps + (threadIdx.x >> 5); r < rows;
       r += (int64_t)gridDim.x * warps) {
    int32_t t = tokens[r];
    if (t < 0 || t >= vocab) {
      if (lane == 0) set_device_error(err, kDevErrBadIndex);
      continue;
    }
    const float* src = dout + r * dim;
    float* dst = dwte + (int64_t)t * dim;
    for (int i = lane; i < dim; i += 32) atomicAdd(dst + i, src[i]);
  }
}

// Deterministic scatter-add: the rows are put in (token, row) order, then one
// warp per token adds that token's rows to dwte[token] in increasing row
// order, so every token row gets its rows added one at a time in row order,
// on every run, as a sequential loop would.
//  1. emb_sort_chunks: one CTA per chunk of kEmbChunk rows sorts the keys
//     token * kEmbChunk + local row in shared memory (bitonic network).
//  2. emb_merge_rank: an element's place in the global order is its index in
//     its chunk plus, for every other chunk, the number of that chunk's keys
//     that come before it (token below, or equal token in an earlier chunk):
//     binary searches over the chunks, staged in shared memory.
//  3. emb_run_sum: one warp per run of equal tokens in the global order.
constexpr int kEmbChunk = 1024;
constexpr int kEmbRowBits = 10;  // log2(kEmbChunk)
constexpr uint32_t kEmbNoKey = 0xFFFFFFFFu;
constexpr int kEmbMaxVec = 8;    // column groups per lane held in registers
constexpr int kEmbSmemChunks = 32;  // chunks staged in shared memory by emb_merge_rank

__global__ void __launch_bounds__(kEmbChunk / 2)
emb_sort_chunks(const int32_t* __restrict__ tokens, int64_t rows, int64_t vocab,
                uint32_t* __restrict__ keys_out, uint32_t* __restrict__ tok_sorted, int* err) {
  __shared__ uint32_t k[kEmbChunk];
  const int64_t r0 = (int64_t)blockIdx.x * kEmbChunk;
  for (int i = threadIdx.x; i < kEmbChunk; i += blockDim.x) {
    uint32_t key = kEmbNoKey;
    if (r0 + i < rows) {
      const int32_t t = tokens[r0 + i];
      if (t < 0 || t >= vocab) set_device_error(err, kDevErrBadIndex);
      else key = ((uint32_t)t << kEmbRowBits) | (uint32_t)i;
    }
    k[i] = key;
    tok_sorted[r0 + i] = kEmbNoKey;  // places no valid row takes stay empty
  }
  __syncthreads();
  for (int size = 2; size <= kEmbChunk; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      const int i = threadIdx.x;  // one compare-exchange per thread
      const int lo = 2 * stride * (i / stride) + (i % stride);
      const int hi = lo + stride;
      const bool up = (lo & size) == 0;
      const uint32_t a = k[lo], b = k[hi];
      if ((a > b) == up) {
        k[lo] = b;
        k[hi] = a;
      }
      __syncthreads();
    }
  }
  for (int i = threadIdx.x; i < kEmbChunk; i += blockDim.x) keys_out[r0 + i] = k[i];
}

// Number of keys of a sorted chunk below x.
__device__ __forceinline__ int emb_count_below(const uint32_t* a, uint32_t x) {
  int lo = 0, hi = kEmbChunk;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (a[mid] < x) lo = mid + 1;
    else hi = mid;
  }
  return lo;
}

__global__ void __launch_bounds__(256)
emb_merge_rank(const uint32_t* __restrict__ keys, int nchunks, uint32_t* __restrict__ tok_sorted,
               uint32_t* __restrict__ row_sorted) {
  extern __shared__ uint32_t sk[];
  const bool staged = nchunks <= kEmbSmemChunks;
  if (staged) {
    for (int i = threadIdx.x; i < nchunks * kEmbChunk; i += blockDim.x) sk[i] = keys[i];
    __syncthreads();
  }
  const uint32_t* src = staged ? sk : keys;
  const int64_t total = (int64_t)nchunks * kEmbChunk;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const uint32_t key = keys[e];
    if (key == kEmbNoKey) continue;
    const uint32_t t = key >> kEmbRowBits;
    const int c = (int)(e / kEmbChunk), i = (int)(e % kEmbChunk);
    int64_t pos = i;
    for (int cc = 0; cc < nchunks; ++cc)
      if (cc != c)
        pos += emb_count_below(src + (int64_t)cc * kEmbChunk,
                               (cc < c ? t + 1 : t) << kEmbRowBits);
    tok_sorted[pos] = t;
    row_sorted[pos] = (uint32_t)(c * kEmbChunk) + (key & (kEmbChunk - 1));
  }
}

// One warp per run start of the globally ordered tokens; columns in groups of
// 32 * 4 * kEmbMaxVec (float4 path) or 32 * kEmbMaxVec.
__global__ void __launch_bounds__(256)
emb_run_sum(const uint32_t* __restrict__ tok_sorted, const uint32_t* __restrict__ row_sorted,
            int64_t n, const float* __restrict__ dout, float* __restrict__ dwte, int dim,
            int vec) {
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  for (int64_t p = (int64_t)blockIdx.x * warps + (threadIdx.x >> 5); p < n;
       p += (int64_t)gridDim.x * warps) {
    const uint32_t t = tok_sorted[p];
    if (t == kEmbNoKey) continue;
    if (p > 0 && tok_sorted[p - 1] == t) continue;  // not the start of a run
    float* dst = dwte + (int64_t)t * dim;
    const int group = (vec ? 4 : 1) * 32 * kEmbMaxVec;
    for (int c0 = 0; c0 < dim; c0 += group) {
      float4 acc[kEmbMaxVec];
#pragma unroll
      for (int u = 0; u < kEmbMaxVec; ++u) {
        const int col = vec ? c0 + 4 * (lane + 32 * u) : c0 + lane + 32 * u;
        acc[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (vec && col < dim) acc[u] = *reinterpret_cast<const float4*>(dst + col);
        else if (!vec && col < dim) acc[u].x = dst[col];
      }
      for (int64_t j = p; j < n && tok_sorted[j] == t; ++j) {
        const float* src = dout + (int64_t)row_sorted[j] * dim;
#pragma unroll
        for (int u = 0; u < kEmbMaxVec; ++u) {
          const int col = vec ? c0 + 4 * (lane + 32 * u) : c0 + lane + 32 * u;
          if (col >= dim) continue;
          if (vec) {
            const float4 d = *reinterpret_cast<const float4*>(src + col);
            acc[u].x = __fadd_rn(acc[u].x, d.x);
            acc[u].y = __fadd_rn(acc[u].y, d.y);
            acc[u].z = __fadd_rn(acc[u].z, d.z);
            acc[u].w = __fadd_rn(acc[u].w, d.w);
          } else {
            acc[u].x = __fadd_rn(acc[u].x, src[col]);
          }
        }
      }
#pragma unroll
      for (int u = 0; u < kEmbMaxVec; ++u) {
        const int col = vec ? c0 + 4 * (lane + 32 * u) : c0 + lane + 32 * u;
        if (vec && col < dim) *reinterpret_cast<float4*>(dst + col) = acc[u];
        else if (!vec && col < dim) dst[col] = acc[u].x;
      }
    }
  }
}

// dwpe[s, i] (+)= sum_b dout[b*seq + s, i], summed in b order (deterministic);
// accumulate = 0 writes the sum.
__global__ void embedding_bwd_pos_kernel(const float* __restrict__ dout, float* __restrict__ dwpe,
                                         int64_t batch, int64_t seq, int dim, int accumulate) {
  int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int64_t total = seq * dim;
  for (; idx < total; idx += (int64_t)gridDim.x * blockDim.x) {
    int64_t s = idx / dim;
    int i = (int)(idx % dim);
    float acc = 0.f;
    for (int64_t b = 0; b < batch; ++b) acc += dout[(b * seq + s) * dim + i];
    dwpe[idx] = accumulate ? dwpe[idx] + acc : acc;
  }
}

// ---- softmax cross-entropy, forward + backward -------------------------------
// Loss.swift:627-660 / GPT main.swift:412-433: shifted = x - max;
// lse = log(sum(exp(shifted))); loss = -(shifted[t] - lse);
// d loss/d x = grad_scale * (softmax(x) - onehot(t)).
template <typename T>
__global__ void __launch_bounds__(1024)
ce_block_kernel(T* __restrict__ logits, const int32_t* __restrict__ targets,
                float* __restrict__ losses, int64_t rows, int classes, int64_t ld,
                float grad_scale, int* err) {
  __shared__ float red[32];
  __shared__ float bcast;
  const int tid = threadIdx.x;
  const int nw = blockDim.x >> 5;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    T* row = logits + r * ld;
    // pass 1: max
    float mx = -INFINITY;
    for (int i = tid; i < classes; i += blockDim.x) mx = fmaxf(mx, to_f32(row[i]));
    mx = warp_max(mx);
    if ((tid & 31) == 0) red[tid >> 5] = mx;
    __syncthreads();
    if (tid < 32) {
      float v = tid < nw ? red[tid] : -INFINITY;
      v = warp_max(v);
      if (tid == 0) bcast = v;
    }
    __syncthreads();
    mx = bcast;
    __syncthreads();
    // pass 2: sum of exp(shifted)
    float s = 0.f;
    for (int i = tid; i < classes; i += blockDim.x) s += expf(to_f32(row[i]) - mx);
    s = warp_sum(s);
    if ((tid & 31) == 0) red[tid >> 5] = s;
    __syncthreads();
    if (tid < 32) {
      float v = tid < nw ? red[tid] : 0.f;
      v = warp_sum(v);
      if (tid == 0) bcast = v;
    }
    __syncthreads();
    const float sum = bcast;
    const float lse = logf(sum);
    int32_t t = targets[r];
    const bool bad = t < 0 || t >= classes;
    if (tid == 0) {
      if (bad) set_device_error(err, kDevErrBadIndex);
      float xt = bad ? mx : to_f32(row[t]);
      losses[r] = -((xt - mx) - lse);
    }
    __syncthreads();  // row[t] read before it is overwritten
    const float inv = 1.0f / sum;
    for (int i = tid; i < (int)ld; i += blockDim.x) {
      float g = 0.f;
      if (i < classes) {
        float p = expf(to_f32(row[i]) - mx) * inv;
        g = grad_scale * (p - (i == t ? 1.f : 0.f));
      }
      row[i] = from_f32<T>(g);
    }
    __syncthreads();
  }
}

// Large class counts, 16-byte-aligned rows with ld % 8 == 0: a CTA per row,
// one read pass with a per-thread online (max, sum of exp) over 8-element
// vectors, a block combine, then one pass that writes the gradient: two reads
// and one write of the row instead of three reads.
__device__ __forceinline__ void online_add(float& m, float& s, float x) {
  if (x > m) {
    s = s * expf(m - x) + 1.0f;
    m = x;
  } else {
    s += expf(x - m);
  }
}
__device__ __forceinline__ void online_merge(float& m, float& s, float m2, float s2) {
  const float mm = fmaxf(m, m2);
  if (mm == -INFINITY) return;
  s = s * expf(m - mm) + s2 * expf(m2 - mm);
  m = mm;
}

template <typename T>
__global__ void __launch_bounds__(512)
ce_block_vec_kernel(T* __restrict__ logits, const int32_t* __restrict__ targets,
                    float* __restrict__ losses, int64_t rows, int classes, int64_t ld,
                    float grad_scale, int* err) {
  __shared__ float red_m[16], red_s[16];
  __shared__ float bm, bs;
  const int tid = threadIdx.x;
  const int nw = blockDim.x >> 5;
  const int nvec = (int)(ld >> 3);
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    T* row = logits + r * ld;
    float m = -INFINITY, s = 0.f;
    for (int vi = tid; vi < nvec; vi += blockDim.x) {
      float v[8];
      load8(row + vi * 8, v);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (vi * 8 + i < classes) online_add(m, s, v[i]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
      const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
      online_merge(m, s, m2, s2);
    }
    if ((tid & 31) == 0) {
      red_m[tid >> 5] = m;
      red_s[tid >> 5] = s;
    }
    __syncthreads();
    if (tid < 32) {
      float mm = tid < nw ? red_m[tid] : -INFINITY;
      float ss = tid < nw ? red_s[tid] : 0.f;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float m2 = __shfl_xor_sync(0xffffffffu, mm, o);
        const float s2 = __shfl_xor_sync(0xffffffffu, ss, o);
        online_merge(mm, ss, m2, s2);
      }
      if (tid == 0) {
        bm = mm;
        bs = ss;
      }
    }
    __syncthreads();
    const float mx = bm, sum = bs;
    const int32_t t = targets[r];
    const bool bad = t < 0 || t >= classes;
    if (tid == 0) {
      if (bad) set_device_error(err, kDevErrBadIndex);
      const float xt = bad ? mx : to_f32(row[t]);
      losses[r] = -((xt - mx) - logf(sum));
    }
    __syncthreads();  // row[t] read before it is overwritten
    const float inv = 1.0f / sum;
    for (int vi = tid; vi < nvec; vi += blockDim.x) {
      float v[8];
      load8(row + vi * 8, v);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int c = vi * 8 + i;
        v[i] = c < classes ? grad_scale * (expf(v[i] - mx) * inv - (c == t ? 1.f : 0.f)) : 0.f;
      }
      store8(row + vi * 8, v);
    }
    __syncthreads();
  }
}

// Softmax cross-entropy from the lm-head GEMM's per-row softmax partials
// (MAGMA_EPI_ROWSTATS: float2 (max, sum exp) per 64-column chunk, chunk-major
// [nchunks][rows]): merge the partials, then one pass over the row writes the
// gradient in place (one read, one write, one exp per element).
template <typename T>
__global__ void __launch_bounds__(512)
ce_rowstats_kernel(T* __restrict__ logits, const float2* __restrict__ stats,
                   const int32_t* __restrict__ targets, float* __restrict__ losses, int64_t rows,
                   int classes, int64_t ld, float grad_scale, int* err) {
  constexpr float kLog2e = 1.4426950408889634f;
  __shared__ float red_m[16], red_s[16];
  __shared__ float bm, bs, bxt;
  const int tid = threadIdx.x;
  const int nw = blockDim.x >> 5;
  const int nvec = (int)(ld >> 3);
  const int nchunks = (classes + 63) >> 6;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    T* row = logits + r * ld;
    float m = -INFINITY, s = 0.f;
    for (int c = tid; c < nchunks; c += blockDim.x) {
      const float2 p = stats[(int64_t)c * rows + r];
      online_merge(m, s, p.x, p.y);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
      const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
      online_merge(m, s, m2, s2);
    }
    if ((tid & 31) == 0) {
      red_m[tid >> 5] = m;
      red_s[tid >> 5] = s;
    }
    const int32_t t = targets[r];
    const bool bad = t < 0 || t >= classes;
    if (tid == 0) bxt = bad ? 0.f : to_f32(row[t]);
    __syncthreads();
    if (tid < 32) {
      float mm = tid < nw ? red_m[tid] : -INFINITY;
      float ss = tid < nw ? red_s[tid] : 0.f;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float m2 = __shfl_xor_sync(0xffffffffu, mm, o);
        const float s2 = __shfl_xor_sync(0xffffffffu, ss, o);
        online_merge(mm, ss, m2, s2);
      }
      if (tid == 0) {
        bm = mm;
        bs = ss;
        if (bad) set_device_error(err, kDevErrBadIndex);
        losses[r] = -(((bad ? mm : bxt) - mm) - logf(ss));
      }
    }
    __syncthreads();  // row[t] read and the row terms published before the row is overwritten
    const float ml = bm * kLog2e, inv = grad_scale / bs;
    for (int vi = tid; vi < nvec; vi += blockDim.x) {
      float v[8];
      load8(row + vi * 8, v);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int c = vi * 8 + i;
        const float p = sm100::ex2_approx(fmaf(v[i], kLog2e, -ml)) * inv;
        v[i] = c < classes ? p - (c == t ? grad_scale : 0.f) : 0.f;
      }
      store8(row + vi * 8, v);
    }
    __syncthreads();
  }
}

// Small class counts: one warp per row.
template <typename T>
__global__ void ce_warp_kernel(T* __restrict__ logits, const int32_t* __restrict__ targets,
                               float* __restrict__ losses, int64_t rows, int classes, int64_t ld,
                               float grad_scale, int* err) {
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  for (int64_t r = (int64_t)blockIdx.x * warps + (threadIdx.x >> 5); r < rows;
       r += (int64_t)gridDim.x * warps) {
    T* row = logits + r * ld;
    float mx = -INFINITY;
    for (int i = lane; i < classes; i += 32) mx = fmaxf(mx, to_f32(row[i]));
    mx = warp_max(mx);
    float s = 0.f;
    for (int i = lane; i < classes; i += 32) s += expf(to_f32(row[i]) - mx);
    s = warp_sum(s);
    const float lse = logf(s);
    int32_t t = targets[r];
    const bool bad = t < 0 || t >= classes;
    float xt = bad ? mx : to_f32(row[bad ? 0 : t]);
    if (lane == 0) {
      if (bad) set_device_error(err, kDevErrBadIndex);
      losses[r] = -((xt - mx) - lse);
    }
    __syncwarp();
    const float inv = 1.0f / s;
    for (int i = lane; i < (int)ld; i += 32) {
      float g = 0.f;
      if (i < classes) {
        float p = expf(to_f32(row[i]) - mx) * inv;
        g = grad_scale * (p - (i == t ? 1.f : 0.f));
      }
      row[i] = from_f32<T>(g);
    }
  }
}

// Deterministic single-CTA sum: fixed per-thread strides, fixed tree.
__global__ void __launch_bounds__(1024)
reduce_sum_kernel(const float* __restrict__ x, float* __restrict__ out, int64_t n, float scale) {
  __shared__ float red[32];
  float s = 0.f;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) s += x[i];
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) out[0] = v * scale;
  }
}

// Mean-squared error of the value-layer example (Examples/ValueLayers/main.swift:
// r = pred - target; loss = sum(r * r) / divisor) and its VJP: the divide's
// pullback gives v = 1 / divisor, the sum's broadcasts it, and the product
// r * r returns v * r to each factor, added: dpred = v * r + v * r. One block;
// every thread sums a fixed stride of elements, then a fixed tree.
__global__ void __launch_bounds__(1024)
mse_kernel(const float* __restrict__ pred, const float* __restrict__ target,
           float* __restrict__ dpred, float* __restrict__ loss, int64_t n, float divisor) {
  __shared__ float red[32];
  const float v = 1.0f / divisor;
  float s = 0.f;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
    const float r = pred[i] - target[i];
    s += r * r;
    if (dpred) dpred[i] = __fadd_rn(__fmul_rn(v, r), __fmul_rn(v, r));
  }
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) loss[0] = t / divisor;
  }
}

// ---- element-wise activations ------------------------------------------------
enum class Act { GeluFwd, GeluBwd, ReluFwd, ReluBwd };

template <typename T, Act A>
__global__ void act_kernel(const T* __restrict__ x, const T* __restrict__ dy, T* __restrict__ y,
                           int64_t n) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    float xv = to_f32(x[i]);
    float r;
    if constexpr (A == Act::GeluFwd) r = gelu_f(xv);
    else if constexpr (A == Act::GeluBwd) r = __fmul_rn(to_f32(dy[i]), gelu_grad_f(xv));
    else if constexpr (A == Act::ReluFwd) r = fmaxf(xv, 0.f);
    else r = xv > 0.f ? to_f32(dy[i]) : 0.f;
    y[i] = from_f32<T>(r);
  }
}

template <Act A>
magma_status_t launch_act(const void* x, const void* dy, void* y, int64_t n, magma_dtype_t dt,
                          cudaStream_t s, const char* name) {
  if (n == 0) return MAGMA_OK;
  int g = grid_for(n, 256);
  if (dt == MAGMA_DTYPE_F32)
    act_kernel<float, A><<<g, 256, 0, s>>>((const float*)x, (const float*)dy, (float*)y, n);
  else
    act_kernel<__nv_bfloat16, A><<<g, 256, 0, s>>>((const __nv_bfloat16*)x,
                                                   (const __nv_bfloat16*)dy, (__nv_bfloat16*)y, n);
  return check_launch(name);
}

// ---- bias gradient -------------------------------------------------------------
// Phase 1: CTA b sums rows [b*rpc, (b+1)*rpc) for 256 columns per CTA-column
// (threads own columns: coalesced); phase 2 sums the partials in CTA order.
constexpr int kBiasMaxRowBlocks = 256;

template <typename T>
__global__ void bias_grad_partial(const T* __restrict__ dy, float* __restrict__ part,
                                  int64_t rows, int cols, int64_t ld, int64_t rows_per_block) {
  int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= cols) return;
  int64_t r0 = (int64_t)blockIdx.y * rows_per_block;
  int64_t r1 = min(rows, r0 + rows_per_block);
  float s = 0.f;
  for (int64_t r = r0; r < r1; ++r) s += to_f32(dy[r * ld + c]);
  part[(int64_t)blockIdx.y * cols + c] = s;
}

// Vectorised partial column sums (cols % 8 == 0, 16-byte aligned rows): a
// 256-thread CTA covers 256 columns (32 groups of 8) x rows_per_block rows;
// thread (group g, phase y) sums rows r0 + y, r0 + y + 8, ... of its 8 columns
// with 16-byte loads, then the 8 phases are added in order (deterministic).
template <typename T>
__global__ void __launch_bounds__(256)
bias_grad_partial_vec(const T* __restrict__ dy, float* __restrict__ part, int64_t rows, int cols,
                      int64_t ld, int64_t rows_per_block) {
  __shared__ float red[8][256 + 4];
  const int g = threadIdx.x & 31, y = threadIdx.x >> 5;
  const int c0 = blockIdx.x * 256 + g * 8;
  const int64_t r0 = (int64_t)blockIdx.y * rows_per_block;
  const int64_t r1 = min(rows, r0 + rows_per_block);
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (c0 < cols) {
#pragma unroll 4
    for (int64_t r = r0 + y; r < r1; r += 8) {
      float v[8];
      load8(dy + r * ld + c0, v);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] += v[i];
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) red[y][g * 8 + i] = acc[i];
  __syncthreads();
  const int c = blockIdx.x * 256 + threadIdx.x;
  if (c < cols) {
    float t = red[0][threadIdx.x];
#pragma unroll
    for (int k = 1; k < 8; ++k) t += red[k][threadIdx.x];
    part[(int64_t)blockIdx.y * cols + c] = t;
  }
}

// Sums the partial rows in a fixed order (32 columns x 8 partial phases per
// CTA, then the 8 phase sums in order).
__global__ void __launch_bounds__(256)
bias_grad_final(const float* __restrict__ part, float* __restrict__ dbias, int nblocks, int cols,
                int accumulate) {
  __shared__ float red[8][33];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + tx;
  float s = 0.f;
  if (c < cols) {
#pragma unroll 4
    for (int b = ty; b < nblocks; b += 8) s += part[(int64_t)b * cols + c];
  }
  red[ty][tx] = s;
  __syncthreads();
  if (ty == 0 && c < cols) {
    float t = red[0][tx];
#pragma unroll
    for (int y = 1; y < 8; ++y) t += red[y][tx];
    dbias[c] = accumulate ? dbias[c] + t : t;
  }
}

int bias_row_blocks(int64_t rows) {
  int64_t b = ceil_div(rows, 64);
  return (int)(b > kBiasMaxRowBlocks ? kBiasMaxRowBlocks : (b < 1 ? 1 : b));
}

template <typename TS, typename TD>
__global__ void convert_kernel(const TS* __restrict__ src, TD* __restrict__ dst, int64_t n) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    dst[i] = from_f32<TD>(to_f32(src[i]));
}

__global__ void scale_kernel(float* __restrict__ y, int64_t n, float alpha) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    y[i] = __fmul_rn(y[i], alpha);
}

}  // namespace
}  // namespace magma

using namespace magma;

extern "C" {

magma_status_t magma_embedding_fwd(const int32_t* tokens, const float* wte, const float* wpe,
                                   float* out, int64_t batch, int64_t seq, int64_t dim,
                                   int64_t vocab, void* stream) {
  MAGMA_REQUIRE(batch >= 0 && seq > 0 && dim > 0 && vocab > 0,
                "magma_embedding_fwd: bad shape");
  int64_t rows = batch * seq;
  if (rows == 0) return MAGMA_OK;
  MAGMA_REQUIRE(tokens && wte && out, "magma_embedding_fwd: NULL pointer");
  int* err = device_error_word();
  embedding_fwd_kernel<<<grid_for(rows, 8), 256, 0, (cudaStream_t)stream>>>(
      tokens, wte, wpe, out, rows, seq, (int)dim, vocab, err);
  return check_launch("embedding_fwd");
}

magma_status_t magma_embedding_bwd(const int32_t* tokens, const float* dout, float* dwte,
                                   float* dwpe, int64_t batch, int64_t seq, int64_t dim,
                                   int64_t vocab, void* stream) {
  MAGMA_REQUIRE(batch >= 0 && seq > 0 && dim > 0 && vocab > 0,
                "magma_embedding_bwd: bad shape");
  int64_t rows = batch * seq;
  if (rows == 0) return MAGMA_OK;
  MAGMA_REQUIRE(tokens && dout && dwte, "magma_embedding_bwd: NULL pointer");
  cudaStream_t s = (cudaStream_t)stream;
  int* err = device_error_word();
  embedding_bwd_tok_kernel<<<grid_for(rows, 8), 256, 0, s>>>(tokens, dout, dwte, rows, (int)dim,
                                                             vocab, err);
  if (magma_status_t st = check_launch("embedding_bwd_tok")) return st;
  if (dwpe != nullptr) {
    embedding_bwd_pos_kernel<<<grid_for(seq * dim, 256), 256, 0, s>>>(dout, dwpe, batch, seq,
                                                                       (int)dim, 1);
    if (magma_status_t st = check_launch("embedding_bwd_pos")) return st;
  }
  return MAGMA_OK;
}

int64_t magma_embedding_bwd_workspace_size(int64_t batch, int64_t seq) {
  const int64_t rows = batch * seq;
  return rows > 0 ? 12 * ceil_div(rows, kEmbChunk) * kEmbChunk : 0;  // keys, tokens, rows
}

magma_status_t magma_embedding_bwd_deterministic(const int32_t* tokens, const float* dout,
                                                 float* dwte, float* dwpe, int64_t batch,
                                                 int64_t seq, int64_t dim, int64_t vocab,
                                                 int32_t accumulate_dwpe, void* workspace,
                                                 int64_t workspace_bytes, void* stream) {
  MAGMA_REQUIRE(batch >= 0 && seq > 0 && dim > 0 && vocab > 0 && dim <= INT32_MAX,
                "magma_embedding_bwd_deterministic: bad shape");
  MAGMA_REQUIRE(vocab < (int64_t)(kEmbNoKey >> kEmbRowBits),
                "magma_embedding_bwd_deterministic: vocab %lld above %u", (long long)vocab,
                kEmbNoKey >> kEmbRowBits);
  const int64_t rows = batch * seq;
  if (rows == 0) return MAGMA_OK;
  MAGMA_REQUIRE(tokens && dout && dwte, "magma_embedding_bwd_deterministic: NULL pointer");
  const int64_t need = magma_embedding_bwd_workspace_size(batch, seq);
  MAGMA_REQUIRE(workspace != nullptr && workspace_bytes >= need && aligned16(workspace),
                "magma_embedding_bwd_deterministic: a 16-byte aligned workspace of %lld bytes "
                "is needed (magma_embedding_bwd_workspace_size)", (long long)need);
  const int64_t nchunks = ceil_div(rows, kEmbChunk);
  MAGMA_REQUIRE(nchunks <= INT32_MAX / kEmbChunk, "magma_embedding_bwd_deterministic: too many rows");
  const int64_t padded = nchunks * kEmbChunk;
  cudaStream_t s = (cudaStream_t)stream;
  uint32_t* keys = static_cast<uint32_t*>(workspace);
  uint32_t* tok_sorted = keys + padded;
  uint32_t* row_sorted = tok_sorted + padded;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    if (magma_status_t st = cuda_status(
            cudaFuncSetAttribute(emb_merge_rank, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 kEmbSmemChunks * kEmbChunk * 4),
            "cudaFuncSetAttribute(emb_merge_rank)"))
      return st;
    attr_set[dev] = true;
  }
  emb_sort_chunks<<<(unsigned)nchunks, kEmbChunk / 2, 0, s>>>(tokens, rows, vocab, keys,
                                                               tok_sorted, device_error_word());
  if (magma_status_t st = check_launch("embedding_bwd_sort")) return st;
  const size_t smem = nchunks <= kEmbSmemChunks ? (size_t)padded * 4 : 0;
  int64_t mb = ceil_div(padded, 256);
  if (mb > 2 * num_sms()) mb = 2 * num_sms();
  emb_merge_rank<<<(unsigned)mb, 256, smem, s>>>(keys, (int)nchunks, tok_sorted, row_sorted);
  if (magma_status_t st = check_launch("embedding_bwd_rank")) return st;
  const int vec = (dim % 4) == 0 && aligned16(dout) && aligned16(dwte);
  emb_run_sum<<<grid_for(rows, 8), 256, 0, s>>>(tok_sorted, row_sorted, padded, dout, dwte,
                                                (int)dim, vec);
  if (magma_status_t st = check_launch("embedding_bwd_runs")) return st;
  if (dwpe != nullptr) {
    embedding_bwd_pos_kernel<<<grid_for(seq * dim, 256), 256, 0, s>>>(dout, dwpe, batch, seq,
                                                                       (int)dim, accumulate_dwpe);
    if (magma_status_t st = check_launch("embedding_bwd_pos")) return st;
  }
  return MAGMA_OK;
}

magma_status_t magma_cross_entropy_fwd_bwd(void* logits, const int32_t* targets, float* losses,
                                           int64_t rows, int64_t classes, int64_t ld,
                                           float grad_scale, magma_dtype_t dtype, void* stream) {
  MAGMA_REQUIRE(rows >= 0 && classes > 0 && ld >= classes && classes < (1LL << 31),
                "magma_cross_entropy_fwd_bwd: bad shape rows=%lld classes=%lld ld=%lld",
                (long long)rows, (long long)classes, (long long)ld);
  MAGMA_REQUIRE(is_float_dtype(dtype), "magma_cross_entropy_fwd_bwd: dtype must be F32 or BF16");
  if (rows == 0) return MAGMA_OK;
  MAGMA_REQUIRE(logits && targets && losses, "magma_cross_entropy_fwd_bwd: NULL pointer");
  cudaStream_t s = (cudaStream_t)stream;
  int* err = device_error_word();
  if (classes <= 2048) {
    int g = grid_for(rows, 8);
    if (dtype == MAGMA_DTYPE_F32)
      ce_warp_kernel<float><<<g, 256, 0, s>>>((float*)logits, targets, losses, rows, (int)classes,
                                              ld, grad_scale, err);
    else
      ce_warp_kernel<__nv_bfloat16><<<g, 256, 0, s>>>((__nv_bfloat16*)logits, targets, losses,
                                                      rows, (int)classes, ld, grad_scale, err);
  } else if (ld % 8 == 0 && aligned16(logits)) {
    int64_t g = rows;
    const int64_t cap = 4LL * num_sms();
    if (g > cap) g = cap;
    if (dtype == MAGMA_DTYPE_F32)
      ce_block_vec_kernel<float><<<(int)g, 512, 0, s>>>((float*)logits, targets, losses, rows,
                                                        (int)classes, ld, grad_scale, err);
    else
      ce_block_vec_kernel<__nv_bfloat16><<<(int)g, 512, 0, s>>>(
          (__nv_bfloat16*)logits, targets, losses, rows, (int)classes, ld, grad_scale, err);
  } else {
    int64_t g = rows;
    int64_t cap = 16LL * num_sms();
    if (g > cap) g = cap;
    if (dtype == MAGMA_DTYPE_F32)
      ce_block_kernel<float><<<(int)g, 1024, 0, s>>>((float*)logits, targets, losses, rows,
                                                     (int)classes, ld, grad_scale, err);
    else
      ce_block_kernel<__nv_bfloat16><<<(int)g, 1024, 0, s>>>(
          (__nv_bfloat16*)logits, targets, losses, rows, (int)classes, ld, grad_scale, err);
  }
  return check_launch("cross_entropy_fwd_bwd");
}

magma_status_t magma_cross_entropy_fwd_bwd_rowstats(void* logits, const void* stats,
                                                    const int32_t* targets, float* losses,
                                                    int64_t rows, int64_t classes, int64_t ld,
                                                    float grad_scale, magma_dtype_t dtype,
                                                    void* stream) {
  MAGMA_REQUIRE(rows >= 0 && classes > 0 && ld >= classes && classes < (1LL << 31),
                "magma_cross_entropy_fwd_bwd_rowstats: bad shape rows=%lld classes=%lld ld=%lld",
                (long long)rows, (long long)classes, (long long)ld);
  MAGMA_REQUIRE(dtype == MAGMA_DTYPE_BF16, "magma_cross_entropy_fwd_bwd_rowstats: BF16 logits only");
  if (rows == 0) return MAGMA_OK;
  MAGMA_REQUIRE(logits && stats && targets && losses,
                "magma_cross_entropy_fwd_bwd_rowstats: NULL pointer");
  MAGMA_REQUIRE(ld % 8 == 0 && aligned16(logits) && (reinterpret_cast<uintptr_t>(stats) & 7u) == 0,
                "magma_cross_entropy_fwd_bwd_rowstats: ld must be a multiple of 8, logits 16-byte "
                "and stats 8-byte aligned");
  int64_t g = rows;
  const int64_t cap = 4LL * num_sms();
  if (g > cap) g = cap;
  ce_rowstats_kernel<__nv_bfloat16><<<(int)g, 512, 0, (cudaStream_t)stream>>>(
      (__nv_bfloat16*)logits, static_cast<const float2*>(stats), targets, losses, rows,
      (int)classes, ld, grad_scale, device_error_word());
  return check_launch("cross_entropy_fwd_bwd_rowstats");
}

magma_status_t magma_reduce_sum(const float* x, float* out, int64_t n, float scale, void* stream) {
  MAGMA_REQUIRE(n >= 0, "magma_reduce_sum: negative size");
  MAGMA_REQUIRE(out != nullptr && (n == 0 || x != nullptr), "magma_reduce_sum: NULL pointer");
  reduce_sum_kernel<<<1, 1024, 0, (cudaStream_t)stream>>>(x, out, n, scale);
  return check_launch("reduce_sum");
}

magma_status_t magma_mse_fwd_bwd(const float* pred, const float* target, float* dpred,
                                float* loss, int64_t n, float divisor, void* stream) {
  MAGMA_REQUIRE(n >= 0 && divisor > 0.f, "magma_mse_fwd_bwd: bad arguments n=%lld divisor=%g",
                (long long)n, (double)divisor);
  MAGMA_REQUIRE(loss != nullptr && (n == 0 || (pred && target)), "magma_mse_fwd_bwd: NULL pointer");
  mse_kernel<<<1, 1024, 0, (cudaStream_t)stream>>>(pred, target, dpred, loss, n, divisor);
  return check_launch("mse");
}

magma_status_t magma_gelu_fwd(const void* x, void* y, int64_t n, magma_dtype_t dtype,
                              void* stream) {
  MAGMA_REQUIRE(n >= 0 && is_float_dtype(dtype), "magma_gelu_fwd: bad arguments");
  MAGMA_REQUIRE(n == 0 || (x && y), "magma_gelu_fwd: NULL pointer");
  return launch_act<Act::GeluFwd>(x, nullptr, y, n, dtype, (cudaStream_t)stream, "gelu_fwd");
}

magma_status_t magma_gelu_bwd(const void* x, const void* dy, void* dx, int64_t n,
                              magma_dtype_t dtype, void* stream) {
  MAGMA_REQUIRE(n >= 0 && is_float_dtype(dtype), "magma_gelu_bwd: bad arguments");
  MAGMA_REQUIRE(n == 0 || (x && dy && dx), "magma_gelu_bwd: NULL pointer");
  return launch_act<Act::GeluBwd>(x, dy, dx, n, dtype, (cudaStream_t)stream, "gelu_bwd");
}

magma_status_t magma_relu_fwd(const void* x, void* y, int64_t n, magma_dtype_t dtype,
                              void* stream) {
  MAGMA_REQUIRE(n >= 0 && is_float_dtype(dtype), "magma_relu_fwd: bad arguments");
  MAGMA_REQUIRE(n == 0 || (x && y), "magma_relu_fwd: NULL pointer");
  return launch_act<Act::ReluFwd>(x, nullptr, y, n, dtype, (cudaStream_t)stream, "relu_fwd");
}

magma_status_t magma_relu_bwd(const void* x, const void* dy, void* dx, int64_t n,
                              magma_dtype_t dtype, void* stream) {
  MAGMA_REQUIRE(n >= 0 && is_float_dtype(dtype), "magma_relu_bwd: bad arguments");
  MAGMA_REQUIRE(n == 0 || (x && dy && dx), "magma_relu_bwd: NULL pointer");
  return launch_act<Act::ReluBwd>(x, dy, dx, n, dtype, (cudaStream_t)stream, "relu_bwd");
}

size_t magma_bias_grad_workspace_size(int64_t rows, int64_t cols) {
  if (rows <= 0 || cols <= 0) return 0;
  return (size_t)bias_row_blocks(rows) * (size_t)cols * sizeof(float);
}

magma_status_t magma_bias_grad(const void* dy, float* dbias, int64_t rows, int64_t cols,
                               int64_t ld, magma_dtype_t dtype, int32_t accumulate,
                               void* workspace, size_t workspace_bytes, void* stream) {
  MAGMA_REQUIRE(rows >= 0 && cols > 0 && ld >= cols && cols < (1LL << 31),
                "magma_bias_grad: bad shape");
  MAGMA_REQUIRE(is_float_dtype(dtype), "magma_bias_grad: dtype must be F32 or BF16");
  MAGMA_REQUIRE(dbias != nullptr, "magma_bias_grad: NULL dbias");
  cudaStream_t s = (cudaStream_t)stream;
  if (rows == 0) {
    if (!accumulate) return magma_memset(dbias, 0, (size_t)cols * sizeof(float), stream);
    return MAGMA_OK;
  }
  MAGMA_REQUIRE(dy != nullptr, "magma_bias_grad: NULL dy");
  size_t need = magma_bias_grad_workspace_size(rows, cols);
  MAGMA_REQUIRE(workspace != nullptr && workspace_bytes >= need,
                "magma_bias_grad: workspace of %zu bytes needed, %zu given", need,
                workspace_bytes);
  int nb = bias_row_blocks(rows);
  int64_t rpb = ceil_div(rows, nb);
  dim3 grid((unsigned)ceil_div(cols, 256), (unsigned)nb);
  float* part = (float*)workspace;
  const size_t esz = dtype == MAGMA_DTYPE_F32 ? 4 : 2;
  if (cols % 8 == 0 && ld % 8 == 0 && aligned16(dy) && (ld * esz) % 16 == 0) {
    // 256-row blocks: enough CTAs to fill the GPU, few partial rows
    nb = (int)ceil_div(rows, 256);
    if (nb > kBiasMaxRowBlocks) nb = kBiasMaxRowBlocks;
    rpb = ceil_div(rows, nb);
    grid = dim3((unsigned)ceil_div(cols, 256), (unsigned)nb);
    if (dtype == MAGMA_DTYPE_F32)
      bias_grad_partial_vec<float><<<grid, 256, 0, s>>>((const float*)dy, part, rows, (int)cols,
                                                        ld, rpb);
    else
      bias_grad_partial_vec<__nv_bfloat16><<<grid, 256, 0, s>>>((const __nv_bfloat16*)dy, part,
                                                                rows, (int)cols, ld, rpb);
  } else if (dtype == MAGMA_DTYPE_F32)
    bias_grad_partial<float><<<grid, 256, 0, s>>>((const float*)dy, part, rows, (int)cols, ld, rpb);
  else
    bias_grad_partial<__nv_bfloat16><<<grid, 256, 0, s>>>((const __nv_bfloat16*)dy, part, rows,
                                                          (int)cols, ld, rpb);
  if (magma_status_t st = check_launch("bias_grad_partial")) return st;
  bias_grad_final<<<(unsigned)ceil_div(cols, 32), 256, 0, s>>>(part, dbias, nb, (int)cols,
                                                               accumulate);
  return check_launch("bias_grad_final");
}

magma_status_t magma_convert(const void* src, void* dst, int64_t n, magma_dtype_t src_dtype,
                             magma_dtype_t dst_dtype, void* stream) {
  MAGMA_REQUIRE(n >= 0 && is_float_dtype(src_dtype) && is_float_dtype(dst_dtype),
                "magma_convert: unsupported conversion %s -> %s", dtype_name(src_dtype),
                dtype_name(dst_dtype));
  if (n == 0) return MAGMA_OK;
  MAGMA_REQUIRE(src && dst, "magma_convert: NULL pointer");
  cudaStream_t s = (cudaStream_t)stream;
  int g = grid_for(n, 256);
  if (src_dtype == MAGMA_DTYPE_F32 && dst_dtype == MAGMA_DTYPE_BF16)
    convert_kernel<float, __nv_bfloat16><<<g, 256, 0, s>>>((const float*)src,
                                                           (__nv_bfloat16*)dst, n);
  else if (src_dtype == MAGMA_DTYPE_BF16 && dst_dtype == MAGMA_DTYPE_F32)
    convert_kernel<__nv_bfloat16, float><<<g, 256, 0, s>>>((const __nv_bfloat16*)src,
                                                           (float*)dst, n);
  else if (src_dtype == MAGMA_DTYPE_F32)
    convert_kernel<float, float><<<g, 256, 0, s>>>((const float*)src, (float*)dst, n);
  else
    convert_kernel<__nv_bfloat16, __nv_bfloat16><<<g, 256, 0, s>>>(
        (const __nv_bfloat16*)src, (__nv_bfloat16*)dst, n);
  return check_launch("convert");
}

magma_status_t magma_scale(float* y, int64_t n, float alpha, void* stream) {
  MAGMA_REQUIRE(n >= 0, "magma_scale: negative size");
  if (n == 0) return MAGMA_OK;
  MAGMA_REQUIRE(y != nullptr, "magma_scale: NULL pointer");
  scale_kernel<<<grid_for(n, 256), 256, 0, (cudaStream_t)stream>>>(y, n, alpha);
  return check_launch("scale");
}

}  // extern "C"
