// Causal scaled-dot-product attention, F32-accurate SIMT path.
//
// Restates the GPT block's attention (Benchmarks/GPT2Shakespeare/Sources/
// main.swift:467-481) and nn.scaledDotProductAttention (Sources/Core/
// Module.swift:2408-2441): S = (Q.K^T)*scale, masked keys (key > query) get
// -1e9 (main.swift:793-801) — here they contribute exactly zero, which is what
// exp(-1e9 - max) rounds to in F32 — P = softmax(S), O = P.V. The reference
// materialises S and P ([B,H,S,S]); this kernel streams 64-key tiles with an
// online softmax and keeps O in registers (flash-style), writing O and the
// row log-sum-exp.
//
// Backward restates the VJP chain (vjpBatchedMatmul Autodiff.swift:309-317,
// vjpSoftmax :379-386, scale multiply :76-82) with P recomputed from lse:
//   delta_i = rowsum(dO*O) (= sum_j dP_ij P_ij), dS = P*(dP - delta),
//   dV = P^T.dO, dK = scale*dS^T.Q (one CTA per key tile, loop over queries),
//   dQ = scale*dS.K (one CTA per query tile, loop over keys).
// Every output element is accumulated by one thread in a fixed order, so the
// results are deterministic (no atomics).
//
// Tile: 64 queries x 64 keys, 256 threads; thread (ty, tx) = (tid/16, tid%16)
// owns rows ty+16i and columns tx+16j, so shared-memory reads are broadcast or
// conflict-free with a +1 row pad. head_dim is zero-padded to HD (64 or 128).
#include <cmath>

#include "common.cuh"

namespace magma {
namespace {

constexpr int kT = 64;        // queries / keys per tile
constexpr int kThreads = 256;

struct AttnGeom {
  int64_t batch, heads, seq, hd;
  int64_t qs[3];  // Q/K/V strides: batch, head, seq (elements)
  int64_t os[3];  // O/dO strides
  float scale;
  int causal;
};

template <typename T>
__device__ __forceinline__ const T* head_ptr(const T* base, const int64_t* st, int64_t b,
                                             int64_t h) {
  return base + b * st[0] + h * st[1];
}

// Loads rows [r0, r0+64) x [0, hd) of a [seq, hd] head into smem[64][HD+1] as
// F32, zero-filling rows >= seq and columns >= hd.
template <int HD, typename T>
__device__ __forceinline__ void load_tile(float* dst, const T* src, int64_t row_stride,
                                          int64_t r0, int64_t seq, int64_t hd) {
  for (int idx = threadIdx.x; idx < kT * HD; idx += kThreads) {
    int r = idx / HD, d = idx % HD;
    float v = 0.f;
    if (r0 + r < seq && d < hd) v = to_f32(src[(r0 + r) * row_stride + d]);
    dst[r * (HD + 1) + d] = v;
  }
}

template <int HD, typename T>
__global__ void __launch_bounds__(kThreads)
attn_fwd_simt(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
              T* __restrict__ o, float* __restrict__ lse, AttnGeom g) {
  extern __shared__ float sm[];
  float* Qs = sm;
  float* Ks = Qs + kT * (HD + 1);
  float* Vs = Ks + kT * (HD + 1);
  float* Ps = Vs + kT * (HD + 1);  // [64][65]
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  const int nq = (int)((g.seq + kT - 1) / kT);
  const int qt = nq - 1 - (int)blockIdx.x;  // heaviest (causal) tiles first
  const int64_t h = blockIdx.y, b = blockIdx.z;
  const int64_t q0 = (int64_t)qt * kT;
  const T* qh = head_ptr(q, g.qs, b, h);
  const T* kh = head_ptr(k, g.qs, b, h);
  const T* vh = head_ptr(v, g.qs, b, h);
  load_tile<HD>(Qs, qh, g.qs[2], q0, g.seq, g.hd);
  constexpr int DJ = HD / 16;
  float acc[4][DJ];
  float m[4], l[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.f;
#pragma unroll
    for (int j = 0; j < DJ; ++j) acc[i][j] = 0.f;
  }
  const int nk = g.causal ? qt + 1 : nq;
  for (int kt = 0; kt < nk; ++kt) {
    const int64_t k0 = (int64_t)kt * kT;
    __syncthreads();
    load_tile<HD>(Ks, kh, g.qs[2], k0, g.seq, g.hd);
    load_tile<HD>(Vs, vh, g.qs[2], k0, g.seq, g.hd);
    __syncthreads();
    float s[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) s[i][j] = 0.f;
    for (int d = 0; d < HD; ++d) {
      float qv[4], kv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) qv[i] = Qs[(ty + 16 * i) * (HD + 1) + d];
#pragma unroll
      for (int j = 0; j < 4; ++j) kv[j] = Ks[(tx + 16 * j) * (HD + 1) + d];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) s[i][j] = fmaf(qv[i], kv[j], s[i][j]);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t qi = q0 + ty + 16 * i;
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int64_t kj = k0 + tx + 16 * j;
        float val = s[i][j] * g.scale;
        if (kj >= g.seq || (g.causal && kj > qi)) val = -INFINITY;
        s[i][j] = val;
        mx = fmaxf(mx, val);
      }
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float mnew = fmaxf(m[i], mx);
      // Rows past seq may see only masked keys; keep them finite.
      const float mref = mnew == -INFINITY ? 0.f : mnew;
      const float alpha = expf(m[i] - mref);
      float rs = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float p = expf(s[i][j] - mref);
        s[i][j] = p;
        rs += p;
      }
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) rs += __shfl_xor_sync(0xffffffffu, rs, o);
      l[i] = l[i] * alpha + rs;
      m[i] = mnew;
#pragma unroll
      for (int j = 0; j < DJ; ++j) acc[i][j] *= alpha;
#pragma unroll
      for (int j = 0; j < 4; ++j) Ps[(ty + 16 * i) * (kT + 1) + tx + 16 * j] = s[i][j];
    }
    __syncthreads();
    for (int c = 0; c < kT; ++c) {
      float pv[4], vv[DJ];
#pragma unroll
      for (int i = 0; i < 4; ++i) pv[i] = Ps[(ty + 16 * i) * (kT + 1) + c];
#pragma unroll
      for (int j = 0; j < DJ; ++j) vv[j] = Vs[c * (HD + 1) + tx + 16 * j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < DJ; ++j) acc[i][j] = fmaf(pv[i], vv[j], acc[i][j]);
    }
  }
  T* oh = o + b * g.os[0] + h * g.os[1];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t qi = q0 + ty + 16 * i;
    if (qi >= g.seq) continue;
    const float inv = 1.0f / l[i];
#pragma unroll
    for (int j = 0; j < DJ; ++j) {
      const int d = tx + 16 * j;
      if (d < g.hd) oh[qi * g.os[2] + d] = from_f32<T>(acc[i][j] * inv);
    }
    if (tx == 0 && lse != nullptr) lse[(b * g.heads + h) * g.seq + qi] = m[i] + logf(l[i]);
  }
}

// delta[b,h,i] = sum_d dO[i,d] * O[i,d]; one warp per row.
template <typename T>
__global__ void attn_bwd_delta(const T* __restrict__ o, const T* __restrict__ d_o,
                               float* __restrict__ delta, AttnGeom g) {
  const int lane = threadIdx.x & 31;
  const int64_t rows = g.batch * g.heads * g.seq;
  for (int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows;
       r += (int64_t)gridDim.x * (blockDim.x >> 5)) {
    const int64_t s = r % g.seq, bh = r / g.seq, h = bh % g.heads, b = bh / g.heads;
    const int64_t off = b * g.os[0] + h * g.os[1] + s * g.os[2];
    float acc = 0.f;
    for (int d = lane; d < g.hd; d += 32) acc += to_f32(d_o[off + d]) * to_f32(o[off + d]);
    acc = warp_sum(acc);
    if (lane == 0) delta[r] = acc;
  }
}

// One CTA per (key tile, head, batch): dK, dV for 64 keys.
template <int HD, typename T>
__global__ void __launch_bounds__(kThreads)
attn_bwd_dkdv_simt(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                   const T* __restrict__ d_o, const float* __restrict__ lse,
                   const float* __restrict__ delta, T* __restrict__ dk, T* __restrict__ dv,
                   AttnGeom g) {
  extern __shared__ float sm[];
  float* Ks = sm;
  float* Vs = Ks + kT * (HD + 1);
  float* Qs = Vs + kT * (HD + 1);
  float* dOs = Qs + kT * (HD + 1);
  float* Ps = dOs + kT * (HD + 1);   // [q][k], 64 x 65
  float* dSs = Ps + kT * (kT + 1);   // [q][k]
  float* Ls = dSs + kT * (kT + 1);   // lse of the q tile
  float* Ds = Ls + kT;               // delta of the q tile
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  const int nq = (int)((g.seq + kT - 1) / kT);
  const int kt = (int)blockIdx.x;
  const int64_t h = blockIdx.y, b = blockIdx.z;
  const int64_t k0 = (int64_t)kt * kT;
  const int64_t bh = b * g.heads + h;
  const T* qh = head_ptr(q, g.qs, b, h);
  const T* kh = head_ptr(k, g.qs, b, h);
  const T* vh = head_ptr(v, g.qs, b, h);
  const T* doh = d_o + b * g.os[0] + h * g.os[1];
  load_tile<HD>(Ks, kh, g.qs[2], k0, g.seq, g.hd);
  load_tile<HD>(Vs, vh, g.qs[2], k0, g.seq, g.hd);
  constexpr int DJ = HD / 16;
  float adk[4][DJ], adv[4][DJ];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < DJ; ++j) adk[i][j] = adv[i][j] = 0.f;
  for (int qt = g.causal ? kt : 0; qt < nq; ++qt) {
    const int64_t q0 = (int64_t)qt * kT;
    __syncthreads();
    load_tile<HD>(Qs, qh, g.qs[2], q0, g.seq, g.hd);
    load_tile<HD>(dOs, doh, g.os[2], q0, g.seq, g.hd);
    if (tid < kT) {
      const int64_t qi = q0 + tid;
      Ls[tid] = qi < g.seq ? lse[bh * g.seq + qi] : 0.f;
      Ds[tid] = qi < g.seq ? delta[bh * g.seq + qi] : 0.f;
    }
    __syncthreads();
    // thread owns queries ty+16i, keys tx+16j
    float s[4][4], dp[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) s[i][j] = dp[i][j] = 0.f;
    for (int d = 0; d < HD; ++d) {
      float qv[4], ov[4], kv[4], vv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        qv[i] = Qs[(ty + 16 * i) * (HD + 1) + d];
        ov[i] = dOs[(ty + 16 * i) * (HD + 1) + d];
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        kv[j] = Ks[(tx + 16 * j) * (HD + 1) + d];
        vv[j] = Vs[(tx + 16 * j) * (HD + 1) + d];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          s[i][j] = fmaf(qv[i], kv[j], s[i][j]);
          dp[i][j] = fmaf(ov[i], vv[j], dp[i][j]);
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int qi_l = ty + 16 * i;
      const int64_t qi = q0 + qi_l;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int kj_l = tx + 16 * j;
        const int64_t kj = k0 + kj_l;
        float p = 0.f;
        if (qi < g.seq && kj < g.seq && !(g.causal && kj > qi))
          p = expf(s[i][j] * g.scale - Ls[qi_l]);
        Ps[qi_l * (kT + 1) + kj_l] = p;
        dSs[qi_l * (kT + 1) + kj_l] = p * (dp[i][j] - Ds[qi_l]) * g.scale;
      }
    }
    __syncthreads();
    // dV[key][d] += sum_q P[q][key] dO[q][d]; dK[key][d] += sum_q dS[q][key] Q[q][d]
    for (int c = 0; c < kT; ++c) {
      float pv[4], sv[4], ov[DJ], qv[DJ];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        pv[i] = Ps[c * (kT + 1) + ty + 16 * i];
        sv[i] = dSs[c * (kT + 1) + ty + 16 * i];
      }
#pragma unroll
      for (int j = 0; j < DJ; ++j) {
        ov[j] = dOs[c * (HD + 1) + tx + 16 * j];
        qv[j] = Qs[c * (HD + 1) + tx + 16 * j];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < DJ; ++j) {
          adv[i][j] = fmaf(pv[i], ov[j], adv[i][j]);
          adk[i][j] = fmaf(sv[i], qv[j], adk[i][j]);
        }
    }
  }
  T* dkh = dk + b * g.qs[0] + h * g.qs[1];
  T* dvh = dv + b * g.qs[0] + h * g.qs[1];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t kj = k0 + ty + 16 * i;
    if (kj >= g.seq) continue;
#pragma unroll
    for (int j = 0; j < DJ; ++j) {
      const int d = tx + 16 * j;
      if (d < g.hd) {
        dkh[kj * g.qs[2] + d] = from_f32<T>(adk[i][j]);
        dvh[kj * g.qs[2] + d] = from_f32<T>(adv[i][j]);
      }
    }
  }
}

// One CTA per (query tile, head, batch): dQ for 64 queries.
template <int HD, typename T>
__global__ void __launch_bounds__(kThreads)
attn_bwd_dq_simt(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                 const T* __restrict__ d_o, const float* __restrict__ lse,
                 const float* __restrict__ delta, T* __restrict__ dq, AttnGeom g) {
  extern __shared__ float sm[];
  float* Qs = sm;
  float* dOs = Qs + kT * (HD + 1);
  float* Ks = dOs + kT * (HD + 1);
  float* Vs = Ks + kT * (HD + 1);
  float* dSs = Vs + kT * (HD + 1);  // [q][k]
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  const int nq = (int)((g.seq + kT - 1) / kT);
  const int qt = nq - 1 - (int)blockIdx.x;
  const int64_t h = blockIdx.y, b = blockIdx.z;
  const int64_t q0 = (int64_t)qt * kT;
  const int64_t bh = b * g.heads + h;
  const T* qh = head_ptr(q, g.qs, b, h);
  const T* kh = head_ptr(k, g.qs, b, h);
  const T* vh = head_ptr(v, g.qs, b, h);
  const T* doh = d_o + b * g.os[0] + h * g.os[1];
  load_tile<HD>(Qs, qh, g.qs[2], q0, g.seq, g.hd);
  load_tile<HD>(dOs, doh, g.os[2], q0, g.seq, g.hd);
  float lq[4], dq_[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t qi = q0 + ty + 16 * i;
    lq[i] = qi < g.seq ? lse[bh * g.seq + qi] : 0.f;
    dq_[i] = qi < g.seq ? delta[bh * g.seq + qi] : 0.f;
  }
  constexpr int DJ = HD / 16;
  float acc[4][DJ];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < DJ; ++j) acc[i][j] = 0.f;
  const int nk = g.causal ? qt + 1 : nq;
  for (int kt = 0; kt < nk; ++kt) {
    const int64_t k0 = (int64_t)kt * kT;
    __syncthreads();
    load_tile<HD>(Ks, kh, g.qs[2], k0, g.seq, g.hd);
    load_tile<HD>(Vs, vh, g.qs[2], k0, g.seq, g.hd);
    __syncthreads();
    float s[4][4], dp[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) s[i][j] = dp[i][j] = 0.f;
    for (int d = 0; d < HD; ++d) {
      float qv[4], ov[4], kv[4], vv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        qv[i] = Qs[(ty + 16 * i) * (HD + 1) + d];
        ov[i] = dOs[(ty + 16 * i) * (HD + 1) + d];
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        kv[j] = Ks[(tx + 16 * j) * (HD + 1) + d];
        vv[j] = Vs[(tx + 16 * j) * (HD + 1) + d];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          s[i][j] = fmaf(qv[i], kv[j], s[i][j]);
          dp[i][j] = fmaf(ov[i], vv[j], dp[i][j]);
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int qi_l = ty + 16 * i;
      const int64_t qi = q0 + qi_l;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int kj_l = tx + 16 * j;
        const int64_t kj = k0 + kj_l;
        float p = 0.f;
        if (qi < g.seq && kj < g.seq && !(g.causal && kj > qi)) p = expf(s[i][j] * g.scale - lq[i]);
        dSs[qi_l * (kT + 1) + kj_l] = p * (dp[i][j] - dq_[i]) * g.scale;
      }
    }
    __syncthreads();
    for (int c = 0; c < kT; ++c) {
      float sv[4], kv[DJ];
#pragma unroll
      for (int i = 0; i < 4; ++i) sv[i] = dSs[(ty + 16 * i) * (kT + 1) + c];
#pragma unroll
      for (int j = 0; j < DJ; ++j) kv[j] = Ks[c * (HD + 1) + tx + 16 * j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < DJ; ++j) acc[i][j] = fmaf(sv[i], kv[j], acc[i][j]);
    }
  }
  T* dqh = dq + b * g.qs[0] + h * g.qs[1];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t qi = q0 + ty + 16 * i;
    if (qi >= g.seq) continue;
#pragma unroll
    for (int j = 0; j < DJ; ++j) {
      const int d = tx + 16 * j;
      if (d < g.hd) dqh[qi * g.qs[2] + d] = from_f32<T>(acc[i][j]);
    }
  }
}

template <int HD>
constexpr size_t fwd_smem() { return (size_t)(3 * kT * (HD + 1) + kT * (kT + 1)) * sizeof(float); }
template <int HD>
constexpr size_t dkdv_smem() {
  return (size_t)(4 * kT * (HD + 1) + 2 * kT * (kT + 1) + 2 * kT) * sizeof(float);
}
template <int HD>
constexpr size_t dq_smem() { return (size_t)(4 * kT * (HD + 1) + kT * (kT + 1)) * sizeof(float); }

template <typename K>
magma_status_t set_smem(K kern, size_t bytes) {
  return cuda_status(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)bytes),
                     "cudaFuncSetAttribute(attention)");
}

template <int HD, typename T>
magma_status_t fwd_simt(const void* q, const void* k, const void* v, void* o, float* lse,
                        const AttnGeom& g, cudaStream_t s) {
  auto kern = attn_fwd_simt<HD, T>;
  if (magma_status_t st = set_smem(kern, fwd_smem<HD>())) return st;
  dim3 grid((unsigned)ceil_div(g.seq, kT), (unsigned)g.heads, (unsigned)g.batch);
  kern<<<grid, kThreads, fwd_smem<HD>(), s>>>((const T*)q, (const T*)k, (const T*)v, (T*)o, lse, g);
  return check_launch("attention_fwd_f32");
}

template <int HD, typename T>
magma_status_t bwd_simt(const void* q, const void* k, const void* v, const void* o,
                        const void* d_o, const float* lse, void* dq, void* dk, void* dv,
                        float* delta, const AttnGeom& g, cudaStream_t s) {
  const int64_t rows = g.batch * g.heads * g.seq;
  int64_t blocks = ceil_div(rows, 8);
  if (blocks > 16LL * num_sms()) blocks = 16LL * num_sms();
  attn_bwd_delta<T><<<(int)blocks, 256, 0, s>>>((const T*)o, (const T*)d_o, delta, g);
  if (magma_status_t st = check_launch("attention_bwd_delta")) return st;
  dim3 grid((unsigned)ceil_div(g.seq, kT), (unsigned)g.heads, (unsigned)g.batch);
  auto k1 = attn_bwd_dkdv_simt<HD, T>;
  if (magma_status_t st = set_smem(k1, dkdv_smem<HD>())) return st;
  k1<<<grid, kThreads, dkdv_smem<HD>(), s>>>((const T*)q, (const T*)k, (const T*)v,
                                             (const T*)d_o, lse, delta, (T*)dk, (T*)dv, g);
  if (magma_status_t st = check_launch("attention_bwd_dkdv_f32")) return st;
  auto k2 = attn_bwd_dq_simt<HD, T>;
  if (magma_status_t st = set_smem(k2, dq_smem<HD>())) return st;
  k2<<<grid, kThreads, dq_smem<HD>(), s>>>((const T*)q, (const T*)k, (const T*)v, (const T*)d_o,
                                           lse, delta, (T*)dq, g);
  return check_launch("attention_bwd_dq_f32");
}

}  // namespace

// delta[b,h,i] = sum_d dO*O for the backward kernels (F32 or BF16 inputs).
magma_status_t attention_bwd_delta(const void* o, const void* d_o, float* delta, int64_t batch,
                                   int64_t heads, int64_t seq, int64_t hd, const int64_t* os,
                                   magma_dtype_t dtype, cudaStream_t s) {
  AttnGeom g{batch, heads, seq, hd, {0, 0, 0}, {os[0], os[1], os[2]}, 0.f, 0};
  const int64_t rows = batch * heads * seq;
  int64_t blocks = ceil_div(rows, 8);
  if (blocks > 16LL * num_sms()) blocks = 16LL * num_sms();
  if (dtype == MAGMA_DTYPE_F32)
    attn_bwd_delta<float><<<(int)blocks, 256, 0, s>>>((const float*)o, (const float*)d_o, delta, g);
  else
    attn_bwd_delta<__nv_bfloat16><<<(int)blocks, 256, 0, s>>>(
        (const __nv_bfloat16*)o, (const __nv_bfloat16*)d_o, delta, g);
  return check_launch("attention_bwd_delta");
}

// Entry points used by attention.cu's dispatcher.
magma_status_t attention_fwd_simt(const void* q, const void* k, const void* v, void* o,
                                  float* lse, int64_t batch, int64_t heads, int64_t seq,
                                  int64_t hd, const int64_t* qs, const int64_t* os, float scale,
                                  int causal, magma_dtype_t dtype, cudaStream_t s) {
  AttnGeom g{batch, heads, seq, hd, {qs[0], qs[1], qs[2]}, {os[0], os[1], os[2]}, scale, causal};
  const bool f32 = dtype == MAGMA_DTYPE_F32;
  if (hd <= 64)
    return f32 ? fwd_simt<64, float>(q, k, v, o, lse, g, s)
               : fwd_simt<64, __nv_bfloat16>(q, k, v, o, lse, g, s);
  return f32 ? fwd_simt<128, float>(q, k, v, o, lse, g, s)
             : fwd_simt<128, __nv_bfloat16>(q, k, v, o, lse, g, s);
}

magma_status_t attention_bwd_simt(const void* q, const void* k, const void* v, const void* o,
                                  const void* d_o, const float* lse, void* dq, void* dk, void* dv,
                                  float* delta, int64_t batch, int64_t heads, int64_t seq,
                                  int64_t hd, const int64_t* qs, const int64_t* os, float scale,
                                  int causal, magma_dtype_t dtype, cudaStream_t s) {
  AttnGeom g{batch, heads, seq, hd, {qs[0], qs[1], qs[2]}, {os[0], os[1], os[2]}, scale, causal};
  const bool f32 = dtype == MAGMA_DTYPE_F32;
  if (hd <= 64)
    return f32 ? bwd_simt<64, float>(q, k, v, o, d_o, lse, dq, dk, dv, delta, g, s)
               : bwd_simt<64, __nv_bfloat16>(q, k, v, o, d_o, lse, dq, dk, dv, delta, g, s);
  return f32 ? bwd_simt<128, float>(q, k, v, o, d_o, lse, dq, dk, dv, delta, g, s)
             : bwd_simt<128, __nv_bfloat16>(q, k, v, o, d_o, lse, dq, dk, dv, delta, g, s);
}

}  // namespace magma
