// LayerNorm forward and backward.
//
// Forward restates nn.LayerNorm.forward (Sources/Core/Module.swift:2754-2791)
// and the GPT block's layerNorm (Benchmarks/GPT2Shakespeare/Sources/main.swift:
// 364-375): mean = sum/D, var = sum((x-mean)^2)/D (population), std =
// sqrt(var+eps), y = ((x-mean)/std)*gamma + beta. The reference divides by std
// (it never multiplies by rsqrt); here the per-element quotient is a multiply
// by RN(1/std) with one Markstein residual correction, which reproduces the
// correctly rounded divide except in rare one-ulp cases.
//
// Backward is the closed form of the reference's autodiff chain through that
// forward (vjpDivide/vjpSqrt/vjpMeanDims/vjpMultiply with sumAlongBroadcastDims,
// Sources/Core/Autodiff.swift:57-94,221-257,351-370; Optimizer.swift:627-633).
//
// Both directions are HBM-bound row kernels. The main path (D % 8 == 0,
// D <= 1024, 16-byte aligned rows) is a persistent grid of one CTA per SM in
// which every warp streams its rows through a small ring of row buffers in
// shared memory: lane 0 fills a buffer with untiled bulk copies
// (cp.async.bulk) that complete on that buffer's mbarrier, so the next rows
// of every warp are in flight while it reduces the current one. Lane l works
// on the 4-element groups 4l + 128c of a row: 16-byte conflict-free shared
// reads, 512-byte coalesced global stores per warp instruction. Reductions
// are warp-shuffle butterflies in a fixed order (deterministic). dgamma/dbeta
// partials stay in registers (each lane owns fixed columns), are summed over
// the CTA's warps in warp order into one partial row per CTA in the caller's
// workspace, then over CTAs in CTA order by a second kernel. Other shapes use
// scalar generic kernels.
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "sm100.cuh"

namespace magma {
namespace {

using sm100::bulk_load;
using sm100::fence_barrier_init;
using sm100::mbar_expect_tx;
using sm100::mbar_init;
using sm100::mbar_wait;
using sm100::smem_u32;

constexpr int kWarps = 8;            // warps per CTA of the generic kernels
constexpr int kMaxBwdBlocks = 592;   // cap on per-CTA partial rows (4 x 148 SMs)

// Row-streaming kernels.
constexpr int kMaxGroups = 8;               // 4-element groups per lane: D <= 1024
constexpr int kStreamSmem = 200 * 1024;     // dynamic shared memory for the rings
constexpr int kBarBytes = 1024;             // mbarrier area at the start of it
constexpr int kFwdRing = 3;                 // row buffers per warp, forward
constexpr int kBwdRing = 2;                 // row buffers per warp, backward
// Forward warps per CTA (128 registers per thread at 16; the widest rows,
// G = 8, run 12). Deeper rings with fewer warps (5 buffers x 12 warps forward,
// 3 x 12 backward) measured slower at [8192, 768] (7.1 -> 7.4 us forward,
// 15.4 -> 16.6 us backward in A/B runs on one box).
constexpr int fwd_max_warps(int groups) { return groups > 6 ? 12 : 16; }
// Backward warps per CTA: 12 keep 170 registers per thread; the widest rows
// (G = 8) need more and run 8 warps.
constexpr int bwd_max_warps(int groups, bool res = false) {
  return (groups > 6 || res) ? 8 : 12;
}

bool stream_ok(int dim) { return dim % 8 == 0 && dim <= kMaxGroups * 128; }

// Warps per CTA whose rings fit the shared-memory budget (0: none fit).
int stream_warps(int ring, size_t row_bytes, int max_warps) {
  int w = (int)((kStreamSmem - kBarBytes) / ((size_t)ring * row_bytes));
  if (w > max_warps) w = max_warps;
  if (w * ring * 8 > kBarBytes) w = kBarBytes / (ring * 8);
  return w < 4 ? 0 : w;
}

// After a failed wait: one more bounded wait on each row copy still in flight
// (rows j0 .. j1-1 of the warp) so the CTA does not leave while bulk copies
// still target its shared memory.
template <int RING>
__device__ void drain_ring(const uint64_t* bars, int64_t j0, int64_t j1, int* err) {
  for (int64_t k = j0; k < j1; ++k)
    mbar_wait(smem_u32(bars + k % RING), (uint32_t)((k / RING) & 1), err);
}

// Forward, streaming: G 4-element groups per lane (D <= 128*G).
template <int G, typename TX, typename TY>
__global__ void __launch_bounds__(fwd_max_warps(G) * 32, 1)
ln_fwd_stream(const TX* __restrict__ x, const float* __restrict__ gamma,
              const float* __restrict__ beta, TY* __restrict__ y, float* __restrict__ mean_out,
              float* __restrict__ rstd_out, int64_t rows, int dim, float eps, int* err) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int nwarps = blockDim.x >> 5;
  const uint32_t row_bytes = (uint32_t)dim * sizeof(TX);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem) + warp * kFwdRing;
  unsigned char* ring = smem + kBarBytes + (size_t)warp * kFwdRing * row_bytes;
  const int64_t stride = (int64_t)gridDim.x * nwarps;
  const int64_t first = (int64_t)blockIdx.x * nwarps + warp;
  const int64_t n = first < rows ? (rows - first + stride - 1) / stride : 0;
  if (lane == 0) {
    for (int b = 0; b < kFwdRing; ++b) mbar_init(smem_u32(bars + b), 1);
    fence_barrier_init();
    for (int64_t j = 0; j < n && j < kFwdRing; ++j) {
      const uint32_t bar = smem_u32(bars + j);
      mbar_expect_tx(bar, row_bytes);
      bulk_load(smem_u32(ring + j * row_bytes), x + (first + j * stride) * dim, row_bytes, bar);
    }
  }
  __syncwarp();
  // gamma / beta of this lane's columns as packed F32 pairs
  unsigned long long g2[G][2], b2[G][2];
#pragma unroll
  for (int c = 0; c < G; ++c) {
    const int e = 128 * c + 4 * lane;
    float gv[4] = {0.f, 0.f, 0.f, 0.f}, bv[4] = {0.f, 0.f, 0.f, 0.f};
    if (e < dim) {
      load4(gamma + e, gv);
      load4(beta + e, bv);
    }
    g2[c][0] = f2_pack(gv[0], gv[1]);
    g2[c][1] = f2_pack(gv[2], gv[3]);
    b2[c][0] = f2_pack(bv[0], bv[1]);
    b2[c][1] = f2_pack(bv[2], bv[3]);
  }
  for (int64_t j = 0; j < n; ++j) {
    const int slot = (int)(j % kFwdRing);
    const int64_t row = first + j * stride;
    if (!mbar_wait(smem_u32(bars + slot), (uint32_t)((j / kFwdRing) & 1), err)) {
      drain_ring<kFwdRing>(bars, j, n < j + kFwdRing ? n : j + kFwdRing, err);
      return;
    }
    const TX* src = reinterpret_cast<const TX*>(ring + slot * row_bytes);
    // the row as packed pairs (columns 4l + 128c + {0,1} and {2,3}); zero
    // past the end of a short row
    unsigned long long v[G][2];
#pragma unroll
    for (int c = 0; c < G; ++c) {
      const int e = 128 * c + 4 * lane;
      float t[4] = {0.f, 0.f, 0.f, 0.f};
      if (e < dim) load4(src + e, t);
      v[c][0] = f2_pack(t[0], t[1]);
      v[c][1] = f2_pack(t[2], t[3]);
    }
    __syncwarp();
    if (lane == 0 && j + kFwdRing < n) {
      const uint32_t bar = smem_u32(bars + slot);
      mbar_expect_tx(bar, row_bytes);
      bulk_load(smem_u32(ring + slot * row_bytes), x + (row + kFwdRing * stride) * dim,
                row_bytes, bar);
    }
    // sums on packed pairs (two running sums per lane, added at the end)
    unsigned long long acc = f2_pack(0.f, 0.f);
#pragma unroll
    for (int c = 0; c < G; ++c) acc = f2_add(acc, f2_add(v[c][0], v[c][1]));
    float s0, s1;
    f2_unpack(acc, s0, s1);
    const float mean = __fdiv_rn(warp_sum(__fadd_rn(s0, s1)), (float)dim);
    const unsigned long long mean2 = f2_pack(mean, mean);
    unsigned long long sq = f2_pack(0.f, 0.f);
#pragma unroll
    for (int c = 0; c < G; ++c) {
      const bool live = 128 * c + 4 * lane < dim;
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const unsigned long long d = f2_sub(v[c][i], mean2);
        v[c][i] = d;
        if (live) sq = f2_fma(d, d, sq);
      }
    }
    float q0, q1;
    f2_unpack(sq, q0, q1);
    const float ss = warp_sum(__fadd_rn(q0, q1));
    const float stdv = __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)dim), eps));
    // (x - mean) / std per element as q = d * RN(1/std); for an F32 output one
    // residual correction follows (Markstein's method: e = d - q*std exact by
    // FMA, q' = q + e*r), which gives the correctly rounded quotient of the
    // reference's divide in all but rare one-ulp cases. A BF16 output keeps q:
    // the one-ulp F32 difference is far below the BF16 rounding step.
    const float rinv = __frcp_rn(stdv);
    const unsigned long long r2 = f2_pack(rinv, rinv), ns2 = f2_pack(-stdv, -stdv);
    TY* yr = y + row * dim;
#pragma unroll
    for (int c = 0; c < G; ++c) {
      const int e = 128 * c + 4 * lane;
      if (e < dim) {
        float o[4];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          unsigned long long q = f2_mul(v[c][i], r2);
          if (std::is_same<TY, float>::value) q = f2_fma(f2_fma(q, ns2, v[c][i]), r2, q);
          f2_unpack(f2_add(f2_mul(q, g2[c][i]), b2[c][i]), o[2 * i], o[2 * i + 1]);
        }
        store4(yr + e, o);
      }
    }
    if (lane == 0) {
      if (mean_out) mean_out[row] = mean;
      if (rstd_out) rstd_out[row] = __fdiv_rn(1.0f, stdv);
    }
  }
}

// Any D (scalar loads, row re-read from L1/L2 for each pass).
template <typename TX, typename TY>
__global__ void __launch_bounds__(kWarps * 32)
ln_fwd_generic(const TX* __restrict__ x, const float* __restrict__ gamma,
               const float* __restrict__ beta, TY* __restrict__ y, float* __restrict__ mean_out,
               float* __restrict__ rstd_out, int64_t rows, int dim, float eps) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  for (int64_t row = (int64_t)blockIdx.x * kWarps + warp; row < rows;
       row += (int64_t)gridDim.x * kWarps) {
    const TX* xr = x + row * dim;
    float s = 0.f;
    for (int i = lane; i < dim; i += 32) s += to_f32(xr[i]);
    s = warp_sum(s);
    const float mean = __fdiv_rn(s, (float)dim);
    float ss = 0.f;
    for (int i = lane; i < dim; i += 32) {
      float d = __fsub_rn(to_f32(xr[i]), mean);
      ss += d * d;
    }
    ss = warp_sum(ss);
    const float stdv = __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)dim), eps));
    TY* yr = y + row * dim;
    for (int i = lane; i < dim; i += 32) {
      float d = __fsub_rn(to_f32(xr[i]), mean);
      yr[i] = from_f32<TY>(__fadd_rn(__fmul_rn(__fdiv_rn(d, stdv), gamma[i]), beta[i]));
    }
    if (lane == 0) {
      if (mean_out) mean_out[row] = mean;
      if (rstd_out) rstd_out[row] = __fdiv_rn(1.0f, stdv);
    }
  }
}

// Backward, streaming: each ring buffer holds [x | dy | dx] of one row (dx
// only when accumulating into it). dgamma/dbeta partials live in registers
// (lane l owns columns 4l + 128c) and are summed over the warps of the CTA in
// warp order into part[blockIdx.x] = [dgamma | dbeta].
// RES (residual stream, F32 dx): also writes a BF16 copy of the final dx
// (dx_bf16, optional) and accumulates its column sums as a third partial row
// [dgamma | dbeta | dcol].
template <int G, bool RES, typename TDY, typename TX, typename TDX>
__global__ void __launch_bounds__(bwd_max_warps(G, RES) * 32, 1)
ln_bwd_stream(const TDY* __restrict__ dy, const TX* __restrict__ x,
              const float* __restrict__ gamma, const float* __restrict__ mean_in,
              const float* __restrict__ rstd_in, TDX* __restrict__ dx,
              __nv_bfloat16* __restrict__ dx_bf16, float* __restrict__ part, int64_t rows,
              int dim, int accumulate_dx, int* err) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int nwarps = blockDim.x >> 5;
  const uint32_t bx = (uint32_t)dim * sizeof(TX);
  const uint32_t bdy = (uint32_t)dim * sizeof(TDY);
  const uint32_t bdx = accumulate_dx ? (uint32_t)dim * sizeof(TDX) : 0u;
  const uint32_t stage = bx + bdy + bdx;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem) + warp * kBwdRing;
  unsigned char* ring = smem + kBarBytes + (size_t)warp * kBwdRing * stage;
  const int64_t stride = (int64_t)gridDim.x * nwarps;
  const int64_t first = (int64_t)blockIdx.x * nwarps + warp;
  const int64_t n = first < rows ? (rows - first + stride - 1) / stride : 0;
  auto issue = [&](int slot, int64_t row) {
    const uint32_t bar = smem_u32(bars + slot);
    const uint32_t dst = smem_u32(ring + (size_t)slot * stage);
    mbar_expect_tx(bar, stage);
    bulk_load(dst, x + row * dim, bx, bar);
    bulk_load(dst + bx, dy + row * dim, bdy, bar);
    if (bdx) bulk_load(dst + bx + bdy, dx + row * dim, bdx, bar);
  };
  if (lane == 0) {
    for (int b = 0; b < kBwdRing; ++b) mbar_init(smem_u32(bars + b), 1);
    fence_barrier_init();
    for (int64_t j = 0; j < n && j < kBwdRing; ++j) issue((int)j, first + j * stride);
  }
  __syncwarp();
  float g[G][4], dg[G][4], db[G][4], dc[RES ? G : 1][4];
#pragma unroll
  for (int c = 0; c < G; ++c) {
    const int e = 128 * c + 4 * lane;
    if (e < dim) load4(gamma + e, g[c]);
#pragma unroll
    for (int i = 0; i < 4; ++i) dg[c][i] = db[c][i] = 0.f;
    if (RES)
#pragma unroll
      for (int i = 0; i < 4; ++i) dc[RES ? c : 0][i] = 0.f;
  }
  bool ok = true;
  // Row statistics of this warp's rows, 32 rows at a time: lane i holds those
  // of row j0 + i (loaded together, ahead of use), broadcast by shuffles.
  float st_mean = 0.f, st_rstd = 0.f;
  for (int64_t j = 0; j < n; ++j) {
    const int slot = (int)(j % kBwdRing);
    const int64_t row = first + j * stride;
    if ((j & 31) == 0) {
      const int64_t jl = j + lane;
      if (jl < n) {
        st_mean = mean_in[first + jl * stride];
        st_rstd = rstd_in[first + jl * stride];
      }
    }
    const float mean = __shfl_sync(0xffffffffu, st_mean, (int)(j & 31));
    const float rstd = __shfl_sync(0xffffffffu, st_rstd, (int)(j & 31));
    if (!mbar_wait(smem_u32(bars + slot), (uint32_t)((j / kBwdRing) & 1), err)) {
      drain_ring<kBwdRing>(bars, j, n < j + kBwdRing ? n : j + kBwdRing, err);
      ok = false;
      break;
    }
    const unsigned char* st = ring + (size_t)slot * stage;
    const TX* xs = reinterpret_cast<const TX*>(st);
    const TDY* dys = reinterpret_cast<const TDY*>(st + bx);
    float xv[G][4], dv[G][4];
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int c = 0; c < G; ++c) {
      const int e = 128 * c + 4 * lane;
      if (e < dim) {
        load4(xs + e, xv[c]);
        load4(dys + e, dv[c]);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float xhat = (xv[c][i] - mean) * rstd;
          const float gg = dv[c][i] * g[c][i];
          dg[c][i] += dv[c][i] * xhat;
          db[c][i] += dv[c][i];
          xv[c][i] = xhat;
          dv[c][i] = gg;
          s1 += gg;
          s2 += gg * xhat;
        }
      }
    }
    s1 = warp_sum(s1) / (float)dim;
    s2 = warp_sum(s2) / (float)dim;
    const float* dxs = reinterpret_cast<const float*>(st + bx + bdy);
    TDX* dst = dx + row * dim;
#pragma unroll
    for (int c = 0; c < G; ++c) {
      const int e = 128 * c + 4 * lane;
      if (e < dim) {
        float o[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) o[i] = rstd * (dv[c][i] - s1 - xv[c][i] * s2);
        if (accumulate_dx) {
          float prev[4];
          load4(dxs + e, prev);
#pragma unroll
          for (int i = 0; i < 4; ++i) o[i] += prev[i];
        }
        store4(dst + e, o);
        if (RES) {
#pragma unroll
          for (int i = 0; i < 4; ++i) dc[RES ? c : 0][i] += o[i];
          if (dx_bf16 != nullptr) store4(dx_bf16 + row * dim + e, o);
        }
      }
    }
    __syncwarp();
    if (lane == 0 && j + kBwdRing < n) issue(slot, row + kBwdRing * stride);
  }
  // This warp's ring (all its copies have landed) now holds its partials.
  float* red = reinterpret_cast<float*>(ring);
#pragma unroll
  for (int c = 0; c < G; ++c) {
    const int e = 128 * c + 4 * lane;
    if (e < dim) {
      store4(red + e, dg[c]);
      store4(red + dim + e, db[c]);
      if (RES) store4(red + 2 * dim + e, dc[RES ? c : 0]);
    }
  }
  __syncthreads();
  if (!ok) return;
  const int width = (RES ? 3 : 2) * dim;
  float* out = part + (int64_t)blockIdx.x * width;
  const size_t wstride = (size_t)kBwdRing * stage / sizeof(float);
  const float* base = reinterpret_cast<const float*>(smem + kBarBytes);
  for (int i = threadIdx.x; i < width; i += blockDim.x) {
    float t = base[i];
    for (int w = 1; w < nwarps; ++w) t += base[(size_t)w * wstride + i];
    out[i] = t;
  }
}

template <typename TDY, typename TX, typename TDX>
__global__ void __launch_bounds__(kWarps * 32)
ln_bwd_generic(const TDY* __restrict__ dy, const TX* __restrict__ x,
               const float* __restrict__ gamma, const float* __restrict__ mean_in,
               const float* __restrict__ rstd_in, TDX* __restrict__ dx,
               float* __restrict__ part, int64_t rows, int dim, int accumulate_dx) {
  // Per-CTA partials accumulated column-wise: each CTA owns a contiguous row
  // range; threads own columns (coalesced), rows visited in order.
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int64_t rows_per_cta = (rows + gridDim.x - 1) / gridDim.x;
  const int64_t r0 = (int64_t)blockIdx.x * rows_per_cta;
  const int64_t r1 = min(rows, r0 + rows_per_cta);
  // dx: one warp per row within the range.
  for (int64_t row = r0 + warp; row < r1; row += kWarps) {
    const float mean = mean_in[row], rstd = rstd_in[row];
    float s1 = 0.f, s2 = 0.f;
    for (int i = lane; i < dim; i += 32) {
      float xhat = (to_f32(x[row * dim + i]) - mean) * rstd;
      float gg = to_f32(dy[row * dim + i]) * gamma[i];
      s1 += gg;
      s2 += gg * xhat;
    }
    s1 = warp_sum(s1) / (float)dim;
    s2 = warp_sum(s2) / (float)dim;
    for (int i = lane; i < dim; i += 32) {
      float xhat = (to_f32(x[row * dim + i]) - mean) * rstd;
      float gg = to_f32(dy[row * dim + i]) * gamma[i];
      float o = rstd * (gg - s1 - xhat * s2);
      if (accumulate_dx) o += to_f32(dx[row * dim + i]);
      dx[row * dim + i] = from_f32<TDX>(o);
    }
  }
  float* out = part + (int64_t)blockIdx.x * 2 * dim;
  for (int col = threadIdx.x; col < dim; col += blockDim.x) {
    float sg = 0.f, sb = 0.f;
    for (int64_t row = r0; row < r1; ++row) {
      float d = to_f32(dy[row * dim + col]);
      sg += d * ((to_f32(x[row * dim + col]) - mean_in[row]) * rstd_in[row]);
      sb += d;
    }
    out[col] = sg;
    out[dim + col] = sb;
  }
}

// Sums per-CTA partial rows: out_k[c] (+)= sum_b part[b][k*dim + c] for the
// outputs k = 0, 1, 2 (dgamma, dbeta, dcol; a null output is skipped). A
// 32 x 32 CTA covers 32 columns; row y of threads sums partials b = y, y+32,
// ... in order, issuing the loads of 8 rows before the first add (the kernel
// is load-latency bound: ~150 partial rows of a few KB), then the 32 sums are
// added in y order (fixed order: deterministic).
constexpr int kReduceRows = 32;
__global__ void __launch_bounds__(32 * kReduceRows)
reduce_partials(const float* __restrict__ part, int nblocks, int width, float* __restrict__ out0,
                float* __restrict__ out1, float* __restrict__ out2, int dim, int accumulate) {
  __shared__ float red[kReduceRows][33];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + tx;
  float s = 0.f;
  if (c < width) {
    for (int b0 = ty; b0 < nblocks; b0 += 8 * kReduceRows) {
      float v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int b = b0 + j * kReduceRows;
        v[j] = b < nblocks ? part[(int64_t)b * width + c] : 0.f;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (b0 + j * kReduceRows < nblocks) s += v[j];
    }
  }
  red[ty][tx] = s;
  __syncthreads();
  if (ty == 0 && c < width) {
    float t = red[0][tx];
#pragma unroll
    for (int y = 1; y < kReduceRows; ++y) t += red[y][tx];
    const int k = c / dim;
    float* out = k == 0 ? out0 : (k == 1 ? out1 : out2);
    if (out == nullptr) return;
    float* dst = out + (c - k * dim);
    *dst = accumulate ? *dst + t : t;
  }
}

void launch_reduce_partials(const float* part, int nblocks, int width, float* out0, float* out1,
                            float* out2, int dim, int accumulate, cudaStream_t stream) {
  reduce_partials<<<(width + 31) / 32, 32 * kReduceRows, 0, stream>>>(part, nblocks, width, out0,
                                                                      out1, out2, dim, accumulate);
}

int bwd_blocks(int64_t rows) {
  int64_t b = ceil_div(rows, kWarps);
  int64_t cap = 2LL * num_sms();
  if (cap > kMaxBwdBlocks) cap = kMaxBwdBlocks;
  if (b > cap) b = cap;
  if (b < 1) b = 1;
  return (int)b;
}

// CTAs of a streaming launch: one per SM at most, no more than the rows need,
// and no more than the partial rows the backward workspace holds.
int stream_blocks(int64_t rows, int warps) {
  int64_t b = ceil_div(rows, warps);
  if (b > num_sms()) b = num_sms();
  int64_t cap = ceil_div(rows, kWarps);
  if (cap > kMaxBwdBlocks) cap = kMaxBwdBlocks;
  if (b > cap) b = cap;
  return b < 1 ? 1 : (int)b;
}

template <typename K>
void set_dynamic_smem(K kern, size_t bytes) {
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

// Backward through ln_bwd_stream when the shape and alignment allow it
// (*launched false otherwise). *blocks: CTAs launched = partial rows written;
// at most `max_blocks`.
template <typename TDY, typename TX, typename TDX, bool RES = false>
magma_status_t launch_bwd_stream(const void* dy, const void* x, const float* gamma,
                                 const float* mean, const float* rstd, void* dx, int64_t rows,
                                 int dim, int acc_dx, float* part, int max_blocks, int* blocks,
                                 bool* launched, cudaStream_t stream, void* dx_bf16 = nullptr) {
  *launched = false;
  if (!stream_ok(dim) || !aligned16(x) || !aligned16(dy) || !aligned16(dx) || !aligned16(gamma) ||
      !aligned16(dx_bf16))
    return MAGMA_OK;
  const size_t stage =
      (size_t)dim * (sizeof(TX) + sizeof(TDY) + (acc_dx ? sizeof(TDX) : 0));
  // the partial rows are staged in each warp's ring at the end
  if (kBwdRing * stage < (size_t)(RES ? 3 : 2) * dim * sizeof(float)) return MAGMA_OK;
  const int groups = ((dim + 255) / 256) * 2;
  const int warps = stream_warps(kBwdRing, stage, bwd_max_warps(groups, RES));
  if (warps == 0) return MAGMA_OK;
  int b = stream_blocks(rows, warps);
  if (b > max_blocks) b = max_blocks;
  *blocks = b;
  const size_t smem = kBarBytes + (size_t)warps * kBwdRing * stage;
#define LN_BWD_STREAM(G)                                                                        \
  do {                                                                                          \
    auto kern = ln_bwd_stream<G, RES, TDY, TX, TDX>;                                            \
    set_dynamic_smem(kern, smem);                                                               \
    kern<<<b, warps * 32, smem, stream>>>((const TDY*)dy, (const TX*)x, gamma, mean, rstd,      \
                                          (TDX*)dx, (__nv_bfloat16*)dx_bf16, part, rows, dim,   \
                                          acc_dx, device_error_word());                         \
  } while (0)
  if (groups == 2) LN_BWD_STREAM(2);
  else if (groups == 4) LN_BWD_STREAM(4);
  else if (groups == 6) LN_BWD_STREAM(6);
  else LN_BWD_STREAM(8);
#undef LN_BWD_STREAM
  *launched = true;
  return check_launch("layernorm_bwd");
}

template <typename TX, typename TY>
magma_status_t launch_fwd(const void* x, const float* gamma, const float* beta, void* y,
                          float* mean, float* rstd, int64_t rows, int dim, float eps,
                          cudaStream_t stream) {
  const bool vec = stream_ok(dim) && aligned16(x) && aligned16(y) && aligned16(gamma) &&
                   aligned16(beta);
  const int groups = ((dim + 255) / 256) * 2;
  const int warps =
      vec ? stream_warps(kFwdRing, (size_t)dim * sizeof(TX), fwd_max_warps(groups)) : 0;
  if (warps > 0) {
    int64_t b = ceil_div(rows, warps);
    if (b > num_sms()) b = num_sms();
    const size_t smem = kBarBytes + (size_t)warps * kFwdRing * dim * sizeof(TX);
#define LN_FWD_STREAM(G)                                                                        \
  do {                                                                                          \
    auto kern = ln_fwd_stream<G, TX, TY>;                                                       \
    set_dynamic_smem(kern, smem);                                                               \
    kern<<<(int)b, warps * 32, smem, stream>>>((const TX*)x, gamma, beta, (TY*)y, mean, rstd,   \
                                               rows, dim, eps, device_error_word());            \
  } while (0)
    if (groups == 2) LN_FWD_STREAM(2);
    else if (groups == 4) LN_FWD_STREAM(4);
    else if (groups == 6) LN_FWD_STREAM(6);
    else LN_FWD_STREAM(8);
#undef LN_FWD_STREAM
  } else {
    int64_t blocks = ceil_div(rows, kWarps);
    const int64_t cap = 16LL * num_sms();
    if (blocks > cap) blocks = cap;
    ln_fwd_generic<TX, TY><<<(int)blocks, kWarps * 32, 0, stream>>>(
        (const TX*)x, gamma, beta, (TY*)y, mean, rstd, rows, dim, eps);
  }
  return check_launch("layernorm_fwd");
}

template <typename TDY, typename TX, typename TDX>
magma_status_t launch_bwd(const void* dy, const void* x, const float* gamma, const float* mean,
                          const float* rstd, void* dx, float* dgamma, float* dbeta,
                          int64_t rows, int dim, int acc_dx, int acc_params, float* part,
                          cudaStream_t stream) {
  int blocks = bwd_blocks(rows);
  bool streamed = false;
  if (magma_status_t st = launch_bwd_stream<TDY, TX, TDX>(dy, x, gamma, mean, rstd, dx, rows, dim,
                                                          acc_dx, part, kMaxBwdBlocks, &blocks,
                                                          &streamed, stream))
    return st;
  if (!streamed) {
    ln_bwd_generic<TDY, TX, TDX><<<blocks, kWarps * 32, 0, stream>>>(
        (const TDY*)dy, (const TX*)x, gamma, mean, rstd, (TDX*)dx, part, rows, dim, acc_dx);
  }
  if (magma_status_t s = check_launch("layernorm_bwd")) return s;
  if (dgamma != nullptr || dbeta != nullptr) {
    int width = 2 * dim;
    launch_reduce_partials(part, blocks, width, dgamma, dbeta, nullptr, dim, acc_params, stream);
    if (magma_status_t s = check_launch("layernorm_bwd_reduce")) return s;
  }
  return MAGMA_OK;
}

// ---- allocation-free backward --------------------------------------------
// Scratch for magma_layernorm_bwd_noalloc: one partial row of [dgamma | dbeta]
// per CTA. Bounds: at most kNoAllocMaxBlocks CTAs and dim <= kNoAllocMaxDim,
// i.e. 296 x 2 x 1024 floats = 2.3 MiB, held on every GPU that loads the
// library until the process exits.
constexpr int kNoAllocMaxDim = 1024;
constexpr int kNoAllocMaxBlocks = 296;
static __device__ __align__(256) float g_ln_bwd_scratch[kNoAllocMaxBlocks * 2 * kNoAllocMaxDim];

constexpr int kNoAllocMaxDevices = 64;
float* g_noalloc_ptr[kNoAllocMaxDevices] = {nullptr};
std::mutex g_noalloc_mu;

// Device address of the scratch array on the current device, resolved once per
// device with that device current. Host code must not use the array's name as
// a pointer: on the host it only stands in for the symbol.
magma_status_t noalloc_scratch(float** out) {
  int dev = 0;
  if (magma_status_t st = cuda_status(cudaGetDevice(&dev), "cudaGetDevice")) return st;
  if (dev < 0 || dev >= kNoAllocMaxDevices)
    return fail(MAGMA_UNIMPLEMENTED, "magma_layernorm_bwd_noalloc: device ordinal %d >= %d", dev,
                kNoAllocMaxDevices);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    cudaError_t err = cudaGetSymbolAddress(&p, g_ln_bwd_scratch);
    if (err != cudaSuccess)
      return cuda_status(err, "cudaGetSymbolAddress(layernorm backward scratch)");
    g_noalloc_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_noalloc_ptr[dev];
  return MAGMA_OK;
}

template <typename TDY, typename TX, typename TDX>
magma_status_t launch_bwd_noalloc(const void* dy, const void* x, const float* gamma,
                                  const float* mean, const float* rstd, void* dx, float* dgamma,
                                  float* dbeta, int64_t rows, int dim, int acc_dx, int acc_params,
                                  float* part, cudaStream_t stream) {
  int blocks = bwd_blocks(rows);
  if (blocks > kNoAllocMaxBlocks) blocks = kNoAllocMaxBlocks;
  bool streamed = false;
  if (magma_status_t st = launch_bwd_stream<TDY, TX, TDX>(dy, x, gamma, mean, rstd, dx, rows, dim,
                                                          acc_dx, part, kNoAllocMaxBlocks,
                                                          &blocks, &streamed, stream))
    return st;
  if (!streamed) {
    ln_bwd_generic<TDY, TX, TDX><<<blocks, kWarps * 32, 0, stream>>>(
        (const TDY*)dy, (const TX*)x, gamma, mean, rstd, (TDX*)dx, part, rows, dim, acc_dx);
  }
  if (magma_status_t s = check_launch("layernorm_bwd_noalloc")) return s;
  if (dgamma != nullptr || dbeta != nullptr) {
    const int width = 2 * dim;
    launch_reduce_partials(part, blocks, width, dgamma, dbeta, nullptr, dim, acc_params, stream);
    if (magma_status_t s = check_launch("layernorm_bwd_noalloc_reduce")) return s;
  }
  return MAGMA_OK;
}

}  // namespace
}  // namespace magma

using namespace magma;

extern "C" {

magma_status_t magma_layernorm_fwd(const void* x, const float* gamma, const float* beta, void* y,
                                   float* mean, float* rstd, int64_t rows, int64_t dim, float eps,
                                   magma_dtype_t x_dtype, magma_dtype_t y_dtype, void* stream) {
  MAGMA_REQUIRE(rows >= 0 && dim > 0 && dim <= (1 << 20),
                "magma_layernorm_fwd: bad shape rows=%lld dim=%lld", (long long)rows,
                (long long)dim);
  MAGMA_REQUIRE(is_float_dtype(x_dtype) && is_float_dtype(y_dtype),
                "magma_layernorm_fwd: unsupported dtypes x=%s y=%s", dtype_name(x_dtype),
                dtype_name(y_dtype));
  if (rows == 0) return MAGMA_OK;
  MAGMA_REQUIRE(x && gamma && beta && y, "magma_layernorm_fwd: NULL pointer");
  cudaStream_t s = (cudaStream_t)stream;
  const int d = (int)dim;
  if (x_dtype == MAGMA_DTYPE_F32 && y_dtype == MAGMA_DTYPE_F32)
    return launch_fwd<float, float>(x, gamma, beta, y, mean, rstd, rows, d, eps, s);
  if (x_dtype == MAGMA_DTYPE_F32 && y_dtype == MAGMA_DTYPE_BF16)
    return launch_fwd<float, __nv_bfloat16>(x, gamma, beta, y, mean, rstd, rows, d, eps, s);
  if (x_dtype == MAGMA_DTYPE_BF16 && y_dtype == MAGMA_DTYPE_F32)
    return launch_fwd<__nv_bfloat16, float>(x, gamma, beta, y, mean, rstd, rows, d, eps, s);
  return launch_fwd<__nv_bfloat16, __nv_bfloat16>(x, gamma, beta, y, mean, rstd, rows, d, eps, s);
}

size_t magma_layernorm_bwd_workspace_size(int64_t rows, int64_t dim) {
  if (rows <= 0 || dim <= 0) return 0;
  int64_t b = ceil_div(rows, kWarps);
  if (b > kMaxBwdBlocks) b = kMaxBwdBlocks;
  return (size_t)b * 2 * (size_t)dim * sizeof(float);
}

magma_status_t magma_layernorm_bwd(const void* dy, const void* x, const float* gamma,
                                   const float* mean, const float* rstd, void* dx, float* dgamma,
                                   float* dbeta, int64_t rows, int64_t dim,
                                   magma_dtype_t dy_dtype, magma_dtype_t x_dtype,
                                   magma_dtype_t dx_dtype, int32_t accumulate_dx,
                                   int32_t accumulate_params, void* workspace,
                                   size_t workspace_bytes, void* stream) {
  MAGMA_REQUIRE(rows >= 0 && dim > 0 && dim <= 8192,
                "magma_layernorm_bwd: bad shape rows=%lld dim=%lld (dim <= 8192)",
                (long long)rows, (long long)dim);
  MAGMA_REQUIRE(is_float_dtype(dy_dtype) && is_float_dtype(x_dtype) && is_float_dtype(dx_dtype),
                "magma_layernorm_bwd: unsupported dtypes");
  MAGMA_REQUIRE(!accumulate_dx || dx_dtype == MAGMA_DTYPE_F32,
                "magma_layernorm_bwd: accumulate_dx needs an F32 dx");
  if (rows == 0) return MAGMA_OK;
  MAGMA_REQUIRE(dy && x && gamma && mean && rstd && dx, "magma_layernorm_bwd: NULL pointer");
  size_t need = magma_layernorm_bwd_workspace_size(rows, dim);
  MAGMA_REQUIRE(workspace != nullptr && workspace_bytes >= need,
                "magma_layernorm_bwd: workspace of %zu bytes needed, %zu given", need,
                workspace_bytes);
  cudaStream_t s = (cudaStream_t)stream;
  float* part = (float*)workspace;
  const int d = (int)dim;
  const bool f_dy = dy_dtype == MAGMA_DTYPE_F32, f_x = x_dtype == MAGMA_DTYPE_F32,
             f_dx = dx_dtype == MAGMA_DTYPE_F32;
#define LN_BWD(TDY, TX, TDX)                                                                    \
  return launch_bwd<TDY, TX, TDX>(dy, x, gamma, mean, rstd, dx, dgamma, dbeta, rows, d,      \
                                  accumulate_dx, accumulate_params, part, s)
  if (f_dy && f_x && f_dx) LN_BWD(float, float, float);
  if (!f_dy && f_x && f_dx) LN_BWD(__nv_bfloat16, float, float);
  if (!f_dy && !f_x && !f_dx) LN_BWD(__nv_bfloat16, __nv_bfloat16, __nv_bfloat16);
  if (!f_dy && !f_x && f_dx) LN_BWD(__nv_bfloat16, __nv_bfloat16, float);
  if (f_dy && !f_x && f_dx) LN_BWD(float, __nv_bfloat16, float);
  if (f_dy && f_x && !f_dx) LN_BWD(float, float, __nv_bfloat16);
  if (!f_dy && f_x && !f_dx) LN_BWD(__nv_bfloat16, float, __nv_bfloat16);
  LN_BWD(float, __nv_bfloat16, __nv_bfloat16);
#undef LN_BWD
}

magma_status_t magma_layernorm_bwd_noalloc(const void* dy, const void* x, const float* gamma,
                                           const float* mean, const float* rstd, void* dx,
                                           float* dgamma, float* dbeta, int64_t rows, int64_t dim,
                                           magma_dtype_t dy_dtype, magma_dtype_t x_dtype,
                                           magma_dtype_t dx_dtype, int32_t accumulate_dx,
                                           int32_t accumulate_params, void* stream) {
  MAGMA_REQUIRE(rows >= 0 && dim > 0, "magma_layernorm_bwd_noalloc: bad shape rows=%lld dim=%lld",
                (long long)rows, (long long)dim);
  MAGMA_REQUIRE(dim <= kNoAllocMaxDim,
                "magma_layernorm_bwd_noalloc: dim %lld exceeds the built-in scratch limit of %d "
                "(use magma_layernorm_bwd with a workspace)",
                (long long)dim, kNoAllocMaxDim);
  MAGMA_REQUIRE(is_float_dtype(dy_dtype) && is_float_dtype(x_dtype) && is_float_dtype(dx_dtype),
                "magma_layernorm_bwd_noalloc: unsupported dtypes");
  MAGMA_REQUIRE(!accumulate_dx || dx_dtype == MAGMA_DTYPE_F32,
                "magma_layernorm_bwd_noalloc: accumulate_dx needs an F32 dx");
  if (rows == 0) return MAGMA_OK;
  MAGMA_REQUIRE(dy && x && gamma && mean && rstd && dx,
                "magma_layernorm_bwd_noalloc: NULL pointer");
  float* part = nullptr;
  if (magma_status_t st = noalloc_scratch(&part)) return st;
  cudaStream_t s = (cudaStream_t)stream;
  const int d = (int)dim;
  const bool f_dy = dy_dtype == MAGMA_DTYPE_F32, f_x = x_dtype == MAGMA_DTYPE_F32,
             f_dx = dx_dtype == MAGMA_DTYPE_F32;
#define LN_BWD_NA(TDY, TX, TDX)                                                                 \
  return launch_bwd_noalloc<TDY, TX, TDX>(dy, x, gamma, mean, rstd, dx, dgamma, dbeta, rows, d, \
                                          accumulate_dx, accumulate_params, part, s)
  if (f_dy && f_x && f_dx) LN_BWD_NA(float, float, float);
  if (!f_dy && f_x && f_dx) LN_BWD_NA(__nv_bfloat16, float, float);
  if (!f_dy && !f_x && !f_dx) LN_BWD_NA(__nv_bfloat16, __nv_bfloat16, __nv_bfloat16);
  if (!f_dy && !f_x && f_dx) LN_BWD_NA(__nv_bfloat16, __nv_bfloat16, float);
  if (f_dy && !f_x && f_dx) LN_BWD_NA(float, __nv_bfloat16, float);
  if (f_dy && f_x && !f_dx) LN_BWD_NA(float, float, __nv_bfloat16);
  if (!f_dy && f_x && !f_dx) LN_BWD_NA(__nv_bfloat16, float, __nv_bfloat16);
  LN_BWD_NA(float, __nv_bfloat16, __nv_bfloat16);
#undef LN_BWD_NA
}

size_t magma_layernorm_bwd_residual_workspace_size(int64_t rows, int64_t dim) {
  if (rows <= 0 || dim <= 0) return 0;
  int64_t b = ceil_div(rows, kWarps);
  if (b > kMaxBwdBlocks) b = kMaxBwdBlocks;
  return (size_t)b * 3 * (size_t)dim * sizeof(float);
}

magma_status_t magma_layernorm_bwd_residual(const void* dy, const float* x, const float* gamma,
                                            const float* mean, const float* rstd, float* dx,
                                            void* dx_bf16, float* dgamma, float* dbeta,
                                            float* dcol, int64_t rows, int64_t dim,
                                            magma_dtype_t dy_dtype, int32_t accumulate_dx,
                                            int32_t accumulate_params, void* workspace,
                                            size_t workspace_bytes, void* stream) {
  MAGMA_REQUIRE(rows >= 0 && dim > 0 && dim % 8 == 0 && dim <= kMaxGroups * 128,
                "magma_layernorm_bwd_residual: dim %lld must be a multiple of 8 and <= %d",
                (long long)dim, kMaxGroups * 128);
  MAGMA_REQUIRE(is_float_dtype(dy_dtype), "magma_layernorm_bwd_residual: unsupported dy dtype");
  if (rows == 0) return MAGMA_OK;
  MAGMA_REQUIRE(dy && x && gamma && mean && rstd && dx,
                "magma_layernorm_bwd_residual: NULL pointer");
  MAGMA_REQUIRE(aligned16(dy) && aligned16(x) && aligned16(gamma) && aligned16(dx) &&
                    aligned16(dx_bf16),
                "magma_layernorm_bwd_residual: dy, x, gamma, dx, dx_bf16 must be 16-byte aligned");
  const size_t need = magma_layernorm_bwd_residual_workspace_size(rows, dim);
  MAGMA_REQUIRE(workspace != nullptr && workspace_bytes >= need,
                "magma_layernorm_bwd_residual: workspace of %zu bytes needed, %zu given", need,
                workspace_bytes);
  cudaStream_t s = (cudaStream_t)stream;
  float* part = (float*)workspace;
  const int d = (int)dim;
  int blocks = bwd_blocks(rows);
  bool launched = false;
  magma_status_t st =
      dy_dtype == MAGMA_DTYPE_F32
          ? launch_bwd_stream<float, float, float, true>(dy, x, gamma, mean, rstd, dx, rows, d,
                                                         accumulate_dx, part, kMaxBwdBlocks,
                                                         &blocks, &launched, s, dx_bf16)
          : launch_bwd_stream<__nv_bfloat16, float, float, true>(
                dy, x, gamma, mean, rstd, dx, rows, d, accumulate_dx, part, kMaxBwdBlocks,
                &blocks, &launched, s, dx_bf16);
  if (st) return st;
  MAGMA_REQUIRE(launched, "magma_layernorm_bwd_residual: shape not supported by the row kernels");
  if (dgamma != nullptr || dbeta != nullptr || dcol != nullptr) {
    const int width = 3 * d;
    launch_reduce_partials(part, blocks, width, dgamma, dbeta, dcol, d, accumulate_params, s);
    if (magma_status_t s2 = check_launch("layernorm_bwd_residual_reduce")) return s2;
  }
  return MAGMA_OK;
}

}  // extern "C"
