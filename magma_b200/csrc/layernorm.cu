// LayerNorm forward and backward.
//
// Forward restates nn.LayerNorm.forward (Sources/Core/Module.swift:2754-2791)
// and the GPT block's layerNorm (Benchmarks/GPT2Shakespeare/Sources/main.swift:
// 364-375): mean = sum/D, var = sum((x-mean)^2)/D (population), std =
// sqrt(var+eps), y = ((x-mean)/std)*gamma + beta, with an IEEE divide by std
// as the reference does (it never multiplies by rsqrt).
//
// Backward is the closed form of the reference's autodiff chain through that
// forward (vjpDivide/vjpSqrt/vjpMeanDims/vjpMultiply with sumAlongBroadcastDims,
// Sources/Core/Autodiff.swift:57-94,221-257,351-370; Optimizer.swift:627-633).
//
// Both kernels are HBM-bound row kernels: a warp owns whole rows (two at a
// time, their loads issued before any arithmetic), 8 elements per lane per
// step via 128-bit loads (BF16) or 2x128-bit loads (F32), rows held in
// registers between the reduction and the store, warp-shuffle reductions in a
// fixed butterfly order (deterministic). dgamma/dbeta are accumulated per warp
// in shared memory, summed over the CTA's warps in warp order into per-CTA
// partial rows in the caller's workspace, then over CTAs in CTA order by a
// second kernel.
#include <mutex>

#include "common.cuh"

namespace magma {
namespace {

constexpr int kWarps = 8;            // warps per CTA (one row per warp at a time)
constexpr int kMaxChunks = 4;        // cached 8-element chunks per lane: D <= 1024
constexpr int kMaxBwdBlocks = 592;   // cap on per-CTA partial rows (4 x 148 SMs)

// D = 8*32*CPL' (CPL' <= CPL chunks per lane), RPW rows per warp: the loads of
// all RPW rows are issued before any reduction so each warp keeps
// RPW x 8 x CPL elements in flight (memory-level parallelism for an
// HBM-bound kernel with one wave of warps).
template <int CPL, int RPW, typename TX, typename TY>
__global__ void __launch_bounds__(kWarps * 32)
ln_fwd_rows(const TX* __restrict__ x, const float* __restrict__ gamma,
            const float* __restrict__ beta, TY* __restrict__ y, float* __restrict__ mean_out,
            float* __restrict__ rstd_out, int64_t rows, int dim, float eps) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int chunks = dim >> 3;
  for (int64_t r0 = ((int64_t)blockIdx.x * kWarps + warp) * RPW; r0 < rows;
       r0 += (int64_t)gridDim.x * kWarps * RPW) {
    float v[RPW][CPL][8];
#pragma unroll
    for (int q = 0; q < RPW; ++q) {
      const int64_t row = r0 + q;
#pragma unroll
      for (int c = 0; c < CPL; ++c) {
        const int chunk = lane + c * 32;
        if (row < rows && chunk < chunks) load8(x + row * dim + chunk * 8, v[q][c]);
      }
    }
#pragma unroll
    for (int q = 0; q < RPW; ++q) {
      const int64_t row = r0 + q;
      if (row >= rows) break;
      float s = 0.f;
#pragma unroll
      for (int c = 0; c < CPL; ++c)
        if (lane + c * 32 < chunks)
#pragma unroll
          for (int i = 0; i < 8; ++i) s += v[q][c][i];
      s = warp_sum(s);
      const float mean = __fdiv_rn(s, (float)dim);
      float ss = 0.f;
#pragma unroll
      for (int c = 0; c < CPL; ++c)
        if (lane + c * 32 < chunks)
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float d = __fsub_rn(v[q][c][i], mean);
            v[q][c][i] = d;
            ss += d * d;
          }
      ss = warp_sum(ss);
      const float stdv = __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)dim), eps));
      TY* yr = y + row * dim;
#pragma unroll
      for (int c = 0; c < CPL; ++c) {
        const int chunk = lane + c * 32;
        if (chunk < chunks) {
          float g[8], b[8], o[8];
          load8(gamma + chunk * 8, g);
          load8(beta + chunk * 8, b);
#pragma unroll
          for (int i = 0; i < 8; ++i)
            o[i] = __fadd_rn(__fmul_rn(__fdiv_rn(v[q][c][i], stdv), g[i]), b[i]);
          store8(yr + chunk * 8, o);
        }
      }
      if (lane == 0) {
        if (mean_out) mean_out[row] = mean;
        if (rstd_out) rstd_out[row] = __fdiv_rn(1.0f, stdv);
      }
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

// Backward, D % 8 == 0, D <= 256*CPL: RPW rows per warp with their loads
// issued up front; each warp accumulates its dgamma/dbeta partials in its own
// shared-memory row (no atomics), the 8 warp rows are then summed in warp
// order into the CTA's partial row part[blockIdx.x] = [dgamma | dbeta].
template <int CPL, int RPW, typename TDY, typename TX, typename TDX>
__global__ void __launch_bounds__(kWarps * 32, 2)
ln_bwd_rows(const TDY* __restrict__ dy, const TX* __restrict__ x,
            const float* __restrict__ gamma, const float* __restrict__ mean_in,
            const float* __restrict__ rstd_in, TDX* __restrict__ dx,
            float* __restrict__ part, int64_t rows, int dim, int accumulate_dx) {
  extern __shared__ float smem[];  // [kWarps][2*dim]
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int chunks = dim >> 3;
  float* wp = smem + (size_t)warp * 2 * dim;
  for (int i = lane; i < 2 * dim; i += 32) wp[i] = 0.f;
  __syncwarp();
  for (int64_t r0 = ((int64_t)blockIdx.x * kWarps + warp) * RPW; r0 < rows;
       r0 += (int64_t)gridDim.x * kWarps * RPW) {
    float xv[RPW][CPL][8], dv[RPW][CPL][8];
#pragma unroll
    for (int q = 0; q < RPW; ++q) {
      const int64_t row = r0 + q;
#pragma unroll
      for (int c = 0; c < CPL; ++c) {
        const int chunk = lane + c * 32;
        if (row < rows && chunk < chunks) {
          load8(x + row * dim + chunk * 8, xv[q][c]);
          load8(dy + row * dim + chunk * 8, dv[q][c]);
        }
      }
    }
#pragma unroll
    for (int q = 0; q < RPW; ++q) {
      const int64_t row = r0 + q;
      if (row >= rows) break;
      const float mean = mean_in[row];
      const float rstd = rstd_in[row];
      float s1 = 0.f, s2 = 0.f;
#pragma unroll
      for (int c = 0; c < CPL; ++c) {
        const int chunk = lane + c * 32;
        if (chunk < chunks) {
          float gm[8];
          load8(gamma + chunk * 8, gm);
          float* pg = wp + chunk * 8;
          float* pb = wp + dim + chunk * 8;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float xhat = (xv[q][c][i] - mean) * rstd;
            const float gg = dv[q][c][i] * gm[i];
            pg[i] += dv[q][c][i] * xhat;
            pb[i] += dv[q][c][i];
            xv[q][c][i] = xhat;
            dv[q][c][i] = gg;
            s1 += gg;
            s2 += gg * xhat;
          }
        }
      }
      s1 = warp_sum(s1) / (float)dim;
      s2 = warp_sum(s2) / (float)dim;
#pragma unroll
      for (int c = 0; c < CPL; ++c) {
        const int chunk = lane + c * 32;
        if (chunk < chunks) {
          float o[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) o[i] = rstd * (dv[q][c][i] - s1 - xv[q][c][i] * s2);
          TDX* dst = dx + row * dim + chunk * 8;
          if (accumulate_dx) {
            float prev[8];
            load8(dst, prev);
#pragma unroll
            for (int i = 0; i < 8; ++i) o[i] += prev[i];
          }
          store8(dst, o);
        }
      }
    }
  }
  __syncthreads();
  float* out = part + (int64_t)blockIdx.x * 2 * dim;
  for (int i = threadIdx.x; i < 2 * dim; i += blockDim.x) {
    float t = smem[i];
#pragma unroll
    for (int w = 1; w < kWarps; ++w) t += smem[(size_t)w * 2 * dim + i];
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

// Sums per-CTA partial rows: out[c] (+)= sum_b part[b][c]. A 32 x 8 CTA
// covers 32 columns; row y of threads sums partials b = y, y+8, ... in order,
// then the 8 sums are added in y order (fixed order: deterministic).
__global__ void __launch_bounds__(256)
reduce_partials(const float* __restrict__ part, int nblocks, int width,
                float* __restrict__ dgamma, float* __restrict__ dbeta, int dim, int accumulate) {
  __shared__ float red[8][33];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + tx;
  float s = 0.f;
  if (c < width) {
#pragma unroll 4
    for (int b = ty; b < nblocks; b += 8) s += part[(int64_t)b * width + c];
  }
  red[ty][tx] = s;
  __syncthreads();
  if (ty == 0 && c < width) {
    float t = red[0][tx];
#pragma unroll
    for (int y = 1; y < 8; ++y) t += red[y][tx];
    float* dst = c < dim ? dgamma + c : dbeta + (c - dim);
    if (dst == nullptr) return;
    *dst = accumulate ? *dst + t : t;
  }
}

int bwd_blocks(int64_t rows) {
  int64_t b = ceil_div(rows, kWarps);
  int64_t cap = 2LL * num_sms();
  if (cap > kMaxBwdBlocks) cap = kMaxBwdBlocks;
  if (b > cap) b = cap;
  if (b < 1) b = 1;
  return (int)b;
}

// Launches ln_bwd_rows; *blocks (in: upper bound on the CTA count the caller's
// partial buffer holds; out: CTAs launched = partial rows written).
template <typename TDY, typename TX, typename TDX>
magma_status_t launch_bwd_rows(const void* dy, const void* x, const float* gamma,
                               const float* mean, const float* rstd, void* dx, int64_t rows,
                               int dim, int acc_dx, float* part, int* blocks,
                               cudaStream_t stream) {
  int64_t b = ceil_div(rows, kWarps * 2);
  const int64_t cap = 2LL * num_sms();
  if (b > cap) b = cap;
  if (b > *blocks) b = *blocks;
  if (b < 1) b = 1;
  *blocks = (int)b;
  const size_t smem = (size_t)kWarps * 2 * dim * sizeof(float);
  const int cpl = (dim + 255) / 256;
#define LN_BWD_ROWS(C)                                                                         \
  do {                                                                                         \
    auto kern = ln_bwd_rows<C, (C <= 3 ? 2 : 1), TDY, TX, TDX>;                                \
    if (smem > 48 * 1024)                                                                      \
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);      \
    kern<<<(int)b, kWarps * 32, smem, stream>>>((const TDY*)dy, (const TX*)x, gamma, mean, rstd, \
                                                 (TDX*)dx, part, rows, dim, acc_dx);           \
  } while (0)
  if (cpl == 1) LN_BWD_ROWS(1);
  else if (cpl == 2) LN_BWD_ROWS(2);
  else if (cpl == 3) LN_BWD_ROWS(3);
  else LN_BWD_ROWS(4);
#undef LN_BWD_ROWS
  return check_launch("layernorm_bwd");
}

template <typename TX, typename TY>
magma_status_t launch_fwd(const void* x, const float* gamma, const float* beta, void* y,
                          float* mean, float* rstd, int64_t rows, int dim, float eps,
                          cudaStream_t stream) {
  int64_t blocks = ceil_div(rows, kWarps);
  int64_t cap = 16LL * num_sms();
  if (blocks > cap) blocks = cap;
  bool vec = (dim % 8 == 0) && dim <= kMaxChunks * 256 && aligned16(x) && aligned16(y) &&
             aligned16(gamma) && aligned16(beta);
  if (vec) {
    const int cpl = (dim + 255) / 256;
    int64_t b2 = ceil_div(rows, kWarps * 2);
    if (b2 > cap) b2 = cap;
    if (cpl == 1)
      ln_fwd_rows<1, 2, TX, TY><<<(int)b2, kWarps * 32, 0, stream>>>(
          (const TX*)x, gamma, beta, (TY*)y, mean, rstd, rows, dim, eps);
    else if (cpl == 2)
      ln_fwd_rows<2, 2, TX, TY><<<(int)b2, kWarps * 32, 0, stream>>>(
          (const TX*)x, gamma, beta, (TY*)y, mean, rstd, rows, dim, eps);
    else if (cpl == 3)
      ln_fwd_rows<3, 2, TX, TY><<<(int)b2, kWarps * 32, 0, stream>>>(
          (const TX*)x, gamma, beta, (TY*)y, mean, rstd, rows, dim, eps);
    else
      ln_fwd_rows<4, 2, TX, TY><<<(int)b2, kWarps * 32, 0, stream>>>(
          (const TX*)x, gamma, beta, (TY*)y, mean, rstd, rows, dim, eps);
  } else
    ln_fwd_generic<TX, TY><<<(int)blocks, kWarps * 32, 0, stream>>>(
        (const TX*)x, gamma, beta, (TY*)y, mean, rstd, rows, dim, eps);
  return check_launch("layernorm_fwd");
}

template <typename TDY, typename TX, typename TDX>
magma_status_t launch_bwd(const void* dy, const void* x, const float* gamma, const float* mean,
                          const float* rstd, void* dx, float* dgamma, float* dbeta,
                          int64_t rows, int dim, int acc_dx, int acc_params, float* part,
                          cudaStream_t stream) {
  int blocks = bwd_blocks(rows);
  bool vec = (dim % 8 == 0) && dim <= kMaxChunks * 256 && aligned16(x) && aligned16(dy) &&
             aligned16(dx) && aligned16(gamma);
  if (vec) {
    if (magma_status_t st = launch_bwd_rows<TDY, TX, TDX>(dy, x, gamma, mean, rstd, dx, rows, dim,
                                                          acc_dx, part, &blocks, stream))
      return st;
  } else {
    ln_bwd_generic<TDY, TX, TDX><<<blocks, kWarps * 32, 0, stream>>>(
        (const TDY*)dy, (const TX*)x, gamma, mean, rstd, (TDX*)dx, part, rows, dim, acc_dx);
  }
  if (magma_status_t s = check_launch("layernorm_bwd")) return s;
  if (dgamma != nullptr || dbeta != nullptr) {
    int width = 2 * dim;
    reduce_partials<<<(width + 31) / 32, 256, 0, stream>>>(part, blocks, width, dgamma, dbeta,
                                                           dim, acc_params);
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
  const bool vec = (dim % 8 == 0) && dim <= kMaxChunks * 256 && aligned16(x) && aligned16(dy) &&
                   aligned16(dx) && aligned16(gamma);
  if (vec) {
    if (magma_status_t st = launch_bwd_rows<TDY, TX, TDX>(dy, x, gamma, mean, rstd, dx, rows, dim,
                                                          acc_dx, part, &blocks, stream))
      return st;
  } else {
    ln_bwd_generic<TDY, TX, TDX><<<blocks, kWarps * 32, 0, stream>>>(
        (const TDY*)dy, (const TX*)x, gamma, mean, rstd, (TDX*)dx, part, rows, dim, acc_dx);
  }
  if (magma_status_t s = check_launch("layernorm_bwd_noalloc")) return s;
  if (dgamma != nullptr || dbeta != nullptr) {
    const int width = 2 * dim;
    reduce_partials<<<(width + 31) / 32, 256, 0, stream>>>(part, blocks, width, dgamma, dbeta,
                                                           dim, acc_params);
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

}  // extern "C"
