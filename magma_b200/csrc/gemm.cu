// The Linear contraction: c = opA(a) . opB(b) with a fused epilogue.
//
// Replaces Tensor.matmul -> stablehlo.dot (Sources/Core/Tensor.swift:1102-1121,
// Sources/StableHLO/Builder/MLIRBuilder.swift:372-378) as emitted by the value
// Linear (ValueLayers.swift:38-41), nn.Linear (Module.swift:266-300), the GPT
// linear (main.swift:353-362) and the matmul VJP (Autodiff.swift:177-191). The
// transposes that the reference materialises in the graph become operand
// majorness here (no transpose kernels), and the bias add / activation /
// residual add / activation VJP that follow the dot are fused into the store.
//
// BF16 path: a persistent, warp-specialised tcgen05 kernel (320 threads).
//   warp 0      TMA producer: A and B tiles of 64 K-elements, 128-byte swizzle,
//               into an up-to-8-stage shared-memory ring (full/empty mbarriers);
//   warp 1      TMEM allocator and MMA issuer: one thread issues
//               tcgen05.mma.kind::f16 (K = 16) into one of two TMEM
//               accumulators and commits, so the next tile's MMAs overlap the
//               epilogue of this one;
//   warps 2..9  epilogue: tcgen05.ld of the accumulator (thread = row), fused
//               epilogue math; plain, bias and row-statistics outputs and
//               split-K partials leave through swizzled 32x32 shared-memory
//               boxes and TMA stores; the auxiliary epilogues (GELU, residual,
//               activation VJPs) go through a padded staging area with
//               16-byte row-segment accesses.
// Tile options, chosen per shape by a cost model fitted to measured times: one
// CTA with a 128x128 or 128x256 tile, or a CTA pair (cta_group::2, M = 256,
// each CTA loading half of A and half of B) with 256x128 or 256x256, plus
// K-split work units summed in a fixed order by a reduce kernel.
// Operands may be K-major or MN-major (instruction-descriptor bits 15/16),
// which covers x.W^T (forward), dY.W (input gradient) and X^T.dY (weight
// gradient) without copies.
//
// F32 path: contractions of at least 2^27 multiply-adds run on the same
// tensor-core kernel through a three-term BF16 split of both operands (six
// BF16 products per F32 product, F32 accumulation; a single TF32 or BF16
// product would miss a 1e-4 relative tolerance). Smaller ones, calls without
// the split's workspace and the row-statistics epilogue use a register-blocked
// FFMA kernel (128x128 tile, 8x8 per thread), as do shapes TMA cannot describe.
#include <cuda.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <type_traits>

#include "common.cuh"
#include "sm100.cuh"

namespace magma {
namespace {

struct EpiArgs {
  int epi;
  const float* bias;
  const void* aux_in;
  void* aux_out;
  int64_t ldc;
};

template <typename TC>
__device__ __forceinline__ float epi_value(const EpiArgs& e, const TC* C, int64_t off, int64_t col,
                                           float acc) {
  switch (e.epi) {
    case MAGMA_EPI_NONE:
      return acc;
    case MAGMA_EPI_BIAS:
      return e.bias ? __fadd_rn(acc, e.bias[col]) : acc;
    case MAGMA_EPI_BIAS_GELU: {
      float pre = e.bias ? __fadd_rn(acc, e.bias[col]) : acc;
      static_cast<TC*>(e.aux_out)[off] = from_f32<TC>(pre);
      return gelu_t<TC>(pre);
    }
    case MAGMA_EPI_BIAS_RESIDUAL: {
      float t = e.bias ? __fadd_rn(acc, e.bias[col]) : acc;
      return __fadd_rn(static_cast<const float*>(e.aux_in)[off], t);
    }
    case MAGMA_EPI_DGELU:
      return __fmul_rn(acc, gelu_grad_t<TC>(to_f32(static_cast<const TC*>(e.aux_in)[off])));
    case MAGMA_EPI_ACCUMULATE:
      return __fadd_rn(to_f32(C[off]), acc);
    case MAGMA_EPI_BIAS_RELU: {
      float pre = e.bias ? __fadd_rn(acc, e.bias[col]) : acc;
      static_cast<TC*>(e.aux_out)[off] = from_f32<TC>(pre);
      return fmaxf(pre, 0.f);
    }
    case MAGMA_EPI_DRELU:
      return to_f32(static_cast<const TC*>(e.aux_in)[off]) > 0.f ? acc : 0.f;
    default:
      return acc;
  }
}

// ============================== F32 FFMA kernel ==============================
constexpr int kSimtBM = 128, kSimtBN = 128, kSimtBK = 8;

// K-split form (ws != nullptr): block z computes the K range [z*kps, (z+1)*kps)
// and stores its raw F32 sums to plane z of ws ([splits][M][N]); the planes
// are added in split order by splitk_reduce, which applies the epilogue.
template <typename TA, typename TC, bool TA_T, bool TB_T>
__global__ void __launch_bounds__(256)
gemm_simt_kernel(const TA* __restrict__ A, const TA* __restrict__ B, TC* __restrict__ C,
                 int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb, EpiArgs e,
                 int64_t kps, float* __restrict__ ws) {
  __shared__ float As[2][kSimtBK][kSimtBM + 4];
  __shared__ float Bs[2][kSimtBK][kSimtBN + 4];
  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const int64_t m0 = (int64_t)blockIdx.y * kSimtBM, n0 = (int64_t)blockIdx.x * kSimtBN;
  const int64_t kbeg = (int64_t)blockIdx.z * kps;
  const int64_t kend = kbeg + kps < K ? kbeg + kps : K;
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
  float ra[4], rb[4];
  auto load_tiles = [&](int64_t k0) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      int idx = tid + i * 256;
      int mm, kk;
      if (!TA_T) { mm = idx >> 3; kk = idx & 7; } else { kk = idx >> 7; mm = idx & 127; }
      int64_t gm = m0 + mm, gk = k0 + kk;
      ra[i] = (gm < M && gk < kend) ? to_f32(TA_T ? A[gk * lda + gm] : A[gm * lda + gk]) : 0.f;
      int nn;
      if (!TB_T) { kk = idx >> 7; nn = idx & 127; } else { nn = idx >> 3; kk = idx & 7; }
      int64_t gn = n0 + nn;
      gk = k0 + kk;
      rb[i] = (gn < N && gk < kend) ? to_f32(TB_T ? B[gn * ldb + gk] : B[gk * ldb + gn]) : 0.f;
    }
  };
  auto store_tiles = [&](int buf) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      int idx = tid + i * 256;
      int mm, kk;
      if (!TA_T) { mm = idx >> 3; kk = idx & 7; } else { kk = idx >> 7; mm = idx & 127; }
      As[buf][kk][mm] = ra[i];
      int nn;
      if (!TB_T) { kk = idx >> 7; nn = idx & 127; } else { nn = idx >> 3; kk = idx & 7; }
      Bs[buf][kk][nn] = rb[i];
    }
  };
  const int64_t ktiles = kend > kbeg ? (kend - kbeg + kSimtBK - 1) / kSimtBK : 0;
  if (ktiles > 0) {
    load_tiles(kbeg);
    store_tiles(0);
  }
  __syncthreads();
  for (int64_t kt = 0; kt < ktiles; ++kt) {
    const int buf = kt & 1;
    if (kt + 1 < ktiles) load_tiles(kbeg + (kt + 1) * kSimtBK);
#pragma unroll
    for (int k = 0; k < kSimtBK; ++k) {
      float a[8], b[8];
      float4 a0 = *reinterpret_cast<const float4*>(&As[buf][k][ty * 4]);
      float4 a1 = *reinterpret_cast<const float4*>(&As[buf][k][64 + ty * 4]);
      float4 b0 = *reinterpret_cast<const float4*>(&Bs[buf][k][tx * 4]);
      float4 b1 = *reinterpret_cast<const float4*>(&Bs[buf][k][64 + tx * 4]);
      a[0] = a0.x; a[1] = a0.y; a[2] = a0.z; a[3] = a0.w;
      a[4] = a1.x; a[5] = a1.y; a[6] = a1.z; a[7] = a1.w;
      b[0] = b0.x; b[1] = b0.y; b[2] = b0.z; b[3] = b0.w;
      b[4] = b1.x; b[5] = b1.y; b[6] = b1.z; b[7] = b1.w;
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    if (kt + 1 < ktiles) store_tiles(buf ^ 1);
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    int64_t row = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
    if (row >= M) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      int64_t col = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + (j - 4));
      if (col >= N) continue;
      if (ws != nullptr) {
        ws[((int64_t)blockIdx.z * M + row) * N + col] = acc[i][j];
        continue;
      }
      int64_t off = row * e.ldc + col;
      C[off] = from_f32<TC>(epi_value<TC>(e, C, off, col, acc[i][j]));
    }
  }
}

// ============================ tcgen05 BF16 kernel ============================
constexpr int kBM = 128, kBK = 64;
// warp 0 TMA producer, warp 1 MMA issuer, warps 2..9 epilogue (two warps per
// TMEM lane quarter, each owning half of the tile's columns)
constexpr int kEpiWarps = 8;
constexpr int kGemmThreads = 32 * (2 + kEpiWarps);

// BN = N extent of one MMA tile. PAIR: a cluster of two CTAs issues one
// M=256 MMA (cta_group::2); each CTA holds 128 rows of A, BN/2 rows of B and a
// 128 x BN accumulator in its own TMEM.
template <int BN, bool PAIR>
struct TcCfg {
  static constexpr int kBRows = PAIR ? BN / 2 : BN;
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = kBRows * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  // Epilogue staging, 8 KB per epilogue warp: either a 32 x 32 F32 chunk of
  // accumulators with row pitch 36 floats (16-byte rows, conflict-free float4
  // access), or the swizzled TMA-store buffers of the direct epilogue (four
  // 32 x 32 BF16 boxes or two 32 x 32 F32 boxes).
  static constexpr int kStagePitch = 36;
  static constexpr int kStageWarpFloats = 2048;
  static constexpr int kStagingBytes = kEpiWarps * kStageWarpFloats * 4;
  static constexpr int kSmemLimit = 232448;  // sm_100 dynamic shared memory per block
  static constexpr int kReserve = kStagingBytes + 1024 + 256;  // staging, alignment, barriers
  static constexpr int kStagesFit = (kSmemLimit - kReserve) / kStageBytes;
  static constexpr int kStages = kStagesFit > 8 ? 8 : kStagesFit;
  static constexpr int kStageOffset = kStages * kStageBytes;
  static constexpr int kBarOffset = kStageOffset + kStagingBytes;
  // full[S], empty[S], tfull[2], tempty[2], done -> 8 B each; then TMEM slot.
  static constexpr int kBarBytes = (2 * kStages + 5) * 8 + 16;
  static constexpr int kSmemBytes = kBarOffset + kBarBytes + 1024;  // + alignment slack
  static_assert(kStages >= 3, "GEMM pipeline too shallow");
  static_assert(kSmemBytes <= kSmemLimit, "GEMM shared memory exceeds the sm_100 per-block limit");
  static constexpr int kTmemCols = 2 * BN;
};

struct TcArgs {
  int64_t M, N, K;
  void* C;
  EpiArgs e;
  int* err;
  int vec_ok;   // C/aux pointers 8-B aligned and ldc even: column-pair vector accesses
  int vec8_ok;  // C 16-B aligned and ldc % 8 == 0: 8-column vector stores
  int epi_vec8; // vec8_ok with 16-B aligned aux and bias: 8-column staged epilogue
  int tma_out;  // direct epilogue stores through the tensor map tmC (C, or the split partials)
  // Split-K: work unit u covers output tile (u % tiles) over k-blocks
  // [s*kb_per_split, (s+1)*kb_per_split) with s = u / tiles. With splits > 1
  // the raw F32 accumulator goes to ws + s*M*N (leading dimension N) and a
  // second kernel applies the epilogue to the sum over s.
  int splits;
  int kb_per_split;
  float* ws;
  // Tile raster: 0 walks M fastest (concurrent CTAs share a B tile), 1 walks
  // N fastest (they share an A block: used when A is far larger than L2 and
  // would otherwise be re-read once per N tile).
  int n_fast;
};

// Epilogue on two consecutive columns (col, col+1) of one row; b0/b1 are the
// columns' bias values (0 without bias). pair: both columns exist and the
// pointers allow one 2-element access.
template <typename TC>
__device__ __forceinline__ void epi_store2(const TcArgs& a, int64_t row, int64_t col, float v0,
                                           float v1, float b0, float b1, bool pair) {
  TC* C = static_cast<TC*>(a.C);
  const int64_t off = row * a.e.ldc + col;
  const int epi = a.e.epi;
  if (!pair) {
    C[off] = from_f32<TC>(epi_value<TC>(a.e, C, off, col, v0));
    if (col + 1 < a.N) C[off + 1] = from_f32<TC>(epi_value<TC>(a.e, C, off + 1, col + 1, v1));
    return;
  }
  float o0, o1;
  if (epi == MAGMA_EPI_NONE) {
    o0 = v0;
    o1 = v1;
  } else if (epi == MAGMA_EPI_BIAS) {
    o0 = __fadd_rn(v0, b0);
    o1 = __fadd_rn(v1, b1);
  } else if (epi == MAGMA_EPI_BIAS_RESIDUAL) {
    const float2 r = *reinterpret_cast<const float2*>(static_cast<const float*>(a.e.aux_in) + off);
    o0 = __fadd_rn(r.x, __fadd_rn(v0, b0));
    o1 = __fadd_rn(r.y, __fadd_rn(v1, b1));
  } else if (epi == MAGMA_EPI_BIAS_GELU || epi == MAGMA_EPI_BIAS_RELU) {
    const float p0 = __fadd_rn(v0, b0), p1 = __fadd_rn(v1, b1);
    store2(static_cast<TC*>(a.e.aux_out) + off, p0, p1);
    if (epi == MAGMA_EPI_BIAS_GELU) {
      o0 = gelu_t<TC>(p0);
      o1 = gelu_t<TC>(p1);
    } else {
      o0 = fmaxf(p0, 0.f);
      o1 = fmaxf(p1, 0.f);
    }
  } else if (epi == MAGMA_EPI_DGELU || epi == MAGMA_EPI_DRELU) {
    float x0, x1;
    load2(static_cast<const TC*>(a.e.aux_in) + off, x0, x1);
    if (epi == MAGMA_EPI_DGELU) {
      o0 = __fmul_rn(v0, gelu_grad_t<TC>(x0));
      o1 = __fmul_rn(v1, gelu_grad_t<TC>(x1));
    } else {
      o0 = x0 > 0.f ? v0 : 0.f;
      o1 = x1 > 0.f ? v1 : 0.f;
    }
  } else {  // ACCUMULATE (F32 output)
    float c0, c1;
    load2(C + off, c0, c1);
    o0 = __fadd_rn(c0, v0);
    o1 = __fadd_rn(c1, v1);
  }
  store2(C + off, o0, o1);
}

// Row-per-thread store of 64 accumulator columns (NONE / BIAS epilogues and
// split-K partials): 16-byte stores, one row per thread — the fewest
// instructions when nothing has to be read back from global memory.
template <typename TO>
__device__ __forceinline__ void direct_store64(TO* dst_row, const float* bias, int64_t col0,
                                               int64_t N, const uint32_t (&ra)[32],
                                               const uint32_t (&rb)[32], bool vec8) {
#pragma unroll
  for (int g = 0; g < 8; ++g) {
    const int64_t col = col0 + 8 * g;
    if (col >= N) break;
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
      v[i] = __uint_as_float(g < 4 ? ra[8 * g + i] : rb[8 * (g - 4) + i]);
    if (bias != nullptr) {
      if (vec8 && col + 8 <= N && (reinterpret_cast<uintptr_t>(bias + col) & 15u) == 0) {
        float bv[8];
        load8(bias + col, bv);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = __fadd_rn(v[i], bv[i]);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i)
          if (col + i < N) v[i] = __fadd_rn(v[i], bias[col + i]);
      }
    }
    if (vec8 && col + 8 <= N) {
      store8(dst_row + col, v);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (col + i < N) dst_row[col + i] = from_f32<TO>(v[i]);
    }
  }
}

// Softmax partials of one row over 64 consecutive columns (ra: the first 32,
// rb: the next 32) of c as stored (rounded to TO): (max, sum of exp(c - max))
// over the columns below N, into *out.
template <typename TO>
__device__ __forceinline__ void row_stats64(const uint32_t (&ra)[32], const uint32_t (&rb)[32],
                                            int64_t col0, int64_t N, float2* out) {
  constexpr float kLog2e = 1.4426950408889634f;
  const int valid = (int)(N - col0 < 64 ? N - col0 : 64);
  auto val = [&](int j) {
    return to_f32(from_f32<TO>(__uint_as_float(j < 32 ? ra[j] : rb[j - 32])));
  };
  float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
  float s4[4] = {0.f, 0.f, 0.f, 0.f};
  if (valid == 64) {
#pragma unroll
    for (int j = 0; j < 64; ++j) m4[j & 3] = fmaxf(m4[j & 3], val(j));
  } else {
#pragma unroll
    for (int j = 0; j < 64; ++j)
      if (j < valid) m4[j & 3] = fmaxf(m4[j & 3], val(j));
  }
  const float m = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
  const float ml = m * kLog2e;
  if (valid == 64) {
#pragma unroll
    for (int j = 0; j < 64; ++j) s4[j & 3] += sm100::ex2_approx(fmaf(val(j), kLog2e, -ml));
  } else {
#pragma unroll
    for (int j = 0; j < 64; ++j)
      if (j < valid) s4[j & 3] += sm100::ex2_approx(fmaf(val(j), kLog2e, -ml));
  }
  *out = make_float2(m, (s4[0] + s4[1]) + (s4[2] + s4[3]));
}

// BF16 output with softmax partials: packs the 64 values once, stores the
// pairs (16-byte stores when vec8 and the chunk is whole) and takes the
// partials from the stored BF16 values, unpacked with integer shifts (the
// conversion unit is shared with the exponentials).
__device__ __forceinline__ void direct_store64_stats(__nv_bfloat16* dst_row, int64_t col0,
                                                     int64_t N, const uint32_t (&ra)[32],
                                                     const uint32_t (&rb)[32], bool vec8,
                                                     float2* out) {
  constexpr float kLog2e = 1.4426950408889634f;
  const int valid = (int)(N - col0 < 64 ? N - col0 : 64);
  uint32_t pk[32];
#pragma unroll
  for (int p = 0; p < 32; ++p) {
    const int j = 2 * p;
    const __nv_bfloat162 h = __floats2bfloat162_rn(
        __uint_as_float(j < 32 ? ra[j] : rb[j - 32]),
        __uint_as_float(j + 1 < 32 ? ra[j + 1] : rb[j + 1 - 32]));
    pk[p] = *reinterpret_cast<const uint32_t*>(&h);
  }
  if (vec8 && valid == 64) {
#pragma unroll
    for (int g = 0; g < 8; ++g)
      *reinterpret_cast<uint4*>(dst_row + col0 + 8 * g) =
          make_uint4(pk[4 * g], pk[4 * g + 1], pk[4 * g + 2], pk[4 * g + 3]);
  } else {
#pragma unroll
    for (int j = 0; j < 64; ++j)
      if (j < valid)
        dst_row[col0 + j] = __ushort_as_bfloat16((unsigned short)(j & 1 ? pk[j >> 1] >> 16
                                                                       : pk[j >> 1] & 0xFFFFu));
  }
  auto val = [&](int j) {
    return __uint_as_float(j & 1 ? pk[j >> 1] & 0xFFFF0000u : pk[j >> 1] << 16);
  };
  float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
  float s4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int j = 0; j < 64; ++j)
    if (j < valid) m4[j & 3] = fmaxf(m4[j & 3], val(j));
  const float m = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
  const float ml = m * kLog2e;
#pragma unroll
  for (int j = 0; j < 64; ++j)
    if (j < valid) s4[j & 3] += sm100::ex2_approx(fmaf(val(j), kLog2e, -ml));
  *out = make_float2(m, (s4[0] + s4[1]) + (s4[2] + s4[3]));
}

// Direct epilogue through TMA stores. A warp's 64-column block of its 32 tile
// rows is written row = lane into swizzled shared-memory boxes of 32 rows x 32
// columns, which lane 0 then stores with TMA: every global write is a whole
// 64- or 128-byte row segment and the stores leave the warp's issue slots. The
// warp's 8 KB hold two BF16 blocks (a block is rewritten once the store of the
// block before the previous one has read it) or one F32 block.
//
// BF16: pk holds the 64 values as packed pairs; boxes have 64-byte rows with
// the 64-byte swizzle (16-byte unit u of row r at unit u ^ ((r >> 1) & 3)).
__device__ __forceinline__ void tma_block64_bf16(uint8_t* wbuf, int it, const uint32_t (&pk)[32],
                                                 const CUtensorMap* map, int x, int y, int64_t N,
                                                 int lane) {
  constexpr int kBox = 32 * 64;
  uint8_t* blk = wbuf + (it & 1) * 2 * kBox;
  if (lane == 0) sm100::bulk_wait_group_read<1>();
  __syncwarp();
  const int sw = (lane >> 1) & 3;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    uint8_t* row = blk + h * kBox + lane * 64;
#pragma unroll
    for (int u = 0; u < 4; ++u)
      *reinterpret_cast<uint4*>(row + ((u ^ sw) << 4)) =
          make_uint4(pk[16 * h + 4 * u], pk[16 * h + 4 * u + 1], pk[16 * h + 4 * u + 2],
                     pk[16 * h + 4 * u + 3]);
  }
  sm100::fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
#pragma unroll
    for (int h = 0; h < 2; ++h)
      if (x + 32 * h < N) sm100::tma_store_2d(map, sm100::smem_u32(blk + h * kBox), x + 32 * h, y);
    sm100::bulk_commit_group();
  }
}

// F32 (outputs and split-K partials): boxes have 128-byte rows with the
// 128-byte swizzle (16-byte unit u of row r at unit u ^ (r & 7)); z >= 0
// selects the 3-D partial map (x, y, split).
__device__ __forceinline__ void tma_block64_f32(uint8_t* wbuf, const uint32_t (&ra)[32],
                                                const uint32_t (&rb)[32], const CUtensorMap* map,
                                                int x, int y, int z, int64_t N, int lane) {
  constexpr int kBox = 32 * 128;
  if (lane == 0) sm100::bulk_wait_group_read<0>();
  __syncwarp();
  const int sw = lane & 7;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const uint32_t(&r)[32] = h ? rb : ra;
    uint8_t* row = wbuf + h * kBox + lane * 128;
#pragma unroll
    for (int u = 0; u < 8; ++u)
      *reinterpret_cast<uint4*>(row + ((u ^ sw) << 4)) =
          make_uint4(r[4 * u], r[4 * u + 1], r[4 * u + 2], r[4 * u + 3]);
  }
  sm100::fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      if (x + 32 * h >= N) continue;
      const uint32_t src = sm100::smem_u32(wbuf + h * kBox);
      if (z >= 0) sm100::tma_store_3d(map, src, x + 32 * h, y, z);
      else sm100::tma_store_2d(map, src, x + 32 * h, y);
    }
    sm100::bulk_commit_group();
  }
}

// Softmax partials of one row over 64 columns from BF16 pairs packed as in
// tma_block64_bf16 (same arithmetic as direct_store64_stats).
__device__ __forceinline__ void stats64_packed(const uint32_t (&pk)[32], int64_t col0, int64_t N,
                                               float2* out) {
  constexpr float kLog2e = 1.4426950408889634f;
  const int valid = (int)(N - col0 < 64 ? N - col0 : 64);
  auto val = [&](int j) {
    return __uint_as_float(j & 1 ? pk[j >> 1] & 0xFFFF0000u : pk[j >> 1] << 16);
  };
  float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
  float s4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int j = 0; j < 64; ++j)
    if (j < valid) m4[j & 3] = fmaxf(m4[j & 3], val(j));
  const float m = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
  const float ml = m * kLog2e;
#pragma unroll
  for (int j = 0; j < 64; ++j)
    if (j < valid) s4[j & 3] += sm100::ex2_approx(fmaf(val(j), kLog2e, -ml));
  *out = make_float2(m, (s4[0] + s4[1]) + (s4[2] + s4[3]));
}

// One 32-column chunk of one warp's 32 tile rows: this lane handles the
// column pair (col, col+1) of rows rsel, rsel+2, ..., st points at that pair
// in row rsel of the staged F32 accumulators (row pitch P). The epilogue is a
// template parameter (no per-row branches) and every auxiliary load is issued
// before the first store so their latencies overlap.
template <typename TC, int EPI, int P>
__device__ __forceinline__ void epi_rows(const TcArgs& a, const float* __restrict__ st,
                                         int64_t row0, int rows_here, int rsel, int64_t col,
                                         float b0, float b1) {
  constexpr bool kAux = EPI == MAGMA_EPI_BIAS_RESIDUAL || EPI == MAGMA_EPI_DGELU ||
                        EPI == MAGMA_EPI_DRELU || EPI == MAGMA_EPI_ACCUMULATE;
  const int64_t ldc = a.e.ldc;
  const int64_t base = (row0 + rsel) * ldc + col;
  TC* c = static_cast<TC*>(a.C) + base;
  float x0[16], x1[16];
  if constexpr (kAux) {
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      x0[i] = x1[i] = 0.f;
      if (2 * i + rsel < rows_here) {
        const int64_t off = base + 2 * i * ldc;
        if constexpr (EPI == MAGMA_EPI_BIAS_RESIDUAL)
          load2(static_cast<const float*>(a.e.aux_in) + off, x0[i], x1[i]);
        else if constexpr (EPI == MAGMA_EPI_ACCUMULATE)
          load2(c + 2 * i * ldc, x0[i], x1[i]);
        else
          load2(static_cast<const TC*>(a.e.aux_in) + off, x0[i], x1[i]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    if (2 * i + rsel < rows_here) {
      const float2 v = *reinterpret_cast<const float2*>(st + 2 * i * P);
      float o0, o1;
      if constexpr (EPI == MAGMA_EPI_NONE) {
        o0 = v.x;
        o1 = v.y;
      } else if constexpr (EPI == MAGMA_EPI_BIAS) {
        o0 = __fadd_rn(v.x, b0);
        o1 = __fadd_rn(v.y, b1);
      } else if constexpr (EPI == MAGMA_EPI_BIAS_RESIDUAL) {
        o0 = __fadd_rn(x0[i], __fadd_rn(v.x, b0));
        o1 = __fadd_rn(x1[i], __fadd_rn(v.y, b1));
      } else if constexpr (EPI == MAGMA_EPI_BIAS_GELU || EPI == MAGMA_EPI_BIAS_RELU) {
        const float p0 = __fadd_rn(v.x, b0), p1 = __fadd_rn(v.y, b1);
        store2(static_cast<TC*>(a.e.aux_out) + base + 2 * i * ldc, p0, p1);
        if constexpr (EPI == MAGMA_EPI_BIAS_GELU) {
          o0 = gelu_t<TC>(p0);
          o1 = gelu_t<TC>(p1);
        } else {
          o0 = fmaxf(p0, 0.f);
          o1 = fmaxf(p1, 0.f);
        }
      } else if constexpr (EPI == MAGMA_EPI_DGELU) {
        o0 = __fmul_rn(v.x, gelu_grad_t<TC>(x0[i]));
        o1 = __fmul_rn(v.y, gelu_grad_t<TC>(x1[i]));
      } else if constexpr (EPI == MAGMA_EPI_DRELU) {
        o0 = x0[i] > 0.f ? v.x : 0.f;
        o1 = x1[i] > 0.f ? v.y : 0.f;
      } else {  // ACCUMULATE
        o0 = __fadd_rn(x0[i], v.x);
        o1 = __fadd_rn(x1[i], v.y);
      }
      store2(c + 2 * i * ldc, o0, o1);
    }
  }
}

// Asynchronous 16-byte global -> shared copies (the LSU path, completion by
// commit groups); valid = false writes 16 zero bytes without reading.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src),
               "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_group 0;" ::: "memory");
}

// Staged epilogue, 8 columns per lane: for one 32-column chunk staged as
// [32 rows][P] floats, lane (r8 = lane / 4, g = lane % 4) handles columns
// [col, col + 8) of rows r8, r8 + 8, r8 + 16, r8 + 24: 16-byte shared reads,
// 16-byte auxiliary loads (all issued first) and 16-byte stores, a warp
// instruction covering 8 rows x 64-128 contiguous bytes. Same arithmetic and
// order as epi_value.
template <typename TC, int EPI, int P>
__device__ __forceinline__ void epi_rows8(const TcArgs& a, const float* __restrict__ st,
                                          int64_t row0, int rows_here, int r8, int64_t col,
                                          const float (&b)[8], const uint4* pre = nullptr) {
  constexpr bool kAux = EPI == MAGMA_EPI_BIAS_RESIDUAL || EPI == MAGMA_EPI_DGELU ||
                        EPI == MAGMA_EPI_DRELU || EPI == MAGMA_EPI_ACCUMULATE;
  // auxiliary operand element type: the F32 residual stream, else C's type
  using AuxT = typename std::conditional<EPI == MAGMA_EPI_BIAS_RESIDUAL, float, TC>::type;
  constexpr int kWords = kAux ? (int)sizeof(AuxT) / 2 : 1;  // 16-B words per 8 elements
  const int64_t ldc = a.e.ldc;
  TC* C = static_cast<TC*>(a.C);
  const bool hb = a.e.bias != nullptr;
  // raw 16-byte words of the four rows' auxiliary operand, all loads in flight
  uint4 raw[4][kWords];
  const AuxT* src = EPI == MAGMA_EPI_ACCUMULATE ? reinterpret_cast<const AuxT*>(C)
                                                : static_cast<const AuxT*>(a.e.aux_in);
#pragma unroll
  for (int it = 0; it < 4; ++it) {
    const int r = it * 8 + r8;
    if (r >= rows_here) break;
    if constexpr (kAux && kWords == 1) {
      if (pre != nullptr) {  // BF16 auxiliary rows already staged in shared memory
        raw[it][0] = pre[it];
      } else if ((it & 1) == 0) {  // two rows' loads in flight at a time
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          if (r + 8 * k < rows_here) {
            const uint4* q = reinterpret_cast<const uint4*>(src + (row0 + r + 8 * k) * ldc + col);
            raw[it + k][0] = q[0];
          }
        }
      }
    } else if constexpr (kAux) {
      if ((it & 1) == 0) {  // two rows' loads in flight at a time
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          if (r + 8 * k < rows_here) {
            const uint4* q = reinterpret_cast<const uint4*>(src + (row0 + r + 8 * k) * ldc + col);
#pragma unroll
            for (int w = 0; w < kWords; ++w) raw[it + k][w] = q[w];
          }
        }
      }
    }
    const float4 lo = *reinterpret_cast<const float4*>(st + r * P);
    const float4 hi = *reinterpret_cast<const float4*>(st + r * P + 4);
    const float v[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
    const int64_t off = (row0 + r) * ldc + col;
    float x[8];
    if constexpr (kAux) load8(reinterpret_cast<const AuxT*>(raw[it]), x);
    float o[8];
    if constexpr (EPI == MAGMA_EPI_BIAS_RESIDUAL) {
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = __fadd_rn(x[i], hb ? __fadd_rn(v[i], b[i]) : v[i]);
    } else if constexpr (EPI == MAGMA_EPI_BIAS_GELU || EPI == MAGMA_EPI_BIAS_RELU) {
      float pre[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) pre[i] = hb ? __fadd_rn(v[i], b[i]) : v[i];
      store8(static_cast<TC*>(a.e.aux_out) + off, pre);
      if constexpr (EPI == MAGMA_EPI_BIAS_GELU && std::is_same<TC, __nv_bfloat16>::value) {
#pragma unroll
        for (int i = 0; i < 8; i += 2) gelu_pair_fast(o[i], o[i + 1], pre[i], pre[i + 1]);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i)
          o[i] = EPI == MAGMA_EPI_BIAS_GELU ? gelu_t<TC>(pre[i]) : fmaxf(pre[i], 0.f);
      }
    } else if constexpr (EPI == MAGMA_EPI_DGELU) {
      if constexpr (std::is_same<TC, __nv_bfloat16>::value) {
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
          float g0, g1;
          gelu_grad_pair_fast(g0, g1, x[i], x[i + 1]);
          f2_unpack(f2_mul(f2_pack(v[i], v[i + 1]), f2_pack(g0, g1)), o[i], o[i + 1]);
        }
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = __fmul_rn(v[i], gelu_grad_t<TC>(x[i]));
      }
    } else if constexpr (EPI == MAGMA_EPI_DRELU) {
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = x[i] > 0.f ? v[i] : 0.f;
    } else {  // ACCUMULATE
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = __fadd_rn(x[i], v[i]);
    }
    store8(C + off, o);
  }
}

template <int BN, bool A_MN, bool B_MN, typename TC, bool PAIR>
__global__ void __launch_bounds__(kGemmThreads, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
               const __grid_constant__ CUtensorMap tmC, TcArgs args) {
  using Cfg = TcCfg<BN, PAIR>;
  constexpr int kTM = PAIR ? 2 * kBM : kBM;  // output rows per tile
  constexpr int S = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = sm100::smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* base_ptr = smem_raw + (base - raw);
  const uint32_t bars = base + Cfg::kBarOffset;
  auto full_bar = [&](int s) { return bars + 8u * s; };
  auto empty_bar = [&](int s) { return bars + 8u * (S + s); };
  auto tfull_bar = [&](int a) { return bars + 8u * (2 * S + a); };
  auto tempty_bar = [&](int a) { return bars + 8u * (2 * S + 2 + a); };
  const uint32_t done_bar = bars + 8u * (2 * S + 4);
  const uint32_t tmem_slot = bars + 8u * (2 * S + 5);
  uint32_t* tmem_slot_ptr = reinterpret_cast<uint32_t*>(base_ptr + Cfg::kBarOffset + 8 * (2 * S + 5));

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t M = args.M, N = args.N, K = args.K;
  const int tiles_m = (int)((M + kTM - 1) / kTM);
  const int tiles_n = (int)((N + BN - 1) / BN);
  const int num_tiles = tiles_m * tiles_n;
  const int num_units = num_tiles * args.splits;
  const int kblocks = (int)((K + kBK - 1) / kBK);
  const uint32_t rank = PAIR ? sm100::cluster_ctarank() : 0u;
  const bool leader = rank == 0;
  const int ustart = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int ustride = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;

  if (threadIdx.x == 0) {
    sm100::prefetch_tensormap(&tmA);
    sm100::prefetch_tensormap(&tmB);
    for (int s = 0; s < S; ++s) {
      sm100::mbar_init(full_bar(s), 1);
      sm100::mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      sm100::mbar_init(tfull_bar(a), 1);
      sm100::mbar_init(tempty_bar(a), PAIR ? 2 * kEpiWarps : kEpiWarps);
    }
    sm100::mbar_init(done_bar, 1);
    sm100::fence_barrier_init();
  }
  if (warp == 1) {
    if constexpr (PAIR) sm100::tmem_alloc_pair(tmem_slot, Cfg::kTmemCols);
    else sm100::tmem_alloc(tmem_slot, Cfg::kTmemCols);
  }
  sm100::tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) sm100::cluster_sync();  // peer barriers initialised before any remote use
  sm100::tc_fence_after();
  const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t*>(tmem_slot_ptr);

  if (warp == 0 && lane == 0) {
    // ---------------------------- TMA producer ----------------------------
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    auto load = [&](uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
      if constexpr (PAIR) sm100::tma_load_2d_pair(dst, map, x, y, sm100::mapa_shared(bar, 0));
      else sm100::tma_load_2d(dst, map, x, y, bar);
    };
    for (int unit = ustart; unit < num_units && ok; unit += ustride) {
      const int tile = unit % num_tiles, split = unit / num_tiles;
      const int tm = args.n_fast ? tile / tiles_n : tile % tiles_m;
      const int tn = args.n_fast ? tile % tiles_n : tile / tiles_m;
      const int a_row0 = tm * kTM + (int)rank * kBM;
      const int b_row0 = tn * BN + (int)rank * Cfg::kBRows;
      const int kb0 = split * args.kb_per_split;
      const int kb1 = min(kblocks, kb0 + args.kb_per_split);
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!sm100::mbar_wait(empty_bar(stage), phase ^ 1u, args.err)) { ok = false; break; }
        const uint32_t sa = base + stage * Cfg::kStageBytes;
        const uint32_t sb = sa + Cfg::kABytes;
        // the leader's full barrier counts both CTAs' bytes
        if (leader) sm100::mbar_expect_tx(full_bar(stage), (PAIR ? 2 : 1) * Cfg::kStageBytes);
        if (!A_MN) {
          load(sa, &tmA, kb * kBK, a_row0, full_bar(stage));
        } else {
#pragma unroll
          for (int j = 0; j < kBM / 64; ++j)
            load(sa + j * 8192, &tmA, a_row0 + j * 64, kb * kBK, full_bar(stage));
        }
        if (!B_MN) {
          load(sb, &tmB, kb * kBK, b_row0, full_bar(stage));
        } else {
#pragma unroll
          for (int j = 0; j < Cfg::kBRows / 64; ++j)
            load(sb + j * 8192, &tmB, b_row0 + j * 64, kb * kBK, full_bar(stage));
        }
        if (++stage == S) { stage = 0; phase ^= 1u; }
      }
    }
    // Re-acquire every slot: all loads issued above have been consumed (and
    // the MMAs reading them completed) before this thread leaves.
    for (int i = 0; i < S && ok; ++i) {
      if (!sm100::mbar_wait(empty_bar(stage), phase ^ 1u, args.err)) ok = false;
      if (++stage == S) { stage = 0; phase ^= 1u; }
    }
  } else if (warp == 1 && lane == 0 && leader) {
    // ----------------------------- MMA issuer -----------------------------
    constexpr uint32_t idesc = sm100::idesc_bf16_f32(kTM, BN, A_MN ? 1 : 0, B_MN ? 1 : 0);
    auto commit = [&](uint32_t bar) {
      if constexpr (PAIR) sm100::mma_commit_pair(bar, 0x3);  // arrive in both CTAs
      else sm100::mma_commit(bar);
    };
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true;
    for (int unit = ustart; unit < num_units && ok; unit += ustride) {
      const int split = unit / num_tiles;
      const int kb0 = split * args.kb_per_split;
      const int kb1 = min(kblocks, kb0 + args.kb_per_split);
      if (!sm100::mbar_wait(tempty_bar(acc), acc_phase ^ 1u, args.err)) { ok = false; break; }
      sm100::tc_fence_after();
      const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!sm100::mbar_wait(full_bar(stage), phase, args.err)) { ok = false; break; }
        sm100::tc_fence_after();
        const uint32_t sa = base + stage * Cfg::kStageBytes;
        const uint32_t sb = sa + Cfg::kABytes;
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk) {
          // K-major: step 16 elements (32 B) inside the 128-B swizzle atom.
          // MN-major: step 16 K-rows (16 x 128 B) = two 1024-B atom rows.
          const uint64_t adesc =
              A_MN ? sm100::smem_desc_sw128(sa + kk * 2048, 8192, 1024)
                   : sm100::smem_desc_sw128(sa + kk * 32, 16, 1024);
          const uint64_t bdesc =
              B_MN ? sm100::smem_desc_sw128(sb + kk * 2048, 8192, 1024)
                   : sm100::smem_desc_sw128(sb + kk * 32, 16, 1024);
          if constexpr (PAIR)
            sm100::mma_bf16_ss_pair(d_tmem, adesc, bdesc, idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
          else
            sm100::mma_bf16_ss(d_tmem, adesc, bdesc, idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
        }
        commit(empty_bar(stage));
        if (++stage == S) { stage = 0; phase ^= 1u; }
      }
      if (!ok) break;
      commit(tfull_bar(acc));
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
    // Wait for every MMA this thread issued before TMEM is released.
    commit(done_bar);
    sm100::mbar_wait(done_bar, 0, args.err);
  } else if (PAIR && warp == 1 && lane == 0) {
    // non-leader: the leader's MMAs write this CTA's TMEM; wait for all of them
    sm100::mbar_wait(done_bar, 0, args.err);
  } else if (warp >= 2) {
    // ------------------------------ epilogue ------------------------------
    // Warp w owns TMEM lane quarter q = w & 3 (tile rows [32q, 32q+32)) and
    // column half h = (w - 2) / 4. Plain / bias epilogues and split-K partials:
    // thread = row, 16-byte stores. Epilogues that read auxiliary tensors or
    // write two outputs: per 32-column chunk the accumulators go through a
    // padded shared-memory stage, then each lane takes a column pair of one of
    // two rows, so every global access is a contiguous row segment, and all
    // auxiliary loads of the chunk are issued before the first store.
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    constexpr int kCols = BN / 2;  // columns per epilogue warp
    float* stage = reinterpret_cast<float*>(base_ptr + Cfg::kStageOffset) +
                   (warp - 2) * Cfg::kStageWarpFloats;
    const bool vec2 = args.vec_ok != 0;
    const bool epi_vec8 = args.epi_vec8 != 0;
    const bool vec8_staged =
        epi_vec8 && (std::is_same<TC, __nv_bfloat16>::value ||
                     args.e.epi == MAGMA_EPI_BIAS_RESIDUAL || args.e.epi == MAGMA_EPI_ACCUMULATE);
    // the tile's bias columns of this warp, staged after the 32 x 36 chunk stage
    float* bias_s = stage + 32 * Cfg::kStagePitch;
    // BF16 activation-VJP epilogues: the next 32-column chunk of the auxiliary
    // operand (32 rows x 64 bytes) is copied into shared memory by cp.async
    // while the current one is computed (the first chunk of a tile while the
    // accumulator is)
    const bool aux_smem = vec8_staged && std::is_same<TC, __nv_bfloat16>::value &&
                          (args.e.epi == MAGMA_EPI_DGELU || args.e.epi == MAGMA_EPI_DRELU);
    uint8_t* aux_s = reinterpret_cast<uint8_t*>(bias_s + 128);
    auto issue_aux = [&](int m0_, int n0_, int c0_) {
      const int r8 = lane >> 2, g8 = lane & 3;
      const __nv_bfloat16* auxp = static_cast<const __nv_bfloat16*>(args.e.aux_in);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int r = r8 + 8 * k;
        const int64_t row = (int64_t)m0_ + q * 32 + r;
        const int64_t col = (int64_t)n0_ + c0_ + 8 * g8;
        const bool valid = row < M && col + 8 <= N;
        cp_async16(sm100::smem_u32(aux_s + r * 64 + g8 * 16),
                   valid ? static_cast<const void*>(auxp + row * args.e.ldc + col)
                         : static_cast<const void*>(auxp),
                   valid);
      }
      cp_async_commit();
    };
    const bool ws_vec8 = (N % 8) == 0;
    const bool c_vec8 = args.vec8_ok != 0;
    const bool direct = args.splits > 1 || args.e.epi == MAGMA_EPI_NONE ||
                        args.e.epi == MAGMA_EPI_BIAS || args.e.epi == MAGMA_EPI_ROWSTATS;
    const bool rowstats = args.splits == 1 && args.e.epi == MAGMA_EPI_ROWSTATS;
    const bool tma_direct = direct && args.tma_out != 0;
    uint8_t* wbuf = reinterpret_cast<uint8_t*>(stage);
    int blk_it = 0;  // 64-column blocks this warp has stored through TMA
    const bool has_bias = args.e.bias != nullptr &&
                          (args.e.epi == MAGMA_EPI_BIAS || args.e.epi == MAGMA_EPI_BIAS_GELU ||
                           args.e.epi == MAGMA_EPI_BIAS_RESIDUAL || args.e.epi == MAGMA_EPI_BIAS_RELU);
    // auxiliary operand the staged epilogue reads, for the L2 prefetch
    const char* aux_pf = nullptr;
    int64_t aux_esz = sizeof(TC);
    if (args.splits == 1) {
      if (args.e.epi == MAGMA_EPI_BIAS_RESIDUAL) {
        aux_pf = static_cast<const char*>(args.e.aux_in);
        aux_esz = 4;
      } else if (args.e.epi == MAGMA_EPI_DGELU || args.e.epi == MAGMA_EPI_DRELU) {
        aux_pf = static_cast<const char*>(args.e.aux_in);
      } else if (args.e.epi == MAGMA_EPI_ACCUMULATE) {
        aux_pf = static_cast<const char*>(args.C);
      }
    }
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int unit = ustart; unit < num_units; unit += ustride) {
      const int tile = unit % num_tiles, split = unit / num_tiles;
      const int tm = args.n_fast ? tile / tiles_n : tile % tiles_m;
      const int tn = args.n_fast ? tile % tiles_n : tile / tiles_m;
      const int m0 = tm * kTM + (int)rank * kBM;
      const int n0 = tn * BN + half * kCols;
      // bias of this warp's columns for the TMA-store epilogue: lane l holds
      // column n0 + 32 j + l, loaded before the accumulator wait
      float bl[kCols / 32];
#pragma unroll
      for (int j = 0; j < kCols / 32; ++j) {
        const int64_t col = (int64_t)n0 + 32 * j + lane;
        bl[j] = (tma_direct && has_bias && args.splits == 1 && col < N) ? args.e.bias[col] : 0.f;
      }
      if (aux_smem) issue_aux(m0, n0, 0);  // the tile's first chunk
      if (vec8_staged && has_bias && !direct) {
        // this warp's kCols bias values, read once per tile while the
        // accumulator is still being computed (columns past N read as 0)
        for (int c = 4 * lane; c < kCols; c += 128) {
          float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
          if ((int64_t)n0 + c + 4 <= N) {
            v = *reinterpret_cast<const float4*>(args.e.bias + n0 + c);
          } else {
            if ((int64_t)n0 + c < N) v.x = args.e.bias[n0 + c];
            if ((int64_t)n0 + c + 1 < N) v.y = args.e.bias[n0 + c + 1];
            if ((int64_t)n0 + c + 2 < N) v.z = args.e.bias[n0 + c + 2];
          }
          *reinterpret_cast<float4*>(bias_s + c) = v;
        }
        __syncwarp();
      }
      if (aux_pf != nullptr) {
        // While the accumulator is still being computed, pull this warp's
        // block of the auxiliary operand (its 32 rows x kCols columns) into L2,
        // one row per lane, so the epilogue's loads of it hit L2.
        const int64_t row = (int64_t)m0 + q * 32 + lane;
        if (row < M && n0 < N) {
          const char* p0 = aux_pf + (row * args.e.ldc + n0) * aux_esz;
          const char* p1 = p0 + min((int64_t)kCols, (int64_t)N - n0) * aux_esz;
          for (const char* p = reinterpret_cast<const char*>(reinterpret_cast<uintptr_t>(p0) & ~(uintptr_t)127);
               p < p1; p += 128)
            asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
        }
      }
      if (!sm100::mbar_wait(tfull_bar(acc), acc_phase, args.err)) break;
      sm100::tc_fence_after();
      const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN) +
                             (uint32_t)(half * kCols);
      const int64_t row0 = (int64_t)m0 + q * 32;
      const int rows_here = (int)min((int64_t)32, M - row0);
      auto release = [&]() {  // last TMEM read of this accumulator by this warp
        sm100::tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if constexpr (PAIR) sm100::mbar_arrive_cluster(sm100::mapa_shared(tempty_bar(acc), 0));
          else sm100::mbar_arrive(tempty_bar(acc));
        }
      };
      if (tma_direct) {
#pragma unroll
        for (int c0 = 0; c0 < kCols; c0 += 64) {
          uint32_t ra[32], rb[32];
          sm100::tmem_ld32(taddr + c0, ra);
          sm100::tmem_ld32(taddr + c0 + 32, rb);
          sm100::tmem_wait_ld();
          if (c0 + 64 >= kCols) release();
          if (n0 + c0 >= N || row0 >= M) continue;
          if (has_bias && args.splits == 1) {  // split partials: bias added by the reduce
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              ra[i] = __float_as_uint(__fadd_rn(__uint_as_float(ra[i]),
                                                __shfl_sync(0xffffffffu, bl[c0 / 32], i)));
              rb[i] = __float_as_uint(__fadd_rn(__uint_as_float(rb[i]),
                                                __shfl_sync(0xffffffffu, bl[c0 / 32 + 1], i)));
            }
          }
          if (args.splits > 1) {
            tma_block64_f32(wbuf, ra, rb, &tmC, n0 + c0, (int)row0, split, N, lane);
          } else if constexpr (std::is_same<TC, float>::value) {
            tma_block64_f32(wbuf, ra, rb, &tmC, n0 + c0, (int)row0, -1, N, lane);
            if (rowstats && row0 + lane < M)
              row_stats64<TC>(ra, rb, (int64_t)n0 + c0, N,
                              static_cast<float2*>(args.e.aux_out) + ((n0 + c0) >> 6) * M + row0 + lane);
          } else {
            uint32_t pk[32];
#pragma unroll
            for (int p = 0; p < 16; ++p) {
              const __nv_bfloat162 lo = __floats2bfloat162_rn(__uint_as_float(ra[2 * p]),
                                                              __uint_as_float(ra[2 * p + 1]));
              const __nv_bfloat162 hi = __floats2bfloat162_rn(__uint_as_float(rb[2 * p]),
                                                              __uint_as_float(rb[2 * p + 1]));
              pk[p] = *reinterpret_cast<const uint32_t*>(&lo);
              pk[16 + p] = *reinterpret_cast<const uint32_t*>(&hi);
            }
            tma_block64_bf16(wbuf, blk_it, pk, &tmC, n0 + c0, (int)row0, N, lane);
            if (rowstats && row0 + lane < M)
              stats64_packed(pk, (int64_t)n0 + c0, N,
                             static_cast<float2*>(args.e.aux_out) + ((n0 + c0) >> 6) * M + row0 + lane);
          }
          ++blk_it;
        }
      } else if (direct) {
#pragma unroll 1
        for (int c0 = 0; c0 < kCols; c0 += 64) {
          uint32_t ra[32], rb[32];
          sm100::tmem_ld32(taddr + c0, ra);
          sm100::tmem_ld32(taddr + c0 + 32, rb);
          sm100::tmem_wait_ld();
          if (c0 + 64 >= kCols) release();
          const int64_t row = row0 + lane;
          if (row < M && n0 + c0 < N) {
            if (args.splits > 1)
              direct_store64<float>(args.ws + (int64_t)split * M * N + row * N, nullptr,
                                    (int64_t)n0 + c0, N, ra, rb, ws_vec8);
            else if (rowstats && std::is_same<TC, __nv_bfloat16>::value)
              direct_store64_stats(reinterpret_cast<__nv_bfloat16*>(args.C) + row * args.e.ldc,
                                   (int64_t)n0 + c0, N, ra, rb, c_vec8,
                                   static_cast<float2*>(args.e.aux_out) + ((n0 + c0) >> 6) * M + row);
            else {
              direct_store64<TC>(static_cast<TC*>(args.C) + row * args.e.ldc,
                                 has_bias ? args.e.bias : nullptr, (int64_t)n0 + c0, N, ra, rb,
                                 c_vec8);
              if (rowstats)
                row_stats64<TC>(ra, rb, (int64_t)n0 + c0, N,
                                static_cast<float2*>(args.e.aux_out) + ((n0 + c0) >> 6) * M + row);
            }
          }
        }
      } else {
        constexpr int P = Cfg::kStagePitch;
        const int cp = lane & 15;     // column pair within the chunk
        const int rsel = lane >> 4;   // row parity handled by this lane
#pragma unroll 1
        for (int c0 = 0; c0 < kCols; c0 += 32) {
          uint32_t ra[32];
          sm100::tmem_ld32(taddr + c0, ra);
          sm100::tmem_wait_ld();
          if (c0 + 32 >= kCols) release();
          float* srow = stage + lane * P;
#pragma unroll
          for (int j = 0; j < 8; ++j)
            *reinterpret_cast<float4*>(srow + 4 * j) =
                make_float4(__uint_as_float(ra[4 * j]), __uint_as_float(ra[4 * j + 1]),
                            __uint_as_float(ra[4 * j + 2]), __uint_as_float(ra[4 * j + 3]));
          __syncwarp();
          if (vec8_staged) {
            const int r8 = lane >> 2, g8 = lane & 3;
            uint4 pre[4];
            if (aux_smem) {  // the whole warp: this chunk's auxiliary rows, then the next copy
              cp_async_wait_all();
              __syncwarp();
#pragma unroll
              for (int k = 0; k < 4; ++k)
                pre[k] = *reinterpret_cast<const uint4*>(aux_s + (r8 + 8 * k) * 64 + g8 * 16);
              __syncwarp();
              if (c0 + 32 < kCols) issue_aux(m0, n0, c0 + 32);
            }
            const int64_t col8 = (int64_t)n0 + c0 + 8 * g8;
            if (col8 < N && rows_here > 0) {
              const float* st8 = stage + r8 * P + 8 * g8;
              if (col8 + 8 <= N) {
                float b8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
                if (has_bias) {  // staged in shared memory at the start of the tile
                  const float4 lo = *reinterpret_cast<const float4*>(bias_s + c0 + 8 * g8);
                  const float4 hi = *reinterpret_cast<const float4*>(bias_s + c0 + 8 * g8 + 4);
                  b8[0] = lo.x; b8[1] = lo.y; b8[2] = lo.z; b8[3] = lo.w;
                  b8[4] = hi.x; b8[5] = hi.y; b8[6] = hi.z; b8[7] = hi.w;
                }
                if constexpr (std::is_same<TC, float>::value) {
                  // F32 outputs take this path only for the transcendental-free epilogues
                  if (args.e.epi == MAGMA_EPI_BIAS_RESIDUAL)
                    epi_rows8<TC, MAGMA_EPI_BIAS_RESIDUAL, P>(args, st8 - r8 * P, row0, rows_here, r8, col8, b8);
                  else
                    epi_rows8<TC, MAGMA_EPI_ACCUMULATE, P>(args, st8 - r8 * P, row0, rows_here, r8, col8, b8);
                } else switch (args.e.epi) {
                  case MAGMA_EPI_BIAS_GELU: epi_rows8<TC, MAGMA_EPI_BIAS_GELU, P>(args, st8 - r8 * P, row0, rows_here, r8, col8, b8); break;
                  case MAGMA_EPI_BIAS_RESIDUAL: epi_rows8<TC, MAGMA_EPI_BIAS_RESIDUAL, P>(args, st8 - r8 * P, row0, rows_here, r8, col8, b8); break;
                  case MAGMA_EPI_DGELU: epi_rows8<TC, MAGMA_EPI_DGELU, P>(args, st8 - r8 * P, row0, rows_here, r8, col8, b8, aux_smem ? pre : nullptr); break;
                  case MAGMA_EPI_ACCUMULATE: epi_rows8<TC, MAGMA_EPI_ACCUMULATE, P>(args, st8 - r8 * P, row0, rows_here, r8, col8, b8); break;
                  case MAGMA_EPI_BIAS_RELU: epi_rows8<TC, MAGMA_EPI_BIAS_RELU, P>(args, st8 - r8 * P, row0, rows_here, r8, col8, b8); break;
                  default: epi_rows8<TC, MAGMA_EPI_DRELU, P>(args, st8 - r8 * P, row0, rows_here, r8, col8, b8, aux_smem ? pre : nullptr); break;
                }
              } else {  // ragged last columns, element by element
                TC* C = static_cast<TC*>(args.C);
                for (int r = r8; r < rows_here; r += 8)
                  for (int i = 0; col8 + i < N; ++i) {
                    const int64_t off = (row0 + r) * args.e.ldc + col8 + i;
                    C[off] = from_f32<TC>(epi_value<TC>(args.e, C, off, col8 + i, st8[(r - r8) * P + i]));
                  }
              }
            }
            __syncwarp();
            continue;
          }
          const int64_t col = (int64_t)n0 + c0 + 2 * cp;
          if (col < N && rows_here > 0) {
            const bool pair = col + 1 < N;
            float b0 = 0.f, b1 = 0.f;
            if (has_bias) {
              b0 = args.e.bias[col];
              b1 = pair ? args.e.bias[col + 1] : 0.f;
            }
            const float* st = stage + rsel * P + 2 * cp;
            if (pair && vec2) {
              switch (args.e.epi) {
                case MAGMA_EPI_BIAS_GELU: epi_rows<TC, MAGMA_EPI_BIAS_GELU, P>(args, st, row0, rows_here, rsel, col, b0, b1); break;
                case MAGMA_EPI_BIAS_RESIDUAL: epi_rows<TC, MAGMA_EPI_BIAS_RESIDUAL, P>(args, st, row0, rows_here, rsel, col, b0, b1); break;
                case MAGMA_EPI_DGELU: epi_rows<TC, MAGMA_EPI_DGELU, P>(args, st, row0, rows_here, rsel, col, b0, b1); break;
                case MAGMA_EPI_ACCUMULATE: epi_rows<TC, MAGMA_EPI_ACCUMULATE, P>(args, st, row0, rows_here, rsel, col, b0, b1); break;
                case MAGMA_EPI_BIAS_RELU: epi_rows<TC, MAGMA_EPI_BIAS_RELU, P>(args, st, row0, rows_here, rsel, col, b0, b1); break;
                default: epi_rows<TC, MAGMA_EPI_DRELU, P>(args, st, row0, rows_here, rsel, col, b0, b1); break;
              }
            } else {
              for (int rr = rsel; rr < rows_here; rr += 2) {
                const float2 v = *reinterpret_cast<const float2*>(st + (rr - rsel) * P);
                epi_store2<TC>(args, row0 + rr, col, v.x, v.y, b0, b1, false);
              }
            }
          }
          __syncwarp();
        }
      }
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
    // the TMA stores must finish before the shared memory they read goes away
    if (tma_direct && lane == 0) sm100::bulk_wait_group_all();
    if (aux_smem) cp_async_wait_all();  // no copy into shared memory outlives the CTA
    __syncwarp();
  }
  sm100::tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) sm100::cluster_sync();
  if (warp == 1) {
    __syncwarp();
    sm100::tc_fence_after();
    if constexpr (PAIR) sm100::tmem_dealloc_pair(tmem_base, Cfg::kTmemCols);
    else sm100::tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
}

struct TcPlan {
  int bn;
  int splits;
  int kb_per_split;
  bool pair;
};

// Override for measurements: MAGMA_GEMM_MODE = 1sm | 2sm | 1sm128 | 1sm256 |
// 2sm128 | 2sm256 restricts the plan to those tile options (default: all).
// Returns a bit mask over the options {1sm128, 1sm256, 2sm128, 2sm256}.
// MAGMA_GEMM_MODE restricts the plan search (1sm, 2sm, 1sm128, 1sm256,
// 2sm128, 2sm256); read on every call so a process can compare options.
int gemm_option_mask() {
  const char* v = getenv("MAGMA_GEMM_MODE");
  if (v == nullptr) return 0xF;
  if (strcmp(v, "1sm") == 0) return 0x3;
  if (strcmp(v, "2sm") == 0) return 0xC;
  if (strcmp(v, "1sm128") == 0) return 0x1;
  if (strcmp(v, "1sm256") == 0) return 0x2;
  if (strcmp(v, "2sm128") == 0) return 0x4;
  if (strcmp(v, "2sm256") == 0) return 0x8;
  return 0xF;
}

// MAGMA_GEMM_PLAN="pair,bn,splits" (e.g. "1,256,3") fixes the plan outright;
// ignored when it does not fit the shape.
bool forced_plan(int64_t M, int64_t K, TcPlan* out) {
  const char* v = getenv("MAGMA_GEMM_PLAN");
  if (v == nullptr) return false;
  int pair = 0, bn = 0, splits = 0;
  if (sscanf(v, "%d,%d,%d", &pair, &bn, &splits) != 3) return false;
  if ((bn != 128 && bn != 256) || splits < 1 || (pair && M < 256)) return false;
  const int kblocks = (int)ceil_div(K, kBK);
  const int kbps = (int)ceil_div(kblocks, splits);
  *out = {bn, (int)ceil_div(kblocks, kbps), kbps, pair != 0};
  return true;
}

// Epilogue cost inputs of the plan model: bytes moved per output element
// (C plus the auxiliary tensor it reads or writes) and issue time per output
// element (us per 10^4 elements of one CTA's tile).
struct EpiCost {
  double bytes;
  double us_1e4;
};
EpiCost epi_cost(int epi, bool c32) {
  const double c = c32 ? 4.0 : 2.0;
  switch (epi) {
    case MAGMA_EPI_BIAS_RESIDUAL: return {c + 4.0, 1.71};
    case MAGMA_EPI_BIAS_GELU:
    case MAGMA_EPI_BIAS_RELU: return {2.0 * c, 2.33};
    case MAGMA_EPI_DGELU:
    case MAGMA_EPI_DRELU: return {2.0 * c, 2.33};
    case MAGMA_EPI_ACCUMULATE: return {2.0 * c, 2.33};
    default: return {c, c32 ? 2.53 : 1.95};   // direct row stores
  }
}

// Picks CTA pairing, tile width BN and the K-split count from a cost model
// fitted to measured B200 times of every option on the GPT-2 training shapes:
// a unit (one output tile, or one K-slice of it) costs the largest of its
// tensor-core time (k-blocks x time per 64-deep k-block), its L2->SMEM load
// time plus output traffic at the per-SM L2 bandwidth, and its epilogue (the
// epilogue of one tile overlaps the next tile's main loop); the launch costs
// waves x unit + one exposed epilogue, plus the cluster set-up for CTA pairs
// and, when splitting, the reduce pass over the F32 partials.
TcPlan choose_plan(int64_t M, int64_t N, int64_t K, int epi, bool c32) {
  TcPlan forced;
  if (forced_plan(M, K, &forced)) return forced;
  const int sms = num_sms();
  const int kblocks = (int)ceil_div(K, kBK);
  // per option {1-CTA 128x128, 1-CTA 128x256, pair 256x128, pair 256x256}:
  const double kb_us[4] = {0.300, 0.515, 0.311, 0.335};    // tensor time per k-block
  const double kb_bytes[4] = {32768, 49152, 24576, 32768};  // SMEM fill per k-block per CTA
  const double l2_bytes_per_us[4] = {96.0e3, 94.7e3, 75.5e3, 87.9e3};  // per SM
  const double pair_setup_us = 1.8, split_setup_us = 0.26, reduce_bytes_per_us = 6.0e6;
  const EpiCost ec = epi_cost(epi, c32);
  const EpiCost ep = epi_cost(MAGMA_EPI_NONE, true);  // F32 partial stores
  const int allowed = gemm_option_mask();
  // Best unsplit and best split plan; a split plan has to win by 10% (it
  // also costs workspace traffic the model does not see in the next kernel).
  TcPlan best1{256, 1, kblocks, false}, bests{256, 1, kblocks, false};
  double t1 = 1e30, ts = 1e30;
  for (int opt = 0; opt < 4; ++opt) {
    const bool pair = opt >= 2;
    if (!(allowed & (1 << opt))) continue;
    if (pair && M < 256) continue;
    const int bn = (opt & 1) ? 256 : 128;
    const int64_t tiles = ceil_div(M, pair ? 256 : kBM) * ceil_div(N, bn);
    const int slots = pair ? sms / 2 : sms;
    for (int s = 1; s <= 16; ++s) {
      const int kbps = (int)ceil_div(kblocks, s);
      if (s > 1 && kbps < 4) break;
      const int splits = (int)ceil_div(kblocks, kbps);
      if (splits != s) continue;
      const EpiCost& e = splits > 1 ? ep : ec;
      const double elems = (double)kBM * bn;  // output elements per CTA tile
      const double epi_us = e.us_1e4 * elems * 1e-4;
      const double load_us = (kbps * kb_bytes[opt] + e.bytes * elems) / l2_bytes_per_us[opt];
      double unit = kbps * kb_us[opt];
      if (load_us > unit) unit = load_us;
      if (epi_us > unit) unit = epi_us;
      const double waves = (double)ceil_div(tiles * splits, slots);
      double t = waves * unit + epi_us + (pair ? pair_setup_us : 0.0);
      if (splits > 1) {
        t += split_setup_us + ((splits + 1) * 4.0 + ec.bytes) * M * N / reduce_bytes_per_us;
        if (t < ts) {
          ts = t;
          bests = {bn, splits, kbps, pair};
        }
      } else if (t < t1) {
        t1 = t;
        best1 = {bn, 1, kbps, pair};
      }
    }
  }
  const TcPlan best = ts < 0.9 * t1 ? bests : best1;
  return best;
}

// c = epilogue(sum over splits of ws[s]) in split order (deterministic).
template <typename TC>
__global__ void __launch_bounds__(256)
splitk_reduce(const float* __restrict__ ws, int splits, int64_t M, int64_t N, TC* __restrict__ C,
              EpiArgs e, int vec_c) {
  // Thread = 4 consecutive columns of one row when N % 4 == 0 (16-byte loads
  // of every partial plane), else one column. Planes are added in split order.
  const int64_t plane = M * N;
  const bool v4 = (N & 3) == 0;
  const int64_t per_row = v4 ? N >> 2 : N;
  for (int64_t row = blockIdx.y; row < M; row += gridDim.y) {
    for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < per_row;
         c += (int64_t)gridDim.x * blockDim.x) {
      if (v4) {
        const int64_t i = row * N + c * 4;
        float acc[4];
        load4(ws + i, acc);
        int sp = 1;
        // four planes' loads in flight before their adds (same addition order)
        for (; sp + 3 < splits; sp += 4) {
          float t[4][4];
#pragma unroll
          for (int j = 0; j < 4; ++j) load4(ws + (int64_t)(sp + j) * plane + i, t[j]);
#pragma unroll
          for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int k = 0; k < 4; ++k) acc[k] += t[j][k];
        }
        for (; sp < splits; ++sp) {
          float t[4];
          load4(ws + (int64_t)sp * plane + i, t);
#pragma unroll
          for (int k = 0; k < 4; ++k) acc[k] += t[k];
        }
        const int64_t off = row * e.ldc + c * 4;
        float o[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) o[k] = epi_value<TC>(e, C, off + k, c * 4 + k, acc[k]);
        if (vec_c) {
          store4(C + off, o);
        } else {
#pragma unroll
          for (int k = 0; k < 4; ++k) C[off + k] = from_f32<TC>(o[k]);
        }
      } else {
        const int64_t i = row * N + c;
        float acc = ws[i];
        for (int sp = 1; sp < splits; ++sp) acc += ws[(int64_t)sp * plane + i];
        const int64_t off = row * e.ldc + c;
        C[off] = from_f32<TC>(epi_value<TC>(e, C, off, c, acc));
      }
    }
  }
}

template <int BN, bool A_MN, bool B_MN, typename TC, bool PAIR>
magma_status_t launch_tc(const void* a, const void* b, int64_t M, int64_t N, int64_t K,
                         int64_t lda, int64_t ldb, const TcArgs& args, cudaStream_t stream) {
  static_assert(BN == 128 || BN == 256, "BN");
  using Cfg = TcCfg<BN, PAIR>;
  CUtensorMap ta, tb;
  magma_status_t st;
  if (!A_MN)
    st = encode_tensor_map_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a, K, M, lda * 2, 64, kBM,
                              CU_TENSOR_MAP_SWIZZLE_128B);
  else
    st = encode_tensor_map_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a, M, K, lda * 2, 64, 64,
                              CU_TENSOR_MAP_SWIZZLE_128B);
  if (st) return st;
  if (!B_MN)
    st = encode_tensor_map_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, b, K, N, ldb * 2, 64,
                              Cfg::kBRows, CU_TENSOR_MAP_SWIZZLE_128B);
  else
    st = encode_tensor_map_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, b, N, K, ldb * 2, 64, 64,
                              CU_TENSOR_MAP_SWIZZLE_128B);
  if (st) return st;
  // Store map of the direct epilogue: the F32 split-K partials [splits][M][N]
  // as a 3-D tensor, or C itself (32 x 32 boxes, 64-byte swizzle for BF16
  // rows of 64 bytes, 128-byte swizzle for F32 rows of 128 bytes).
  CUtensorMap tc;
  memset(&tc, 0, sizeof(tc));
  TcArgs a2 = args;
  a2.tma_out = 0;
  const bool direct = args.splits > 1 || args.e.epi == MAGMA_EPI_NONE ||
                      args.e.epi == MAGMA_EPI_BIAS || args.e.epi == MAGMA_EPI_ROWSTATS;
  if (direct && args.splits > 1) {
    if (N % 4 == 0 && aligned16(args.ws)) {
      const uint64_t dims[3] = {(uint64_t)N, (uint64_t)M, (uint64_t)args.splits};
      const uint64_t strides[2] = {(uint64_t)N * 4, (uint64_t)(M * N * 4)};
      const uint32_t box[3] = {32, 32, 1};
      if (magma_status_t s3 = encode_tensor_map_3d(&tc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, args.ws,
                                                   dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B))
        return s3;
      a2.tma_out = 1;
    }
  } else if (direct) {
    const int64_t row_bytes = args.e.ldc * (int64_t)sizeof(TC);
    if (row_bytes % 16 == 0 && aligned16(args.C)) {
      const bool bf = std::is_same<TC, __nv_bfloat16>::value;
      if (magma_status_t s3 = encode_tensor_map_2d(
              &tc, bf ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, args.C,
              N, M, row_bytes, 32, 32, bf ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B))
        return s3;
      a2.tma_out = 1;
    }
  }
  auto kern = gemm_tc_kernel<BN, A_MN, B_MN, TC, PAIR>;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    if (magma_status_t s2 = cuda_status(
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes),
            "cudaFuncSetAttribute(gemm)"))
      return s2;
    attr_set[dev] = true;
  }
  const int64_t units = ceil_div(M, PAIR ? 2 * kBM : kBM) * ceil_div(N, BN) * args.splits;
  if constexpr (PAIR) {
    int pairs = num_sms() / 2;
    if (units < pairs) pairs = (int)units;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(2 * pairs));
    cfg.blockDim = dim3(kGemmThreads);
    cfg.dynamicSmemBytes = Cfg::kSmemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (magma_status_t st = cuda_status(cudaLaunchKernelEx(&cfg, kern, ta, tb, tc, a2),
                                        "gemm_tcgen05_pair launch"))
      return st;
  } else {
    int grid = num_sms();
    if (units < grid) grid = (int)units;
    kern<<<grid, kGemmThreads, Cfg::kSmemBytes, stream>>>(ta, tb, tc, a2);
  }
  if (magma_status_t st = check_launch("gemm_tcgen05")) return st;
  if (args.splits > 1) {
    const int64_t per_row = (N & 3) == 0 ? N / 4 : N;
    int64_t gx = ceil_div(per_row, 256);
    if (gx > 16) gx = 16;
    int64_t gy = (8LL * num_sms() + gx - 1) / gx;
    if (gy > M) gy = M;
    if (gy > 65535) gy = 65535;
    const int vec_c = (args.e.ldc % 4) == 0 && aligned16(args.C);
    splitk_reduce<TC><<<dim3((unsigned)gx, (unsigned)gy), 256, 0, stream>>>(
        args.ws, args.splits, M, N, static_cast<TC*>(args.C), args.e, vec_c);
    return check_launch("gemm_splitk_reduce");
  }
  return MAGMA_OK;
}

template <int BN, typename TC, bool PAIR>
magma_status_t dispatch_major(const void* a, const void* b, int64_t M, int64_t N, int64_t K,
                              int64_t lda, int64_t ldb, int ta, int tb, const TcArgs& args,
                              cudaStream_t s) {
  const bool a_mn = ta != 0;   // A stored [K, M]
  const bool b_mn = tb == 0;   // B stored [K, N]
  if (!a_mn && !b_mn) return launch_tc<BN, false, false, TC, PAIR>(a, b, M, N, K, lda, ldb, args, s);
  if (!a_mn && b_mn) return launch_tc<BN, false, true, TC, PAIR>(a, b, M, N, K, lda, ldb, args, s);
  if (a_mn && !b_mn) return launch_tc<BN, true, false, TC, PAIR>(a, b, M, N, K, lda, ldb, args, s);
  return launch_tc<BN, true, true, TC, PAIR>(a, b, M, N, K, lda, ldb, args, s);
}

template <typename TC>
magma_status_t dispatch_plan(const TcPlan& plan, const void* a, const void* b, int64_t M,
                             int64_t N, int64_t K, int64_t lda, int64_t ldb, int ta, int tb,
                             const TcArgs& args, cudaStream_t s) {
  if (plan.pair)
    return plan.bn == 256 ? dispatch_major<256, TC, true>(a, b, M, N, K, lda, ldb, ta, tb, args, s)
                          : dispatch_major<128, TC, true>(a, b, M, N, K, lda, ldb, ta, tb, args, s);
  return plan.bn == 256 ? dispatch_major<256, TC, false>(a, b, M, N, K, lda, ldb, ta, tb, args, s)
                        : dispatch_major<128, TC, false>(a, b, M, N, K, lda, ldb, ta, tb, args, s);
}

// K splits of the F32 kernel: when its output tiles fill under half of the
// SMs and K is long, the K loop is cut into up to 16 chunks of whole 64-deep
// blocks (so that every SM-limited, latency-bound chain is shorter).
int simt_splits(int64_t M, int64_t N, int64_t K, int64_t* kps) {
  const int64_t tiles = ceil_div(N, kSimtBN) * ceil_div(M, kSimtBM);
  *kps = K;
  if (tiles * 2 > num_sms() || K < 256) return 1;
  int64_t sp = ceil_div(num_sms(), tiles);
  if (sp > 16) sp = 16;
  if (sp > K / 64) sp = K / 64;
  if (sp < 2) return 1;
  *kps = ceil_div(ceil_div(K, sp), 64) * 64;
  return (int)ceil_div(K, *kps);
}

size_t simt_workspace(int64_t M, int64_t N, int64_t K) {
  int64_t kps;
  const int sp = simt_splits(M, N, K, &kps);
  return sp > 1 ? (size_t)sp * M * N * sizeof(float) : 0;
}

template <typename TA, typename TC>
magma_status_t launch_simt(const void* a, const void* b, void* c, int64_t M, int64_t N, int64_t K,
                           int64_t lda, int64_t ldb, int ta, int tb, const EpiArgs& e,
                           void* workspace, size_t workspace_bytes, cudaStream_t s) {
  int64_t kps = K;
  int splits = simt_splits(M, N, K, &kps);
  if (splits > 1 && (workspace == nullptr || !aligned16(workspace) ||
                     workspace_bytes < (size_t)splits * M * N * sizeof(float))) {
    splits = 1;
    kps = K;
  }
  float* ws = splits > 1 ? static_cast<float*>(workspace) : nullptr;
  dim3 grid((unsigned)ceil_div(N, kSimtBN), (unsigned)ceil_div(M, kSimtBM), (unsigned)splits);
  const TA* A = (const TA*)a;
  const TA* B = (const TA*)b;
  TC* C = (TC*)c;
  if (!ta && !tb) gemm_simt_kernel<TA, TC, false, false><<<grid, 256, 0, s>>>(A, B, C, M, N, K, lda, ldb, e, kps, ws);
  else if (!ta && tb) gemm_simt_kernel<TA, TC, false, true><<<grid, 256, 0, s>>>(A, B, C, M, N, K, lda, ldb, e, kps, ws);
  else if (ta && !tb) gemm_simt_kernel<TA, TC, true, false><<<grid, 256, 0, s>>>(A, B, C, M, N, K, lda, ldb, e, kps, ws);
  else gemm_simt_kernel<TA, TC, true, true><<<grid, 256, 0, s>>>(A, B, C, M, N, K, lda, ldb, e, kps, ws);
  if (magma_status_t st = check_launch("gemm_f32")) return st;
  if (splits > 1) {
    const int64_t per_row = (N & 3) == 0 ? N / 4 : N;
    int64_t gx = ceil_div(per_row, 256);
    if (gx > 16) gx = 16;
    int64_t gy = (8LL * num_sms() + gx - 1) / gx;
    if (gy > M) gy = M;
    if (gy > 65535) gy = 65535;
    const int vec_c = (e.ldc % 4) == 0 && aligned16(c);
    splitk_reduce<TC><<<dim3((unsigned)gx, (unsigned)gy), 256, 0, s>>>(ws, splits, M, N, C, e,
                                                                       vec_c);
    return check_launch("gemm_f32_splitk_reduce");
  }
  return MAGMA_OK;
}

// ---- F32 contraction on the BF16 tensor cores (three-term split) -----------
// An F32 operand x is split into three BF16 terms, x1 = RN(x), x2 = RN(x -
// x1), x3 = RN(x - x1 - x2) (each difference is exact in F32), which carry 24
// significant bits between them. The product sum_k a b is then formed as the
// six products whose magnitude reaches 2^-16 of a b, a1 b1 + a1 b2 + a2 b1 +
// a1 b3 + a2 b2 + a3 b1 (the dropped terms a2 b3, a3 b2, a3 b3 are below 2^-24
// relative), by one BF16 GEMM over a K six times as long:
//   A' = [a1 | a1 | a2 | a1 | a2 | a3],  B' = [b1 | b2 | b1 | b3 | b2 | b1]
// (each segment Kp = K rounded up to a multiple of 8 columns, zero padded),
// accumulated in F32 by the tensor cores, with the epilogue of the F32 call.
constexpr uint32_t kSplitPatA = (1u << 0) | (1u << 2) | (2u << 4) | (1u << 6) | (2u << 8) | (3u << 10);
constexpr uint32_t kSplitPatB = (1u << 0) | (2u << 2) | (1u << 4) | (3u << 6) | (2u << 8) | (1u << 10);
// below this many multiply-adds the one-pass FFMA kernel is used
constexpr double kBf16x3MinMacs = 134217728.0;

// dst [R][6 Kp] (BF16, row-major) from the F32 matrix element (r, k) =
// src[r * rs + k * ks], r < R, k < Kc (zero for Kc <= k < Kp); segment s of a
// row holds term (pat >> 2s) & 3 of every element. 32 x 32 tiles through
// shared memory, so both the reads (along whichever index is contiguous) and
// the writes (along k) are coalesced.
__global__ void __launch_bounds__(256)
split_bf16x3(const float* __restrict__ src, int64_t R, int64_t Kc, int64_t rs, int64_t ks,
             int64_t Kp, uint32_t pat, __nv_bfloat16* __restrict__ dst) {
  __shared__ float tile[32][33];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int64_t r0 = (int64_t)blockIdx.y * 32, k0 = (int64_t)blockIdx.x * 32;
  const bool kcontig = ks == 1;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int a = ty + 8 * i;
    // (r, k) of this thread's read: consecutive threads along the contiguous index
    const int rl = kcontig ? a : tx, kl = kcontig ? tx : a;
    const int64_t r = r0 + rl, k = k0 + kl;
    tile[rl][kl] = (r < R && k < Kc) ? src[r * rs + k * ks] : 0.f;
  }
  __syncthreads();
  const int64_t ld = 6 * Kp;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int rl = ty + 8 * i;
    const int64_t r = r0 + rl, k = k0 + tx;
    if (r >= R || k >= Kp) continue;
    const float x = tile[rl][tx];
    __nv_bfloat16 t[4];
    t[1] = __float2bfloat16_rn(x);
    const float e1 = __fsub_rn(x, __bfloat162float(t[1]));
    t[2] = __float2bfloat16_rn(e1);
    t[3] = __float2bfloat16_rn(__fsub_rn(e1, __bfloat162float(t[2])));
    __nv_bfloat16* row = dst + r * ld + k;
#pragma unroll
    for (int sgm = 0; sgm < 6; ++sgm) row[sgm * Kp] = t[(pat >> (2 * sgm)) & 3];
  }
}

int64_t bf16x3_kp(int64_t K) { return ceil_div(K, 8) * 8; }

// Workspace of the three-term path: A' and B' (each 256-byte aligned), then
// the split-K partials of the BF16 plan over K' = 6 Kp.
size_t bf16x3_workspace(int64_t M, int64_t N, int64_t K, int epi, TcPlan* plan_out) {
  const int64_t kp = bf16x3_kp(K);
  const size_t a_bytes = ((size_t)M * 6 * kp * 2 + 255) & ~(size_t)255;
  const size_t b_bytes = ((size_t)N * 6 * kp * 2 + 255) & ~(size_t)255;
  const TcPlan plan = choose_plan(M, N, 6 * kp, epi, true);
  if (plan_out) *plan_out = plan;
  const size_t part = plan.splits > 1 ? (size_t)plan.splits * M * N * sizeof(float) : 0;
  return a_bytes + b_bytes + part;
}

bool bf16x3_eligible(int64_t M, int64_t N, int64_t K) {
  return (double)M * (double)N * (double)K >= kBf16x3MinMacs;
}

// op(A) [M x K] . op(B) [K x N] in F32 through the split (ta / tb as in
// magma_gemm), output of type TC with epilogue e. Returns MAGMA_UNAVAILABLE
// (nothing launched) when the workspace is too small, so the caller can take
// the FFMA kernel instead.
template <typename TC>
magma_status_t gemm_f32_bf16x3(const float* a, const float* b, void* c, int64_t M, int64_t N,
                               int64_t K, int64_t lda, int64_t ldb, int ta, int tb,
                               const EpiArgs& e, void* workspace, size_t workspace_bytes,
                               cudaStream_t s) {
  TcPlan plan;
  const size_t need = bf16x3_workspace(M, N, K, e.epi, &plan);
  if (workspace == nullptr || !aligned16(workspace) || workspace_bytes < need ||
      e.epi == MAGMA_EPI_ROWSTATS)
    return MAGMA_UNAVAILABLE;
  const int64_t kp = bf16x3_kp(K), kq = 6 * kp;
  uint8_t* w = static_cast<uint8_t*>(workspace);
  __nv_bfloat16* a2 = reinterpret_cast<__nv_bfloat16*>(w);
  __nv_bfloat16* b2 = reinterpret_cast<__nv_bfloat16*>(
      w + (((size_t)M * kq * 2 + 255) & ~(size_t)255));
  float* part = reinterpret_cast<float*>(
      reinterpret_cast<uint8_t*>(b2) + (((size_t)N * kq * 2 + 255) & ~(size_t)255));
  // op(A)(i, k): A[i*lda + k] (ta = 0) or A[k*lda + i]; op(B)(k, j) taken as
  // B'(j, k): B[j*ldb + k] (tb = 1) or B[k*ldb + j]
  split_bf16x3<<<dim3((unsigned)ceil_div(kp, 32), (unsigned)ceil_div(M, 32)), 256, 0, s>>>(
      a, M, K, ta ? 1 : lda, ta ? lda : 1, kp, kSplitPatA, a2);
  if (magma_status_t st = check_launch("gemm_f32 split A")) return st;
  split_bf16x3<<<dim3((unsigned)ceil_div(kp, 32), (unsigned)ceil_div(N, 32)), 256, 0, s>>>(
      b, N, K, tb ? ldb : 1, tb ? 1 : ldb, kp, kSplitPatB, b2);
  if (magma_status_t st = check_launch("gemm_f32 split B")) return st;
  auto al8 = [](const void* p) { return p == nullptr || (reinterpret_cast<uintptr_t>(p) & 7u) == 0; };
  const int vec_ok = (e.ldc % 2) == 0 && al8(c) && al8(e.aux_in) && al8(e.aux_out);
  const int vec8_ok = (e.ldc % 8) == 0 && aligned16(c);
  const int epi_vec8 = vec8_ok && aligned16(e.aux_in) && aligned16(e.aux_out) && aligned16(e.bias);
  const double a_bytes = 2.0 * (double)M * (double)kq, b_bytes = 2.0 * (double)N * (double)kq;
  const int n_fast = (a_bytes > 64e6 && a_bytes >= b_bytes && N > (plan.pair ? 256 : 128)) ? 1 : 0;
  TcArgs args{M, N, kq, c, e, device_error_word(), vec_ok, vec8_ok, epi_vec8, 0, plan.splits,
              plan.kb_per_split, part, n_fast};
  return dispatch_plan<TC>(plan, a2, b2, M, N, kq, kq, kq, 0, 1, args, s);
}

}  // namespace
}  // namespace magma

using namespace magma;

extern "C" {

size_t magma_gemm_workspace_size(int64_t m, int64_t n, int64_t k, magma_dtype_t ab_dtype) {
  if (m <= 0 || n <= 0 || k <= 0) return 0;
  if (ab_dtype == MAGMA_DTYPE_F32) {
    // the three-term tensor-core path where it applies (largest over the
    // epilogue classes), else the FFMA kernel's split-K partials
    size_t need = simt_workspace(m, n, k);
    if (bf16x3_eligible(m, n, k)) {
      static const int kEpisF[] = {MAGMA_EPI_NONE, MAGMA_EPI_BIAS_RESIDUAL, MAGMA_EPI_BIAS_GELU,
                                   MAGMA_EPI_DGELU};
      for (int epi : kEpisF) {
        const size_t w = bf16x3_workspace(m, n, k, epi, nullptr);
        if (w > need) need = w;
      }
    }
    return need;
  }
  if (ab_dtype != MAGMA_DTYPE_BF16) return 0;
  // The plan depends on the epilogue and output type, which this query does
  // not take: return the largest split workspace over the epilogue classes.
  static const int kEpis[] = {MAGMA_EPI_NONE, MAGMA_EPI_BIAS_RESIDUAL, MAGMA_EPI_BIAS_GELU,
                              MAGMA_EPI_DGELU};
  size_t need = 0;
  for (int epi : kEpis)
    for (int c32 = 0; c32 < 2; ++c32) {
      const TcPlan p = choose_plan(m, n, k, epi, c32 != 0);
      const size_t w = p.splits > 1 ? (size_t)p.splits * (size_t)m * (size_t)n * sizeof(float) : 0;
      if (w > need) need = w;
    }
  return need;
}

magma_status_t magma_gemm(const void* a, const void* b, void* c, int64_t m, int64_t n, int64_t k,
                          int64_t lda, int64_t ldb, int64_t ldc, int32_t trans_a, int32_t trans_b,
                          magma_dtype_t ab_dtype, magma_dtype_t c_dtype, int32_t epilogue,
                          const float* bias, const void* aux_in, void* aux_out, void* workspace,
                          size_t workspace_bytes, void* stream) {
  MAGMA_REQUIRE(m >= 0 && n >= 0 && k >= 0, "magma_gemm: negative size");
  MAGMA_REQUIRE(m < (1LL << 31) && n < (1LL << 31) && k < (1LL << 31),
                "magma_gemm: dimension exceeds 2^31");
  MAGMA_REQUIRE(is_float_dtype(ab_dtype) && is_float_dtype(c_dtype),
                "magma_gemm: unsupported dtypes ab=%s c=%s", dtype_name(ab_dtype),
                dtype_name(c_dtype));
  MAGMA_REQUIRE(epilogue >= MAGMA_EPI_NONE && epilogue <= MAGMA_EPI_ROWSTATS,
                "magma_gemm: unknown epilogue %d", epilogue);
  MAGMA_REQUIRE(epilogue != MAGMA_EPI_ROWSTATS || (aux_out != nullptr && ab_dtype == MAGMA_DTYPE_BF16 &&
                                                   (reinterpret_cast<uintptr_t>(aux_out) & 7u) == 0),
                "magma_gemm: ROWSTATS needs BF16 operands and an 8-byte aligned aux_out");
  MAGMA_REQUIRE(lda >= (trans_a ? m : k) && ldb >= (trans_b ? k : n) && ldc >= n,
                "magma_gemm: leading dimensions too small (lda=%lld ldb=%lld ldc=%lld)",
                (long long)lda, (long long)ldb, (long long)ldc);
  if (m == 0 || n == 0) return MAGMA_OK;
  MAGMA_REQUIRE(c != nullptr && (k == 0 || (a != nullptr && b != nullptr)),
                "magma_gemm: NULL operand");
  MAGMA_REQUIRE(epilogue != MAGMA_EPI_ACCUMULATE || c_dtype == MAGMA_DTYPE_F32,
                "magma_gemm: ACCUMULATE needs an F32 output");
  MAGMA_REQUIRE(epilogue != MAGMA_EPI_BIAS_RESIDUAL || aux_in != nullptr,
                "magma_gemm: BIAS_RESIDUAL needs aux_in (F32 residual)");
  MAGMA_REQUIRE((epilogue != MAGMA_EPI_DGELU && epilogue != MAGMA_EPI_DRELU) || aux_in != nullptr,
                "magma_gemm: activation VJP epilogue needs aux_in (pre-activation)");
  MAGMA_REQUIRE((epilogue != MAGMA_EPI_BIAS_GELU && epilogue != MAGMA_EPI_BIAS_RELU) ||
                    aux_out != nullptr,
                "magma_gemm: activation epilogue needs aux_out for the pre-activation");
  cudaStream_t s = (cudaStream_t)stream;
  EpiArgs e{epilogue, bias, aux_in, aux_out, ldc};
  const bool c32 = c_dtype == MAGMA_DTYPE_F32;

  const bool tc_ok = ab_dtype == MAGMA_DTYPE_BF16 && k > 0 && aligned16(a) && aligned16(b) &&
                     (lda % 8) == 0 && (ldb % 8) == 0;
  if (tc_ok) {
    auto al8 = [](const void* p) { return p == nullptr || (reinterpret_cast<uintptr_t>(p) & 7u) == 0; };
    const int vec_ok = (ldc % 2) == 0 && al8(c) && al8(aux_in) && al8(aux_out);
    TcPlan plan = choose_plan(m, n, k, epilogue, c32);
    // Split-K only with a large enough caller workspace; otherwise one pass.
    const size_t need = plan.splits > 1 ? (size_t)plan.splits * m * n * sizeof(float) : 0;
    if (plan.splits > 1 && (workspace == nullptr || workspace_bytes < need || !aligned16(workspace) ||
                            epilogue == MAGMA_EPI_ROWSTATS))
      plan = {plan.bn, 1, (int)ceil_div(k, kBK), plan.pair};
    const int vec8_ok = (ldc % 8) == 0 && aligned16(c);
    // A larger than L2 and several N tiles: walk N fastest so the CTAs that
    // share an A block run together and it is read from HBM once.
    const double a_bytes = 2.0 * (double)m * (double)k, b_bytes = 2.0 * (double)n * (double)k;
    const int n_fast = (a_bytes > 64e6 && a_bytes >= b_bytes && n > (plan.pair ? 256 : 128)) ? 1 : 0;
    const int epi_vec8 = vec8_ok && aligned16(aux_in) && aligned16(aux_out) && aligned16(bias);
    TcArgs args{m, n, k, c, e, device_error_word(), vec_ok, vec8_ok, epi_vec8, 0, plan.splits,
                plan.kb_per_split, static_cast<float*>(workspace), n_fast};
    return c32 ? dispatch_plan<float>(plan, a, b, m, n, k, lda, ldb, trans_a, trans_b, args, s)
               : dispatch_plan<__nv_bfloat16>(plan, a, b, m, n, k, lda, ldb, trans_a, trans_b,
                                              args, s);
  }
  MAGMA_REQUIRE(epilogue != MAGMA_EPI_ROWSTATS,
                "magma_gemm: ROWSTATS needs the tensor-core path (16-byte aligned operands, "
                "lda and ldb multiples of 8)");
  if (ab_dtype == MAGMA_DTYPE_F32 && k > 0 && bf16x3_eligible(m, n, k)) {
    // F32-accurate contraction on the tensor cores (three-term BF16 split);
    // falls through to the FFMA kernel when the workspace is too small
    const magma_status_t st =
        c32 ? gemm_f32_bf16x3<float>(static_cast<const float*>(a), static_cast<const float*>(b), c,
                                     m, n, k, lda, ldb, trans_a, trans_b, e, workspace,
                                     workspace_bytes, s)
            : gemm_f32_bf16x3<__nv_bfloat16>(static_cast<const float*>(a),
                                             static_cast<const float*>(b), c, m, n, k, lda, ldb,
                                             trans_a, trans_b, e, workspace, workspace_bytes, s);
    if (st != MAGMA_UNAVAILABLE) return st;
  }
  if (ab_dtype == MAGMA_DTYPE_F32)
    return c32 ? launch_simt<float, float>(a, b, c, m, n, k, lda, ldb, trans_a, trans_b, e,
                                           workspace, workspace_bytes, s)
               : launch_simt<float, __nv_bfloat16>(a, b, c, m, n, k, lda, ldb, trans_a, trans_b,
                                                   e, workspace, workspace_bytes, s);
  return c32 ? launch_simt<__nv_bfloat16, float>(a, b, c, m, n, k, lda, ldb, trans_a, trans_b, e,
                                                 workspace, workspace_bytes, s)
             : launch_simt<__nv_bfloat16, __nv_bfloat16>(a, b, c, m, n, k, lda, ldb, trans_a,
                                                         trans_b, e, workspace, workspace_bytes,
                                                         s);
}

}  // extern "C"
