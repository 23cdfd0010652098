// Causal attention on the tcgen05 tensor cores (BF16 in, F32 accumulate),
// head_dim 64. Same math as the SIMT path (GPT block attention,
// Benchmarks/GPT2Shakespeare/Sources/main.swift:467-481; VJP chain
// Sources/Core/Autodiff.swift:309-317,379-386), tiled 128 x 128.
//
// Kernels (each with a TMA producer warp over 4-D tensor maps straight on the
// caller's strided [B, H, S, D] views — Q/K/V are read in place from the fused
// QKV projection, no head transposes — and one warp that allocates TMEM and
// issues the tcgen05.mma from a single thread; score tiles and accumulators
// live in TMEM):
//   attn_fwd_tc    one CTA per pair of 128-query tiles, two softmax warpgroups
//                  (thread = query row) taking turns on the exponentials;
//                  S_t = Q_t K_j^T in TMEM, P_t written back over S_t as BF16
//                  and used from TMEM as the A operand of O_t += P_t V_j;
//                  outputs O (BF16) and the row log-sum-exp.
//   attn_delta_tc  delta = rowsum(dO * O) for the softmax VJP.
//   attn_bwd_tc    one CTA per 128-key tile looping over its query tiles:
//                  S^T = K Q^T, dP^T = V dO^T, P^T = exp(S^T*scale - lse),
//                  dS^T = P^T (dP^T - delta); dV += P^T dO, dK += dS^T Q (TMEM
//                  accumulators, P^T / dS^T as TMEM A operands), dQ_ij = dS K_j
//                  drained as an F32 partial tile.
//   attn_dq_reduce sums the dQ partials over key tiles in a fixed order
//                  (deterministic, no atomics).
//   attn_bwd_dkdv_tc / attn_bwd_dq_tc  two-pass backward for workspaces too
//                  small for the partial tiles.
// All mbarrier waits are bounded (they set the device error word and the
// kernel winds down instead of hanging).
#include <cuda.h>

#include <type_traits>

#include "common.cuh"
#include "sm100.cuh"

namespace magma {

namespace {

using namespace sm100;

constexpr int kTile = 128;     // queries / keys per tile
constexpr int kHd = 64;        // head dim
constexpr int kThreads = 192;  // 4 row warps + producer + MMA
constexpr int kTileBytes = kTile * kHd * 2;  // 16 KB: one [128 x 64] BF16 tile
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

struct AttnTcArgs {
  int S, H, B;
  float scale;
  int causal;
  void* o;         // fwd output / bwd: unused
  float* lse;
  const float* delta;
  void* dq;        // dQ / dK / dV outputs (qkv strides)
  void* dk;
  void* dv;
  int64_t os0, os1, os2;  // O strides (elements)
  int64_t qs0, qs1, qs2;  // Q/K/V (and dQ/dK/dV) strides
  int* err;
};

__device__ __forceinline__ uint64_t desc_k(uint32_t addr) { return smem_desc_sw128(addr, 16, 1024); }
__device__ __forceinline__ uint64_t desc_mn(uint32_t addr) {
  return smem_desc_sw128(addr, 8192, 1024);
}

// Address in a [128 rows x 128 cols] BF16 K-major SW128 operand (two 64-column
// blocks of 16 KB) of the 16-byte chunk holding columns [8*chunk, 8*chunk+8)
// of row r.
__device__ __forceinline__ uint32_t swz_chunk_addr(uint32_t base, int r, int chunk) {
  const int blk = chunk >> 3, c = chunk & 7;
  return base + blk * 16384 + r * 128 + ((c ^ (r & 7)) << 4);
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Writes 32 F32 values as BF16 columns [32*c32, 32*c32+32) of row r.
__device__ __forceinline__ void store_row32(uint32_t base, int r, int c32, const float (&v)[32]) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int chunk = c32 * 4 + q;
    st_shared_v4(swz_chunk_addr(base, r, chunk), pack_bf16(v[q * 8 + 0], v[q * 8 + 1]),
                 pack_bf16(v[q * 8 + 2], v[q * 8 + 3]), pack_bf16(v[q * 8 + 4], v[q * 8 + 5]),
                 pack_bf16(v[q * 8 + 6], v[q * 8 + 7]));
  }
}

// Stores 64 F32 values * mul as one BF16 row of 128 bytes.
__device__ __forceinline__ void store_global_row64(__nv_bfloat16* dst, const float* v, float mul) {
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    uint4 u;
    u.x = pack_bf16(v[q * 8 + 0] * mul, v[q * 8 + 1] * mul);
    u.y = pack_bf16(v[q * 8 + 2] * mul, v[q * 8 + 3] * mul);
    u.z = pack_bf16(v[q * 8 + 4] * mul, v[q * 8 + 5] * mul);
    u.w = pack_bf16(v[q * 8 + 6] * mul, v[q * 8 + 7] * mul);
    reinterpret_cast<uint4*>(dst)[q] = u;
  }
}

__device__ __forceinline__ uint32_t align1024(uint8_t* raw, uint8_t** aligned_ptr) {
  const uint32_t a = smem_u32(raw);
  const uint32_t base = (a + 1023u) & ~1023u;
  *aligned_ptr = raw + (base - a);
  return base;
}

// =============================================================== forward
// One CTA per pair of 128-query tiles (t = 0, 1: query rows q0 .. q0+255),
// heaviest causal pairs first. Warps 0-3 run the softmax of tile 0, warps 4-7
// that of tile 1, warp 8 is the TMA producer, warp 9 allocates TMEM and issues
// the MMAs. Both tiles stream the same K/V tiles, so while one warpgroup
// turns S_t into P_t the tensor cores work on the other tile:
//   MMA order: S0(0) S1(0) | PV0(0) S0(1) PV1(0) S1(1) | PV0(1) S0(2) ...
// TMEM: S_t at columns 128t (F32 128x128); P_t is written back as BF16 over
// the first 64 columns of S_t and is the A operand of PV_t = P_t V_j, which
// accumulates into O_t at columns 256 + 64t. tcgen05.mma executes in issue
// order, so S_t(j+1), issued after PV_t(j), cannot overwrite P_t(j) early, and
// the commit that reports S_t(j+1) done also covers PV_t(j). O_t and the row
// sum are rescaled only when a row maximum grows by more than 2^8 (otherwise
// the stale maximum is kept: P <= 2^8, exact after the final division).
constexpr int kFwdStages = 3;
constexpr int kFwdThreads = 320;                 // 8 softmax warps + producer + MMA
constexpr int kFwdQ = 0;                         // Q tiles 0, 1 (2 x 16 KB)
constexpr int kFwdKv = 2 * kTileBytes;           // K, V per stage
constexpr int kFwdBar = kFwdKv + kFwdStages * 2 * kTileBytes;
// q_full, kv_full[3], kv_empty[3], s_full[2], p_full[2], pv_done[2], done
constexpr int kFwdNumBars = 14;
constexpr int kFwdSmem = kFwdBar + kFwdNumBars * 8 + 16 + 1024;
constexpr float kRescaleLog2 = 8.0f;

__global__ void __launch_bounds__(kFwdThreads, 1)
attn_fwd_tc(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
            const __grid_constant__ CUtensorMap tmV, AttnTcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sp;
  const uint32_t base = align1024(smem_raw, &sp);
  auto sQ = [&](int t) { return base + kFwdQ + t * kTileBytes; };
  auto sK = [&](int st) { return base + kFwdKv + st * 2 * kTileBytes; };
  auto sV = [&](int st) { return base + kFwdKv + st * 2 * kTileBytes + kTileBytes; };
  const uint32_t bars = base + kFwdBar;
  const uint32_t q_full = bars;
  auto kv_full = [&](int st) { return bars + 8u * (1 + st); };
  auto kv_empty = [&](int st) { return bars + 8u * (4 + st); };
  auto s_full = [&](int t) { return bars + 8u * (7 + t); };
  auto p_full = [&](int t) { return bars + 8u * (9 + t); };
  auto pv_done = [&](int t) { return bars + 8u * (11 + t); };
  const uint32_t done_bar = bars + 8u * 13;
  const uint32_t tslot = bars + 8u * kFwdNumBars;
  uint32_t* tslot_ptr = reinterpret_cast<uint32_t*>(sp + kFwdBar + 8 * kFwdNumBars);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_qt = (a.S + kTile - 1) / kTile;
  const int n_pairs = (n_qt + 1) / 2;
  // Blocks are dispatched in linear index order; the pair index varies
  // slowest so that every head's heaviest pair (most key tiles under causal)
  // starts first and the lightest ones fill the tail.
  const int lin = (int)(blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z));
  const int heads = (int)(gridDim.y * gridDim.z);
  const int qt0 = 2 * (n_pairs - 1 - lin / heads);
  const bool has1 = qt0 + 1 < n_qt;
  const int h = (lin % heads) % (int)gridDim.y, b = (lin % heads) / (int)gridDim.y;
  // key tiles visited by query tile t
  const int nk0 = a.causal ? qt0 + 1 : n_qt;
  const int nk1 = has1 ? (a.causal ? qt0 + 2 : n_qt) : 0;
  const int n_kv = nk0 > nk1 ? nk0 : nk1;

  if (threadIdx.x == 0) {
    prefetch_tensormap(&tmQ);
    prefetch_tensormap(&tmK);
    prefetch_tensormap(&tmV);
    mbar_init(q_full, 1);
    for (int st = 0; st < kFwdStages; ++st) {
      mbar_init(kv_full(st), 1);
      mbar_init(kv_empty(st), 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(s_full(t), 1);
      mbar_init(p_full(t), 4);
      mbar_init(pv_done(t), 1);
    }
    mbar_init(done_bar, 1);
    fence_barrier_init();
  }
  if (warp == 9) tmem_alloc(tslot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tslot_ptr);
  auto tS = [&](int t) { return tmem + (uint32_t)(t * kTile); };
  auto tO = [&](int t) { return tmem + 256u + (uint32_t)(t * kHd); };

  if (warp == 8) {
    if (lane == 0) {
      bool ok = true;
      mbar_expect_tx(q_full, (has1 ? 2 : 1) * kTileBytes);
      tma_load_4d(sQ(0), &tmQ, 0, qt0 * kTile, h, b, q_full);
      if (has1) tma_load_4d(sQ(1), &tmQ, 0, (qt0 + 1) * kTile, h, b, q_full);
      for (int j = 0; j < n_kv && ok; ++j) {
        const int st = j % kFwdStages;
        if (!mbar_wait(kv_empty(st), (uint32_t)(((j / kFwdStages) & 1) ^ 1), a.err)) {
          ok = false;
          break;
        }
        mbar_expect_tx(kv_full(st), 2 * kTileBytes);
        tma_load_4d(sK(st), &tmK, 0, j * kTile, h, b, kv_full(st));
        tma_load_4d(sV(st), &tmV, 0, j * kTile, h, b, kv_full(st));
      }
      // every stage issued above has been consumed before the producer leaves
      for (int j = n_kv; j < n_kv + kFwdStages && ok; ++j) {
        const int st = j % kFwdStages;
        if (!mbar_wait(kv_empty(st), (uint32_t)(((j / kFwdStages) & 1) ^ 1), a.err)) ok = false;
      }
    }
  } else if (warp == 9) {
    if (lane == 0) {
      constexpr uint32_t idS = idesc_bf16_f32(kTile, kTile, 0, 0);
      constexpr uint32_t idPV = idesc_bf16_f32(kTile, kHd, 0, 1);
      bool ok = mbar_wait(q_full, 0, a.err);
      int kv_ready = -1;  // highest key tile whose K/V have been waited for
      auto wait_kv = [&](int j) -> bool {
        if (j <= kv_ready) return true;
        kv_ready = j;
        if (!mbar_wait(kv_full(j % kFwdStages), (uint32_t)((j / kFwdStages) & 1), a.err))
          return false;
        tc_fence_after();
        return true;
      };
      auto issue_s = [&](int t, int j) {
        const int st = j % kFwdStages;
#pragma unroll
        for (int kk = 0; kk < kHd / 16; ++kk)
          mma_bf16_ss(tS(t), desc_k(sQ(t) + kk * 32), desc_k(sK(st) + kk * 32), idS,
                      kk > 0 ? 1u : 0u);
        mma_commit(s_full(t));
      };
      auto issue_pv = [&](int t, int j) -> bool {
        if (!mbar_wait(p_full(t), (uint32_t)(j & 1), a.err)) return false;
        tc_fence_after();
        const int st = j % kFwdStages;
#pragma unroll
        for (int kk = 0; kk < kTile / 16; ++kk)
          mma_bf16_ts(tO(t), tS(t) + kk * 8, desc_mn(sV(st) + kk * 2048), idPV,
                      (j > 0 || kk > 0) ? 1u : 0u);
        mma_commit(pv_done(t));
        return true;
      };
      if (ok && n_kv > 0) {
        ok = wait_kv(0);
        if (ok) {
          issue_s(0, 0);
          if (nk1 > 0) issue_s(1, 0);
        }
      }
      for (int j = 0; j < n_kv && ok; ++j) {
        for (int t = 0; t < 2 && ok; ++t) {
          const int nk = t ? nk1 : nk0;
          if (j >= nk) continue;
          if (!issue_pv(t, j)) { ok = false; break; }
          if (j + 1 < nk) {
            if (!wait_kv(j + 1)) { ok = false; break; }
            issue_s(t, j + 1);
          }
        }
        if (ok) mma_commit(kv_empty(j % kFwdStages));
      }
      mma_commit(done_bar);
      mbar_wait(done_bar, 0, a.err);
    }
  } else {
    // ---------------------------- softmax warpgroups ----------------------------
    const int t = warp >> 2;
    const int nk = t ? nk1 : nk0;
    const int qt = qt0 + t;
    const int r = (warp & 3) * 32 + lane;
    const int qg = qt * kTile + r;
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t srow = tS(t) + lane_off;
    const uint32_t orow = tO(t) + lane_off;
    const float sl2 = a.scale * kLog2e;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    // The two warpgroups take turns on the exponential pass (MUFU is the
    // bottleneck unit): tile 0 step j, tile 1 step j, tile 0 step j+1, ...
    // Named barrier 1 + t hands the turn to warpgroup t. A warpgroup that hit
    // a wait limit keeps the turn protocol (skipping its work) so the other
    // one is never left at a named barrier.
    const int nk_other = t ? nk0 : nk1;
    for (int j = 0; j < nk; ++j) {
      // waits for the other warpgroup's step j-1 (t = 0) or step j (t = 1)
      const bool wait_turn = t ? (j < nk_other) : (j >= 1 && j - 1 < nk_other);
      // hands over after step j to its step j (t = 0) or step j+1 (t = 1)
      const bool give_turn = t ? (j + 1 < nk_other) : (j < nk_other);
      const int k0 = j * kTile;
      // Only the diagonal tile (causal) and a ragged last tile need masking;
      // every other tile takes the mask-free path (warp-uniform branch).
      const bool diag = a.causal && j == qt;
      const bool tail = k0 + kTile > a.S;
      const bool masked_tile = diag || tail;
      int lim = 127;  // last unmasked column of this row
      if (diag) lim = qg - k0;
      if (tail && a.S - 1 - k0 < lim) lim = a.S - 1 - k0;
      if (ok && !mbar_wait(s_full(t), (uint32_t)(j & 1), a.err)) ok = false;
      ok = __all_sync(0xffffffffu, ok);  // warp-uniform for the collective TMEM ops
      if (ok) {
        tc_fence_after();
        // pass 1: row maximum (S read from TMEM in two 64-column halves; eight
        // independent max chains)
        float mx8[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) mx8[i] = -INFINITY;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          uint32_t v[2][32];
          tmem_ld32(srow + hh * 64, v[0]);
          tmem_ld32(srow + hh * 64 + 32, v[1]);
          tmem_wait_ld();
          if (!masked_tile) {
#pragma unroll
            for (int e = 0; e < 64; ++e)
              mx8[e & 7] = fmaxf(mx8[e & 7], __uint_as_float(v[e >> 5][e & 31]));
          } else {
#pragma unroll
            for (int e = 0; e < 64; ++e)
              if (hh * 64 + e <= lim)
                mx8[e & 7] = fmaxf(mx8[e & 7], __uint_as_float(v[e >> 5][e & 31]));
          }
        }
        const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                               fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
        const float m_new = fmaxf(m_run, mx * sl2);
        if (j == 0) {
          m_run = m_new == -INFINITY ? 0.f : m_new;
        } else if (__any_sync(0xffffffffu, m_new > m_run + kRescaleLog2)) {
          // O_t holds PV_t(0 .. j-1) (complete: covered by the S_t(j) commit).
          const float alpha = ex2_approx(m_run - m_new);
          m_run = m_new;
          l_run *= alpha;
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            uint32_t o[32];
            tmem_ld32(orow + half * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int c = 0; c < 32; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
            tmem_st32(orow + half * 32, o);
          }
          tmem_wait_st();
        }
      }
      // pass 2: P = exp2(S * scale * log2(e) - m), written back over S as
      // BF16. The first half of the row is read from TMEM before the turn
      // starts, the second half while the first is exponentiated; the turn is
      // handed on as soon as the last exponential is issued.
      uint32_t va[2][32];
      if (ok) {
        tmem_ld32(srow, va[0]);
        tmem_ld32(srow + 32, va[1]);
        tmem_wait_ld();
      }
      if (wait_turn) named_barrier(1 + t, 256);
      if (ok) {
        float rs4[4] = {0.f, 0.f, 0.f, 0.f};
        // Exponentiates 32 columns starting at column c of S (v) into 16
        // packed BF16 pairs stored over BF16 columns [c/2, c/2 + 16) (S
        // columns already read).
        auto exp32 = [&](const uint32_t (&v)[32], int c) {
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            float p0 = ex2_approx(fmaf(__uint_as_float(v[2 * e]), sl2, -m_run));
            float p1 = ex2_approx(fmaf(__uint_as_float(v[2 * e + 1]), sl2, -m_run));
            if (masked_tile) {
              if (c + 2 * e > lim) p0 = 0.f;
              if (c + 2 * e + 1 > lim) p1 = 0.f;
            }
            rs4[e & 3] += p0 + p1;
            pk[e] = pack_bf16(p0, p1);
          }
          tmem_st16(srow + c / 2, pk);
        };
        uint32_t vb[32];
        tmem_ld32(srow + 64, vb);  // lands while columns 0-63 are exponentiated
        exp32(va[0], 0);
        exp32(va[1], 32);
        tmem_wait_ld();
        uint32_t vc[32];
        tmem_ld32(srow + 96, vc);
        exp32(vb, 64);
        tmem_wait_ld();
        exp32(vc, 96);
        if (give_turn) named_barrier_arrive(2 - t, 256);
        l_run += (rs4[0] + rs4[1]) + (rs4[2] + rs4[3]);
        tmem_wait_st();
      } else if (give_turn) {
        named_barrier_arrive(2 - t, 256);
      }
      if (ok) {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(p_full(t));
      }
    }
    if (ok && nk > 0 && !mbar_wait(pv_done(t), (uint32_t)((nk - 1) & 1), a.err)) ok = false;
    ok = __all_sync(0xffffffffu, ok);
    if (ok && nk > 0) {
      tc_fence_after();
      uint32_t o0[32], o1[32];
      tmem_ld32(orow, o0);
      tmem_ld32(orow + 32, o1);
      tmem_wait_ld();
      if (qg < a.S) {
        float of[kHd];
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          of[c] = __uint_as_float(o0[c]);
          of[32 + c] = __uint_as_float(o1[c]);
        }
        const float inv = 1.0f / l_run;
        __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(a.o) + (int64_t)b * a.os0 +
                             (int64_t)h * a.os1 + (int64_t)qg * a.os2;
        store_global_row64(dst, of, inv);
        if (a.lse != nullptr)
          a.lse[((int64_t)b * a.H + h) * a.S + qg] = m_run * kLn2 + logf(l_run);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ========================================================== backward dK/dV
constexpr int kKvK = 0;
constexpr int kKvV = kTileBytes;
constexpr int kKvQdo = 2 * kTileBytes;                       // 2 stages x (Q, dO)
constexpr int kKvPT = kKvQdo + 2 * 2 * kTileBytes;           // 32 KB
constexpr int kKvDST = kKvPT + 2 * kTileBytes;               // 32 KB
constexpr int kKvStats = kKvDST + 2 * kTileBytes;            // lse[2][128], delta[2][128]
constexpr int kKvBar = kKvStats + 4 * kTile * 4;
// kv_full, qdo_full[2], qdo_empty[2], st_full, pds_full, final
constexpr int kKvNumBars = 8;
constexpr int kKvSmem = kKvBar + kKvNumBars * 8 + 16 + 1024;

__global__ void __launch_bounds__(kThreads, 1)
attn_bwd_dkdv_tc(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                 const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO,
                 AttnTcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sp;
  const uint32_t base = align1024(smem_raw, &sp);
  const uint32_t sK = base + kKvK, sV = base + kKvV;
  auto sQ = [&](int st) { return base + kKvQdo + st * 2 * kTileBytes; };
  auto sdO = [&](int st) { return base + kKvQdo + st * 2 * kTileBytes + kTileBytes; };
  const uint32_t sPT = base + kKvPT, sDST = base + kKvDST;
  float* lse_s = reinterpret_cast<float*>(sp + kKvStats);           // [2][128]
  float* delta_s = reinterpret_cast<float*>(sp + kKvStats + 2 * kTile * 4);
  const uint32_t bars = base + kKvBar;
  const uint32_t kv_full = bars;
  auto qdo_full = [&](int s) { return bars + 8u * (1 + s); };
  auto qdo_empty = [&](int s) { return bars + 8u * (3 + s); };
  const uint32_t st_full = bars + 8u * 5;
  const uint32_t pds_full = bars + 8u * 6;
  const uint32_t final_bar = bars + 8u * 7;
  const uint32_t tslot = bars + 8u * kKvNumBars;
  uint32_t* tslot_ptr = reinterpret_cast<uint32_t*>(sp + kKvBar + 8 * kKvNumBars);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_t = (a.S + kTile - 1) / kTile;
  // Linear dispatch order with the key tile varying slowest: key tile 0 has
  // the most query tiles under causal, so the heaviest blocks start first and
  // the lightest fill the tail.
  const int lin = (int)(blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z));
  const int heads = (int)(gridDim.y * gridDim.z);
  const int kt = lin / heads;
  const int h = (lin % heads) % (int)gridDim.y, b = (lin % heads) / (int)gridDim.y;
  const int k0 = kt * kTile;
  const int first_q = a.causal ? kt : 0;
  const int n_it = n_t - first_q;

  if (threadIdx.x == 0) {
    prefetch_tensormap(&tmQ);
    prefetch_tensormap(&tmK);
    prefetch_tensormap(&tmV);
    prefetch_tensormap(&tmdO);
    mbar_init(kv_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(qdo_full(s), 1);
      mbar_init(qdo_empty(s), 1);
    }
    mbar_init(st_full, 1);
    mbar_init(pds_full, 4);
    mbar_init(final_bar, 1);
    fence_barrier_init();
  }
  if (warp == 5) tmem_alloc(tslot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tslot_ptr);
  const uint32_t tST = tmem, tDPT = tmem + 128, tDV = tmem + 256, tDK = tmem + 320;

  if (warp == 4) {
    if (lane == 0) {
      bool ok = true;
      mbar_expect_tx(kv_full, 2 * kTileBytes);
      tma_load_4d(sK, &tmK, 0, k0, h, b, kv_full);
      tma_load_4d(sV, &tmV, 0, k0, h, b, kv_full);
      for (int i = 0; i < n_it && ok; ++i) {
        const int st = i & 1;
        const int q0 = (first_q + i) * kTile;
        if (!mbar_wait(qdo_empty(st), (uint32_t)(((i >> 1) & 1) ^ 1), a.err)) { ok = false; break; }
        mbar_expect_tx(qdo_full(st), 2 * kTileBytes);
        tma_load_4d(sQ(st), &tmQ, 0, q0, h, b, qdo_full(st));
        tma_load_4d(sdO(st), &tmdO, 0, q0, h, b, qdo_full(st));
      }
      for (int i = n_it; i < n_it + 2 && ok; ++i) {
        const int st = i & 1;
        if (!mbar_wait(qdo_empty(st), (uint32_t)(((i >> 1) & 1) ^ 1), a.err)) ok = false;
      }
    }
  } else if (warp == 5) {
    if (lane == 0) {
      constexpr uint32_t idS = idesc_bf16_f32(kTile, kTile, 0, 0);
      constexpr uint32_t idG = idesc_bf16_f32(kTile, kHd, 0, 1);
      bool ok = mbar_wait(kv_full, 0, a.err);
      auto issue_grad = [&](int i) -> bool {
        const int st = i & 1;
        if (!mbar_wait(pds_full, (uint32_t)(i & 1), a.err)) return false;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kTile / 16; ++kk) {
          const uint32_t aoff = (kk >> 2) * 16384 + (kk & 3) * 32;
          mma_bf16_ss(tDV, desc_k(sPT + aoff), desc_mn(sdO(st) + kk * 2048), idG,
                      (i > 0 || kk > 0) ? 1u : 0u);
          mma_bf16_ss(tDK, desc_k(sDST + aoff), desc_mn(sQ(st) + kk * 2048), idG,
                      (i > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(qdo_empty(st));
        return true;
      };
      for (int i = 0; i < n_it && ok; ++i) {
        const int st = i & 1;
        if (!mbar_wait(qdo_full(st), (uint32_t)((i >> 1) & 1), a.err)) { ok = false; break; }
        tc_fence_after();
        if (i > 0 && !issue_grad(i - 1)) { ok = false; break; }
#pragma unroll
        for (int kk = 0; kk < kHd / 16; ++kk) {
          mma_bf16_ss(tST, desc_k(sK + kk * 32), desc_k(sQ(st) + kk * 32), idS, kk > 0 ? 1u : 0u);
          mma_bf16_ss(tDPT, desc_k(sV + kk * 32), desc_k(sdO(st) + kk * 32), idS,
                      kk > 0 ? 1u : 0u);
        }
        mma_commit(st_full);
      }
      if (ok && n_it >= 1) issue_grad(n_it - 1);
      mma_commit(final_bar);
      mbar_wait(final_bar, 0, a.err);
    }
  } else {
    // row threads: r = key row
    const int r = warp * 32 + lane;
    const int kg = k0 + r;
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    const float sl2 = a.scale * kLog2e;
    const int64_t bh = (int64_t)b * a.H + h;
    bool ok = true;
    for (int i = 0; i < n_it; ++i) {
      const int st = i & 1;
      const int q0 = (first_q + i) * kTile;
      {
        const int qi = q0 + r;
        lse_s[st * kTile + r] = qi < a.S ? a.lse[bh * a.S + qi] * kLog2e : INFINITY;
        delta_s[st * kTile + r] = qi < a.S ? a.delta[bh * a.S + qi] : 0.f;
      }
      named_barrier(1, 128);
      if (!mbar_wait(st_full, (uint32_t)(i & 1), a.err)) { ok = false; break; }
      tc_fence_after();
      const bool diag = a.causal && (q0 < k0 + kTile);
      const bool tail = q0 + kTile > a.S || k0 + kTile > a.S;
      const bool masked_tile = diag || tail;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t vs[32], vd[32];
        tmem_ld32(tST + lane_off + c * 32, vs);
        tmem_ld32(tDPT + lane_off + c * 32, vd);
        float ls[32], dl[32];
        const float4* l4 = reinterpret_cast<const float4*>(lse_s + st * kTile + c * 32);
        const float4* d4 = reinterpret_cast<const float4*>(delta_s + st * kTile + c * 32);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float4 lv = l4[j], dv4 = d4[j];
          ls[4 * j] = lv.x; ls[4 * j + 1] = lv.y; ls[4 * j + 2] = lv.z; ls[4 * j + 3] = lv.w;
          dl[4 * j] = dv4.x; dl[4 * j + 1] = dv4.y; dl[4 * j + 2] = dv4.z; dl[4 * j + 3] = dv4.w;
        }
        tmem_wait_ld();
        float p[32], ds[32];
        if (!masked_tile) {
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const float pe = ex2_approx(fmaf(__uint_as_float(vs[e]), sl2, -ls[e]));
            p[e] = pe;
            ds[e] = pe * (__uint_as_float(vd[e]) - dl[e]);
          }
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const int qg = q0 + c * 32 + e;
            const bool masked = (diag && qg < kg) || (tail && (qg >= a.S || kg >= a.S));
            const float pe = masked ? 0.f : ex2_approx(fmaf(__uint_as_float(vs[e]), sl2, -ls[e]));
            p[e] = pe;
            ds[e] = pe * (__uint_as_float(vd[e]) - dl[e]);
          }
        }
        store_row32(sPT, r, c, p);
        store_row32(sDST, r, c, ds);
      }
      tc_fence_before();
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(pds_full);
    }
    if (ok && mbar_wait(final_bar, 0, a.err)) {
      tc_fence_after();
      float acc[kHd];
      uint32_t v0[32], v1[32];
      tmem_ld32(tDV + lane_off, v0);
      tmem_ld32(tDV + lane_off + 32, v1);
      tmem_wait_ld();
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        acc[c] = __uint_as_float(v0[c]);
        acc[32 + c] = __uint_as_float(v1[c]);
      }
      const int64_t off = (int64_t)b * a.qs0 + (int64_t)h * a.qs1 + (int64_t)kg * a.qs2;
      if (kg < a.S) store_global_row64(static_cast<__nv_bfloat16*>(a.dv) + off, acc, 1.f);
      tmem_ld32(tDK + lane_off, v0);
      tmem_ld32(tDK + lane_off + 32, v1);
      tmem_wait_ld();
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        acc[c] = __uint_as_float(v0[c]);
        acc[32 + c] = __uint_as_float(v1[c]);
      }
      if (kg < a.S) store_global_row64(static_cast<__nv_bfloat16*>(a.dk) + off, acc, a.scale);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ============================================================= backward dQ
constexpr int kDqQ = 0;
constexpr int kDqDo = kTileBytes;
constexpr int kDqKv = 2 * kTileBytes;                    // 2 stages x (K, V)
constexpr int kDqDs = kDqKv + 2 * 2 * kTileBytes;        // 32 KB
constexpr int kDqBar = kDqDs + 2 * kTileBytes;
// q_full, kv_full[2], kv_empty[2], s_full, ds_full, final
constexpr int kDqNumBars = 8;
constexpr int kDqSmem = kDqBar + kDqNumBars * 8 + 16 + 1024;

__global__ void __launch_bounds__(kThreads, 1)
attn_bwd_dq_tc(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
               const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO,
               AttnTcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sp;
  const uint32_t base = align1024(smem_raw, &sp);
  const uint32_t sQ = base + kDqQ, sdO = base + kDqDo;
  auto sK = [&](int st) { return base + kDqKv + st * 2 * kTileBytes; };
  auto sV = [&](int st) { return base + kDqKv + st * 2 * kTileBytes + kTileBytes; };
  const uint32_t sDS = base + kDqDs;
  const uint32_t bars = base + kDqBar;
  const uint32_t q_full = bars;
  auto kv_full = [&](int s) { return bars + 8u * (1 + s); };
  auto kv_empty = [&](int s) { return bars + 8u * (3 + s); };
  const uint32_t s_full = bars + 8u * 5;
  const uint32_t ds_full = bars + 8u * 6;
  const uint32_t final_bar = bars + 8u * 7;
  const uint32_t tslot = bars + 8u * kDqNumBars;
  uint32_t* tslot_ptr = reinterpret_cast<uint32_t*>(sp + kDqBar + 8 * kDqNumBars);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_t = (a.S + kTile - 1) / kTile;
  const int qt = n_t - 1 - (int)blockIdx.x;
  const int h = blockIdx.y, b = blockIdx.z;
  const int q0 = qt * kTile;
  const int n_kv = a.causal ? qt + 1 : n_t;

  if (threadIdx.x == 0) {
    prefetch_tensormap(&tmQ);
    prefetch_tensormap(&tmK);
    prefetch_tensormap(&tmV);
    prefetch_tensormap(&tmdO);
    mbar_init(q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(kv_full(s), 1);
      mbar_init(kv_empty(s), 1);
    }
    mbar_init(s_full, 1);
    mbar_init(ds_full, 4);
    mbar_init(final_bar, 1);
    fence_barrier_init();
  }
  if (warp == 5) tmem_alloc(tslot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tslot_ptr);
  const uint32_t tS = tmem, tDP = tmem + 128, tDQ = tmem + 256;

  if (warp == 4) {
    if (lane == 0) {
      bool ok = true;
      mbar_expect_tx(q_full, 2 * kTileBytes);
      tma_load_4d(sQ, &tmQ, 0, q0, h, b, q_full);
      tma_load_4d(sdO, &tmdO, 0, q0, h, b, q_full);
      for (int j = 0; j < n_kv && ok; ++j) {
        const int st = j & 1;
        if (!mbar_wait(kv_empty(st), (uint32_t)(((j >> 1) & 1) ^ 1), a.err)) { ok = false; break; }
        mbar_expect_tx(kv_full(st), 2 * kTileBytes);
        tma_load_4d(sK(st), &tmK, 0, j * kTile, h, b, kv_full(st));
        tma_load_4d(sV(st), &tmV, 0, j * kTile, h, b, kv_full(st));
      }
      for (int j = n_kv; j < n_kv + 2 && ok; ++j) {
        const int st = j & 1;
        if (!mbar_wait(kv_empty(st), (uint32_t)(((j >> 1) & 1) ^ 1), a.err)) ok = false;
      }
    }
  } else if (warp == 5) {
    if (lane == 0) {
      constexpr uint32_t idS = idesc_bf16_f32(kTile, kTile, 0, 0);
      constexpr uint32_t idG = idesc_bf16_f32(kTile, kHd, 0, 1);
      bool ok = mbar_wait(q_full, 0, a.err);
      auto issue_dq = [&](int j) -> bool {
        const int st = j & 1;
        if (!mbar_wait(ds_full, (uint32_t)(j & 1), a.err)) return false;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kTile / 16; ++kk)
          mma_bf16_ss(tDQ, desc_k(sDS + (kk >> 2) * 16384 + (kk & 3) * 32),
                      desc_mn(sK(st) + kk * 2048), idG, (j > 0 || kk > 0) ? 1u : 0u);
        mma_commit(kv_empty(st));
        return true;
      };
      for (int j = 0; j < n_kv && ok; ++j) {
        const int st = j & 1;
        if (!mbar_wait(kv_full(st), (uint32_t)((j >> 1) & 1), a.err)) { ok = false; break; }
        tc_fence_after();
        if (j > 0 && !issue_dq(j - 1)) { ok = false; break; }
#pragma unroll
        for (int kk = 0; kk < kHd / 16; ++kk) {
          mma_bf16_ss(tS, desc_k(sQ + kk * 32), desc_k(sK(st) + kk * 32), idS, kk > 0 ? 1u : 0u);
          mma_bf16_ss(tDP, desc_k(sdO + kk * 32), desc_k(sV(st) + kk * 32), idS,
                      kk > 0 ? 1u : 0u);
        }
        mma_commit(s_full);
      }
      if (ok && n_kv >= 1) issue_dq(n_kv - 1);
      mma_commit(final_bar);
      mbar_wait(final_bar, 0, a.err);
    }
  } else {
    const int r = warp * 32 + lane;
    const int qg = q0 + r;
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    const float sl2 = a.scale * kLog2e;
    const int64_t bh = (int64_t)b * a.H + h;
    const float lse2 = qg < a.S ? a.lse[bh * a.S + qg] * kLog2e : INFINITY;
    const float dl = qg < a.S ? a.delta[bh * a.S + qg] : 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      const int k0 = j * kTile;
      if (!mbar_wait(s_full, (uint32_t)(j & 1), a.err)) { ok = false; break; }
      tc_fence_after();
      const bool diag = a.causal && (k0 + kTile > q0);
      const bool tail = k0 + kTile > a.S || q0 + kTile > a.S;
      const bool masked_tile = diag || tail;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t vs[32], vd[32];
        tmem_ld32(tS + lane_off + c * 32, vs);
        tmem_ld32(tDP + lane_off + c * 32, vd);
        tmem_wait_ld();
        float ds[32];
        if (!masked_tile) {
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const float pe = ex2_approx(fmaf(__uint_as_float(vs[e]), sl2, -lse2));
            ds[e] = pe * (__uint_as_float(vd[e]) - dl);
          }
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const int kg = k0 + c * 32 + e;
            const bool masked = (diag && kg > qg) || (tail && kg >= a.S) || qg >= a.S;
            const float pe = masked ? 0.f : ex2_approx(fmaf(__uint_as_float(vs[e]), sl2, -lse2));
            ds[e] = pe * (__uint_as_float(vd[e]) - dl);
          }
        }
        store_row32(sDS, r, c, ds);
      }
      tc_fence_before();
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(ds_full);
    }
    if (ok && mbar_wait(final_bar, 0, a.err)) {
      tc_fence_after();
      float acc[kHd];
      uint32_t v0[32], v1[32];
      tmem_ld32(tDQ + lane_off, v0);
      tmem_ld32(tDQ + lane_off + 32, v1);
      tmem_wait_ld();
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        acc[c] = __uint_as_float(v0[c]);
        acc[32 + c] = __uint_as_float(v1[c]);
      }
      if (qg < a.S)
        store_global_row64(static_cast<__nv_bfloat16*>(a.dq) + (int64_t)b * a.qs0 +
                               (int64_t)h * a.qs1 + (int64_t)qg * a.qs2,
                           acc, a.scale);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ===================================================== backward, fused
// One CTA per 128-key tile j (heaviest causal tiles first), looping over the
// query tiles i that see it. Per (i, j):
//   S^T = K_j Q_i^T, dP^T = V_j dO_i^T                     (TMEM)
//   P^T = exp2(S^T*scale*log2e - lse_i*log2e), dS^T = P^T (dP^T - delta_i)
//   dV_j += P^T dO_i, dK_j += dS^T Q_i                     (TMEM accumulators)
//   dQ_ij = dS K_j -> F32 partial tile in the workspace      (TMEM, drained)
// P^T and dS^T go to 128-byte-swizzled shared memory as BF16; the dS^T buffer
// is the K-major A operand of dK and, read MN-major, the A operand of dQ. The
// dQ partials are summed over j in a fixed order by attn_dq_reduce
// (deterministic; no atomics).
// Warps 0-7: element math, thread = key row (TMEM lane quarter warp % 4) x
// one half of the 128 query columns (warp / 4); warp 8: TMA producer;
// warp 9: TMEM allocator and MMA issuer.
constexpr int kBwThreads = 320;
constexpr int kBwK = 0;
constexpr int kBwV = kTileBytes;
constexpr int kBwQdo = 2 * kTileBytes;                      // 2 stages x (Q, dO)
constexpr int kBwDST = kBwQdo + 2 * 2 * kTileBytes;         // 2 buffers x 32 KB
constexpr int kBwStats = kBwDST + 2 * 2 * kTileBytes;       // lse2[128], delta[128]
constexpr int kBwBar = kBwStats + 2 * kTile * 4;
// kv_full, qdo_full[2], qdo_empty[2], st_full, pds_full, dq_full[2], dq_free[2], final
constexpr int kBwNumBars = 12;
constexpr int kBwSmem = kBwBar + kBwNumBars * 8 + 16 + 1024;
constexpr int kDqTileFloats = kTile * kHd;                  // one F32 dQ partial tile

// Index of the dQ partial of (query tile i, key tile j) among a head's slots.
__host__ __device__ __forceinline__ int64_t dq_slot(int i, int j, int n_t, int causal) {
  return causal ? (int64_t)i * (i + 1) / 2 + j : (int64_t)i * n_t + j;
}
__host__ __device__ __forceinline__ int64_t dq_slots(int n_t, int causal) {
  return causal ? (int64_t)n_t * (n_t + 1) / 2 : (int64_t)n_t * n_t;
}
// A partial tile is stored as 16 column groups of 4 floats x 128 rows, i.e.
// float4 index (column / 4) * 128 + row, so that a warp's stores of one column
// group over its 32 rows are 512 contiguous bytes.

// Writes 32 packed BF16 pairs (64 columns) of row r at columns [64*half,
// 64*half+64) of a [128 x 128] K-major SW128 tile.
__device__ __forceinline__ void store_row_packed(uint32_t base, int r, int c32,
                                                 const uint32_t* pk) {
#pragma unroll
  for (int q = 0; q < 4; ++q)
    st_shared_v4(swz_chunk_addr(base, r, c32 * 4 + q), pk[4 * q], pk[4 * q + 1], pk[4 * q + 2],
                 pk[4 * q + 3]);
}

// Pipeline over query tiles it = 0, 1, ...:
//   MMA warp:   S(0) | [P(it) ready] dV(it) dK(it) S(it+1) dQ(it) | ...
//   math warps: softmax(it) -> P(it) ready -> drain dQ(it-1) -> softmax(it+1)
// P^T and dS^T are written back into TMEM over the S^T and dP^T columns each
// thread has read (thread half h: columns [64h, 64h+32)) and are the A
// operands of dV and dK, read from TMEM; dS^T also goes to shared memory as
// the MN-major A operand of dQ. dQ alternates between two TMEM buffers, dS^T
// between two shared buffers, so dQ(it) and the drain of dQ(it-1) run under
// the exponentials of tile it+1.
__global__ void __launch_bounds__(kBwThreads, 1)
attn_bwd_tc(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
            const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO,
            AttnTcArgs a, float* __restrict__ dq_part) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sp;
  const uint32_t base = align1024(smem_raw, &sp);
  const uint32_t sK = base + kBwK, sV = base + kBwV;
  auto sQ = [&](int st) { return base + kBwQdo + st * 2 * kTileBytes; };
  auto sdO = [&](int st) { return base + kBwQdo + st * 2 * kTileBytes + kTileBytes; };
  auto sDST = [&](int pb) { return base + kBwDST + pb * 2 * kTileBytes; };
  float* lse_s = reinterpret_cast<float*>(sp + kBwStats);           // [128], log2 units
  float* delta_s = reinterpret_cast<float*>(sp + kBwStats + kTile * 4);
  const uint32_t bars = base + kBwBar;
  const uint32_t kv_full = bars;
  auto qdo_full = [&](int st) { return bars + 8u * (1 + st); };
  auto qdo_empty = [&](int st) { return bars + 8u * (3 + st); };
  const uint32_t st_full = bars + 8u * 5;
  const uint32_t pds_full = bars + 8u * 6;
  auto dq_full = [&](int db) { return bars + 8u * (7 + db); };
  auto dq_free = [&](int db) { return bars + 8u * (9 + db); };
  const uint32_t final_bar = bars + 8u * 11;
  const uint32_t tslot = bars + 8u * kBwNumBars;
  uint32_t* tslot_ptr = reinterpret_cast<uint32_t*>(sp + kBwBar + 8 * kBwNumBars);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_t = (a.S + kTile - 1) / kTile;
  // Linear dispatch order with the key tile varying slowest: key tile 0 has
  // the most query tiles under causal, so the heaviest blocks start first and
  // the lightest fill the tail.
  const int lin = (int)(blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z));
  const int heads = (int)(gridDim.y * gridDim.z);
  const int kt = lin / heads;
  const int h = (lin % heads) % (int)gridDim.y, b = (lin % heads) / (int)gridDim.y;
  const int k0 = kt * kTile;
  const int first_q = a.causal ? kt : 0;
  const int n_it = n_t - first_q;

  if (threadIdx.x == 0) {
    prefetch_tensormap(&tmQ);
    prefetch_tensormap(&tmK);
    prefetch_tensormap(&tmV);
    prefetch_tensormap(&tmdO);
    mbar_init(kv_full, 1);
    for (int st = 0; st < 2; ++st) {
      mbar_init(qdo_full(st), 1);
      mbar_init(qdo_empty(st), 1);
      mbar_init(dq_full(st), 1);
      mbar_init(dq_free(st), 8);
    }
    mbar_init(st_full, 1);
    mbar_init(pds_full, 8);
    mbar_init(final_bar, 1);
    fence_barrier_init();
  }
  if (warp == 9) tmem_alloc(tslot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tslot_ptr);
  const uint32_t tST = tmem, tDPT = tmem + 128, tDV = tmem + 256, tDK = tmem + 320;
  auto tDQ = [&](int db) { return tmem + 384u + (uint32_t)(db * kHd); };

  if (warp == 8) {
    if (lane == 0) {
      bool ok = true;
      mbar_expect_tx(kv_full, 2 * kTileBytes);
      tma_load_4d(sK, &tmK, 0, k0, h, b, kv_full);
      tma_load_4d(sV, &tmV, 0, k0, h, b, kv_full);
      for (int it = 0; it < n_it && ok; ++it) {
        const int st = it & 1;
        const int q0 = (first_q + it) * kTile;
        if (!mbar_wait(qdo_empty(st), (uint32_t)(((it >> 1) & 1) ^ 1), a.err)) {
          ok = false;
          break;
        }
        mbar_expect_tx(qdo_full(st), 2 * kTileBytes);
        tma_load_4d(sQ(st), &tmQ, 0, q0, h, b, qdo_full(st));
        tma_load_4d(sdO(st), &tmdO, 0, q0, h, b, qdo_full(st));
      }
      for (int it = n_it; it < n_it + 2 && ok; ++it) {
        const int st = it & 1;
        if (!mbar_wait(qdo_empty(st), (uint32_t)(((it >> 1) & 1) ^ 1), a.err)) ok = false;
      }
    }
  } else if (warp == 9) {
    if (lane == 0) {
      constexpr uint32_t idS = idesc_bf16_f32(kTile, kTile, 0, 0);
      constexpr uint32_t idG = idesc_bf16_f32(kTile, kHd, 0, 1);   // A K-major, B MN-major
      constexpr uint32_t idQ = idesc_bf16_f32(kTile, kHd, 1, 1);   // A MN-major (dS from dS^T)
      auto issue_s = [&](int it) -> bool {
        const int st = it & 1;
        if (!mbar_wait(qdo_full(st), (uint32_t)((it >> 1) & 1), a.err)) return false;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kHd / 16; ++kk) {
          mma_bf16_ss(tST, desc_k(sK + kk * 32), desc_k(sQ(st) + kk * 32), idS, kk > 0 ? 1u : 0u);
          mma_bf16_ss(tDPT, desc_k(sV + kk * 32), desc_k(sdO(st) + kk * 32), idS,
                      kk > 0 ? 1u : 0u);
        }
        mma_commit(st_full);
        return true;
      };
      bool ok = mbar_wait(kv_full, 0, a.err);
      if (ok && n_it > 0) ok = issue_s(0);
      for (int it = 0; it < n_it && ok; ++it) {
        const int st = it & 1, pb = it & 1;
        if (!mbar_wait(pds_full, (uint32_t)(it & 1), a.err)) { ok = false; break; }
        tc_fence_after();
        // dV += P^T dO, dK += dS^T Q with P^T / dS^T read from TMEM: queries
        // [0, 64) at columns [0, 32), queries [64, 128) at columns [64, 96).
#pragma unroll
        for (int kk = 0; kk < kTile / 16; ++kk) {
          const uint32_t acol = (uint32_t)((kk >> 2) * 64 + (kk & 3) * 8);
          mma_bf16_ts(tDV, tST + acol, desc_mn(sdO(st) + kk * 2048), idG,
                      (it > 0 || kk > 0) ? 1u : 0u);
          mma_bf16_ts(tDK, tDPT + acol, desc_mn(sQ(st) + kk * 2048), idG,
                      (it > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(qdo_empty(st));
        // S(it+1) overwrites P^T / dS^T(it): issued after the MMAs reading them
        if (it + 1 < n_it && !issue_s(it + 1)) { ok = false; break; }
        // dQ buffer pb was last used by dQ(it-2); its drain must be done
        if (it >= 2 && !mbar_wait(dq_free(pb), (uint32_t)(((it - 2) >> 1) & 1), a.err)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // dQ_ij = dS K_j: A = dS^T read MN-major (query blocks of 64 are 16 KB
        // apart), B = K_j MN-major; 16 keys per step = 16 rows of 128 bytes.
#pragma unroll
        for (int kk = 0; kk < kTile / 16; ++kk)
          mma_bf16_ss(tDQ(pb), smem_desc_sw128(sDST(pb) + kk * 2048, 16384, 1024),
                      desc_mn(sK + kk * 2048), idQ, kk > 0 ? 1u : 0u);
        mma_commit(dq_full(pb));
      }
      mma_commit(final_bar);
      mbar_wait(final_bar, 0, a.err);
    }
  } else {
    // ------------------------------ element math ------------------------------
    const int quarter = warp & 3, half = warp >> 2;
    const int r = quarter * 32 + lane;  // key row within the tile / dQ row
    const int kg = k0 + r;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const int cbase = half * 64;        // this thread's query columns [cbase, cbase + 64)
    const float sl2 = a.scale * kLog2e;
    const int64_t bh = (int64_t)b * a.H + h;
    float* part_base = dq_part + bh * dq_slots(n_t, a.causal) * kDqTileFloats;
    const int t = threadIdx.x;  // 0..255: lse (t < 128) or delta of query row t & 127
    auto load_stat = [&](int it) -> float {
      const int qi = (first_q + it) * kTile + (t & 127);
      if (t < 128) return qi < a.S ? a.lse[bh * a.S + qi] * kLog2e : INFINITY;
      return qi < a.S ? a.delta[bh * a.S + qi] : 0.f;
    };
    // Drains dQ(it) (TMEM buffer it & 1): row r, column groups 8*half .. +8.
    auto drain = [&](int it, bool ok) -> bool {
      const int db = it & 1;
      if (ok && !mbar_wait(dq_full(db), (uint32_t)((it >> 1) & 1), a.err)) ok = false;
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) return false;
      tc_fence_after();
      uint32_t v[32];
      tmem_ld32(tDQ(db) + lane_off + half * 32, v);
      tmem_wait_ld();
      float4* dst = reinterpret_cast<float4*>(
          part_base + dq_slot(first_q + it, kt, n_t, a.causal) * kDqTileFloats);
#pragma unroll
      for (int g = 0; g < 8; ++g)
        dst[(half * 8 + g) * kTile + r] =
            make_float4(__uint_as_float(v[4 * g]), __uint_as_float(v[4 * g + 1]),
                        __uint_as_float(v[4 * g + 2]), __uint_as_float(v[4 * g + 3]));
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(dq_free(db));
      return true;
    };
    bool ok = true;
    float stat = n_it > 0 ? load_stat(0) : 0.f;
    for (int it = 0; it < n_it; ++it) {
      const int pb = it & 1;
      const int qt = first_q + it;
      const int q0 = qt * kTile;
      (t < 128 ? lse_s[t] : delta_s[t - 128]) = stat;
      if (it + 1 < n_it) stat = load_stat(it + 1);  // lands during this tile
      named_barrier(1, 256);
      if (ok && !mbar_wait(st_full, (uint32_t)(it & 1), a.err)) ok = false;
      ok = __all_sync(0xffffffffu, ok);
      if (ok) {
        tc_fence_after();
        const bool diag = a.causal && qt == kt;
        const bool tail = q0 + kTile > a.S || k0 + kTile > a.S;
        // P^T and dS^T for this thread's 64 query columns, 32 at a time; the
        // masked variant only runs on the diagonal tile and a ragged edge.
        auto chunk = [&](auto masked_c, int c) {
          constexpr bool kMasked = decltype(masked_c)::value;
          const int col = cbase + 32 * c;
          uint32_t vs[32], vd[32];
          tmem_ld32(tST + lane_off + col, vs);
          tmem_ld32(tDPT + lane_off + col, vd);
          const float4* l4 = reinterpret_cast<const float4*>(lse_s + col);
          const float4* d4 = reinterpret_cast<const float4*>(delta_s + col);
          tmem_wait_ld();
          uint32_t pp[16], pd[16];
#pragma unroll
          for (int g = 0; g < 8; ++g) {
            const float4 lv = l4[g], dv4 = d4[g];
            const float ls[4] = {lv.x, lv.y, lv.z, lv.w};
            const float dl[4] = {dv4.x, dv4.y, dv4.z, dv4.w};
            float pe[4], de[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const int e = 4 * g + u;
              pe[u] = ex2_approx(fmaf(__uint_as_float(vs[e]), sl2, -ls[u]));
              de[u] = pe[u] * (__uint_as_float(vd[e]) - dl[u]);
              if (kMasked) {
                const int qg = q0 + col + e;
                if ((diag && qg < kg) || qg >= a.S || kg >= a.S) pe[u] = de[u] = 0.f;
              }
            }
            pp[2 * g] = pack_bf16(pe[0], pe[1]);
            pp[2 * g + 1] = pack_bf16(pe[2], pe[3]);
            pd[2 * g] = pack_bf16(de[0], de[1]);
            pd[2 * g + 1] = pack_bf16(de[2], de[3]);
          }
          // BF16 columns [64*half + 16*c, +16): S^T / dP^T columns this thread
          // has already read
          tmem_st16(tST + lane_off + cbase + 16 * c, pp);
          tmem_st16(tDPT + lane_off + cbase + 16 * c, pd);
          store_row_packed(sDST(pb), r, col >> 5, pd);
        };
        if (diag || tail) {
          chunk(std::true_type{}, 0);
          chunk(std::true_type{}, 1);
        } else {
          chunk(std::false_type{}, 0);
          chunk(std::false_type{}, 1);
        }
        tmem_wait_st();
        fence_proxy_async_smem();
        tc_fence_before();
      }
      named_barrier(2, 256);  // every thread is done with the row terms of this tile
      if (ok && lane == 0) mbar_arrive(pds_full);
      if (it >= 1) ok = drain(it - 1, ok) && ok;
    }
    if (n_it >= 1) ok = drain(n_it - 1, ok) && ok;
    if (ok && !mbar_wait(final_bar, 0, a.err)) ok = false;
    ok = __all_sync(0xffffffffu, ok);
    if (ok) {
      tc_fence_after();
      uint32_t v0[32], v1[32];
      tmem_ld32(tDV + lane_off + half * 32, v0);
      tmem_ld32(tDK + lane_off + half * 32, v1);
      tmem_wait_ld();
      if (kg < a.S) {
        const int64_t off =
            (int64_t)b * a.qs0 + (int64_t)h * a.qs1 + (int64_t)kg * a.qs2 + half * 32;
        __nv_bfloat16* dvp = static_cast<__nv_bfloat16*>(a.dv) + off;
        __nv_bfloat16* dkp = static_cast<__nv_bfloat16*>(a.dk) + off;
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          uint4 u, w;
          u.x = pack_bf16(__uint_as_float(v0[8 * g + 0]), __uint_as_float(v0[8 * g + 1]));
          u.y = pack_bf16(__uint_as_float(v0[8 * g + 2]), __uint_as_float(v0[8 * g + 3]));
          u.z = pack_bf16(__uint_as_float(v0[8 * g + 4]), __uint_as_float(v0[8 * g + 5]));
          u.w = pack_bf16(__uint_as_float(v0[8 * g + 6]), __uint_as_float(v0[8 * g + 7]));
          w.x = pack_bf16(__uint_as_float(v1[8 * g + 0]) * a.scale,
                          __uint_as_float(v1[8 * g + 1]) * a.scale);
          w.y = pack_bf16(__uint_as_float(v1[8 * g + 2]) * a.scale,
                          __uint_as_float(v1[8 * g + 3]) * a.scale);
          w.z = pack_bf16(__uint_as_float(v1[8 * g + 4]) * a.scale,
                          __uint_as_float(v1[8 * g + 5]) * a.scale);
          w.w = pack_bf16(__uint_as_float(v1[8 * g + 6]) * a.scale,
                          __uint_as_float(v1[8 * g + 7]) * a.scale);
          reinterpret_cast<uint4*>(dvp)[g] = u;
          reinterpret_cast<uint4*>(dkp)[g] = w;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// delta[b, h, s] = sum_d dO * O over a row of 64 (BF16): 8 threads per row,
// 16-byte loads, 32 rows per CTA; grid (ceil(S / 32), H, B).
__global__ void __launch_bounds__(256)
attn_delta_tc(const __nv_bfloat16* __restrict__ o, const __nv_bfloat16* __restrict__ d_o,
              float* __restrict__ delta, int S, int H, int64_t os0, int64_t os1, int64_t os2) {
  const int row = blockIdx.x * 32 + (threadIdx.x >> 3);
  const int part = threadIdx.x & 7;
  const int h = blockIdx.y, b = blockIdx.z;
  float acc = 0.f;
  if (row < S) {
    const int64_t off = (int64_t)b * os0 + (int64_t)h * os1 + (int64_t)row * os2 + part * 8;
    float x[8], y[8];
    load8(o + off, x);
    load8(d_o + off, y);
#pragma unroll
    for (int i = 0; i < 8; ++i) acc += x[i] * y[i];
  }
  acc += __shfl_xor_sync(0xffffffffu, acc, 4);
  acc += __shfl_xor_sync(0xffffffffu, acc, 2);
  acc += __shfl_xor_sync(0xffffffffu, acc, 1);
  if (part == 0 && row < S) delta[((int64_t)b * H + h) * S + row] = acc;
}

// dQ[b, h, q] = scale * sum over key tiles j (in order) of the F32 partials
// of query tile i -> BF16 (caller's strided layout). One CTA per (i, h, b);
// thread = 4 consecutive columns of 8 rows.
__global__ void __launch_bounds__(256)
attn_dq_reduce(const float* __restrict__ dq_part, __nv_bfloat16* __restrict__ dq, int S, int H,
               int causal, float scale, int64_t qs0, int64_t qs1, int64_t qs2) {
  const int n_t = (S + kTile - 1) / kTile;
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int64_t bh = (int64_t)b * H + h;
  const float* base = dq_part + bh * dq_slots(n_t, causal) * kDqTileFloats;
  const int j_end = causal ? qt + 1 : n_t;
#pragma unroll 1
  for (int g = threadIdx.x; g < kDqTileFloats / 4; g += blockDim.x) {
    const int row = g % kTile, col = (g / kTile) * 4;  // column-group-major tiles
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = 0; j < j_end; ++j) {
      const float4 t = reinterpret_cast<const float4*>(
          base + dq_slot(qt, j, n_t, causal) * kDqTileFloats)[g];
      acc.x += t.x;
      acc.y += t.y;
      acc.z += t.z;
      acc.w += t.w;
    }
    const int q = qt * kTile + row;
    if (q < S) {
      uint2 u;
      u.x = pack_bf16(acc.x * scale, acc.y * scale);
      u.y = pack_bf16(acc.z * scale, acc.w * scale);
      *reinterpret_cast<uint2*>(dq + (int64_t)b * qs0 + (int64_t)h * qs1 + (int64_t)q * qs2 +
                                col) = u;
    }
  }
}

// 4-D tensor map over a [B, H, S, 64] BF16 view with element strides
// (sb, sh, ss), box [128 rows x 64] with 128-byte swizzle.
magma_status_t head_map(CUtensorMap* m, const void* base, int64_t B, int64_t H, int64_t S,
                        int64_t sb, int64_t sh, int64_t ss) {
  const uint64_t dims[4] = {(uint64_t)kHd, (uint64_t)S, (uint64_t)H, (uint64_t)B};
  const uint64_t strides[3] = {(uint64_t)ss * 2, (uint64_t)sh * 2, (uint64_t)sb * 2};
  const uint32_t box[4] = {(uint32_t)kHd, (uint32_t)kTile, 1, 1};
  return encode_tensor_map_nd(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, base, 4, dims, strides, box,
                              CU_TENSOR_MAP_SWIZZLE_128B);
}

// Opts kernel `ID` into `bytes` of dynamic shared memory once per device
// (the cache is keyed by ID: the kernels share one function type).
template <int ID, typename K>
magma_status_t set_smem_attr(K kern, int bytes) {
  static bool done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && done[dev]) return MAGMA_OK;
  if (magma_status_t s = cuda_status(
          cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes),
          "cudaFuncSetAttribute(attention_tc)"))
    return s;
  if (dev >= 0 && dev < 64) done[dev] = true;
  return MAGMA_OK;
}

bool strides_ok(const int64_t* s) {
  for (int i = 0; i < 3; ++i)
    if ((s[i] * 2) % 16 != 0) return false;
  return true;
}

}  // namespace

// True if the tcgen05 kernels can take this problem (BF16, head_dim 64, TMA-
// compatible strides and 16-byte aligned bases).
bool attention_tc_supported(const void* q, const void* k, const void* v, const void* o,
                            int64_t hd, const int64_t* qs, const int64_t* os,
                            magma_dtype_t dtype, int64_t batch, int64_t heads, int64_t seq) {
  return dtype == MAGMA_DTYPE_BF16 && hd == kHd && aligned16(q) && aligned16(k) && aligned16(v) &&
         aligned16(o) && strides_ok(qs) && strides_ok(os) && batch < 65536 && heads < 65536 &&
         seq < (1LL << 30);
}

magma_status_t attention_fwd_tc(const void* q, const void* k, const void* v, void* o, float* lse,
                                int64_t B, int64_t H, int64_t S, const int64_t* qs,
                                const int64_t* os, float scale, int causal, cudaStream_t s) {
  CUtensorMap mq, mk, mv;
  if (magma_status_t st = head_map(&mq, q, B, H, S, qs[0], qs[1], qs[2])) return st;
  if (magma_status_t st = head_map(&mk, k, B, H, S, qs[0], qs[1], qs[2])) return st;
  if (magma_status_t st = head_map(&mv, v, B, H, S, qs[0], qs[1], qs[2])) return st;
  AttnTcArgs a{};
  a.S = (int)S; a.H = (int)H; a.B = (int)B; a.scale = scale; a.causal = causal;
  a.o = o; a.lse = lse;
  a.os0 = os[0]; a.os1 = os[1]; a.os2 = os[2];
  a.qs0 = qs[0]; a.qs1 = qs[1]; a.qs2 = qs[2];
  a.err = device_error_word();
  if (magma_status_t st = set_smem_attr<0>(attn_fwd_tc, kFwdSmem)) return st;
  dim3 grid((unsigned)ceil_div(ceil_div(S, kTile), 2), (unsigned)H, (unsigned)B);
  attn_fwd_tc<<<grid, kFwdThreads, kFwdSmem, s>>>(mq, mk, mv, a);
  return check_launch("attention_fwd_tcgen05");
}

// Workspace of the fused backward: delta (B*H*S floats), then the F32 dQ
// partial tiles (query tile x key tile pairs of every head).
size_t attention_bwd_tc_partials_bytes(int64_t B, int64_t H, int64_t S, int causal) {
  const int n_t = (int)ceil_div(S, kTile);
  return (size_t)(B * H) * (size_t)dq_slots(n_t, causal) * kDqTileFloats * sizeof(float);
}
size_t attention_bwd_tc_delta_bytes(int64_t B, int64_t H, int64_t S) {
  return ((size_t)(B * H * S) * sizeof(float) + 255) & ~(size_t)255;
}

magma_status_t attention_bwd_tc(const void* q, const void* k, const void* v, const void* o,
                                const void* d_o, const float* lse, void* dq, void* dk, void* dv,
                                void* workspace, size_t ws_bytes, int64_t B, int64_t H, int64_t S,
                                const int64_t* qs, const int64_t* os, float scale, int causal,
                                cudaStream_t s) {
  float* delta = static_cast<float*>(workspace);
  attn_delta_tc<<<dim3((unsigned)ceil_div(S, 32), (unsigned)H, (unsigned)B), 256, 0, s>>>(
      static_cast<const __nv_bfloat16*>(o), static_cast<const __nv_bfloat16*>(d_o), delta, (int)S,
      (int)H, os[0], os[1], os[2]);
  if (magma_status_t st = check_launch("attention_bwd_delta")) return st;
  CUtensorMap mq, mk, mv, mdo;
  if (magma_status_t st = head_map(&mq, q, B, H, S, qs[0], qs[1], qs[2])) return st;
  if (magma_status_t st = head_map(&mk, k, B, H, S, qs[0], qs[1], qs[2])) return st;
  if (magma_status_t st = head_map(&mv, v, B, H, S, qs[0], qs[1], qs[2])) return st;
  if (magma_status_t st = head_map(&mdo, d_o, B, H, S, os[0], os[1], os[2])) return st;
  AttnTcArgs a{};
  a.S = (int)S; a.H = (int)H; a.B = (int)B; a.scale = scale; a.causal = causal;
  a.lse = const_cast<float*>(lse); a.delta = delta;
  a.dq = dq; a.dk = dk; a.dv = dv;
  a.os0 = os[0]; a.os1 = os[1]; a.os2 = os[2];
  a.qs0 = qs[0]; a.qs1 = qs[1]; a.qs2 = qs[2];
  a.err = device_error_word();
  dim3 grid((unsigned)ceil_div(S, kTile), (unsigned)H, (unsigned)B);
  const size_t dbytes = attention_bwd_tc_delta_bytes(B, H, S);
  if (ws_bytes >= dbytes + attention_bwd_tc_partials_bytes(B, H, S, causal)) {
    float* part = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + dbytes);
    if (magma_status_t st = set_smem_attr<3>(attn_bwd_tc, kBwSmem)) return st;
    attn_bwd_tc<<<grid, kBwThreads, kBwSmem, s>>>(mq, mk, mv, mdo, a, part);
    if (magma_status_t st = check_launch("attention_bwd_tcgen05")) return st;
    attn_dq_reduce<<<grid, 256, 0, s>>>(part, static_cast<__nv_bfloat16*>(dq), (int)S, (int)H,
                                        causal, scale, qs[0], qs[1], qs[2]);
    return check_launch("attention_bwd_dq_reduce");
  }
  // Without room for the partials: dK/dV and dQ in two passes.
  if (magma_status_t st = set_smem_attr<1>(attn_bwd_dkdv_tc, kKvSmem)) return st;
  if (magma_status_t st = set_smem_attr<2>(attn_bwd_dq_tc, kDqSmem)) return st;
  attn_bwd_dkdv_tc<<<grid, kThreads, kKvSmem, s>>>(mq, mk, mv, mdo, a);
  if (magma_status_t st = check_launch("attention_bwd_dkdv_tcgen05")) return st;
  attn_bwd_dq_tc<<<grid, kThreads, kDqSmem, s>>>(mq, mk, mv, mdo, a);
  return check_launch("attention_bwd_dq_tcgen05");
}

}  // namespace magma
