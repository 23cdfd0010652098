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
//                  (thread = query row) running their exponential passes
//                  concurrently; S_t = Q_t K_j^T in TMEM, P_t written to TMEM
//                  as BF16 and used from there as the A operand of
//                  O_t += P_t V_j;
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
// desc(addr + off) for a descriptor d = desc(addr): the start address sits in
// the low 14 bits in 16-byte units, and shared-memory addresses stay below
// 256 KB, so the sum never carries out of that field.
__device__ __forceinline__ uint64_t desc_add(uint64_t d, uint32_t off_bytes) {
  return d + (uint64_t)(off_bytes >> 4);
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

// The r-th work unit of CTA c among G persistent CTAs (snake order: round r
// takes units r*G .. r*G+G-1, even rounds in CTA order, odd rounds
// reversed), or -1 past the end.
__device__ __forceinline__ int bw_unit(int r, int c, int G, int U) {
  const int u = r * G + ((r & 1) ? G - 1 - c : c);
  return u < U ? u : -1;
}

// =============================================================== forward
// Persistent: one CTA per SM walks a static list of work units (a pair of
// 128-query tiles t = 0, 1 of one head, query rows q0 .. q0+255), heaviest
// causal pairs first, in the same snake order over the CTAs as the backward.
// Warps 0-3 run the softmax of tile 0, warps 4-7 that of tile 1, warp 8 is
// the TMA producer (Q double-buffered per unit, K/V through a 3-stage ring
// that runs on across units), warp 9 allocates TMEM and issues the MMAs. Both
// tiles stream the same K/V tiles, so while one warpgroup turns S_t into P_t
// the tensor cores work on the other tile:
//   MMA order: S0(0) S1(0) | S0(1) PV0(0) S1(1) PV1(0) | S0(2) PV0(1) ...
// TMEM: S_t at columns 128t (F32 128x128), O_t at 256 + 64t, P_t (BF16
// pairs, the TMEM A operand of PV_t = P_t V_j) at 384 + 64t. A warpgroup
// releases S_t's columns (s_free) as soon as its exponential pass has read
// the last of them, so S_t(j+1) (or the next unit's S_t(0)) is computed while
// the pass finishes and while the other warpgroup runs its own; before it
// writes P_t or rescales or reads O_t it waits for the previous PV_t
// (pv_done). O_t and the row sum are rescaled only when a row maximum grows
// by more than 2^8 (otherwise the stale maximum is kept: P <= 2^8, exact
// after the final division). Barrier phases count a warpgroup's steps over
// all its units.
constexpr int kFwdStages = 3;
constexpr int kFwdThreads = 320;                 // 8 softmax warps + producer + MMA
constexpr int kFwdQ = 0;                         // 2 buffers x Q tiles 0, 1 (4 x 16 KB)
constexpr int kFwdKv = 4 * kTileBytes;           // K, V per stage
constexpr int kFwdBar = kFwdKv + kFwdStages * 2 * kTileBytes;
// q_full[2], q_empty[2], kv_full[3], kv_empty[3], s_full[2], s_free[2], p_full[2],
// pv_done[2], done
constexpr int kFwdNumBars = 19;
constexpr int kFwdSmem = kFwdBar + kFwdNumBars * 8 + 16 + 1024;
constexpr float kRescaleLog2 = 8.0f;

__global__ void __launch_bounds__(kFwdThreads, 1)
attn_fwd_tc(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
            const __grid_constant__ CUtensorMap tmV, AttnTcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sp;
  const uint32_t base = align1024(smem_raw, &sp);
  auto sQ = [&](int qb, int t) { return base + kFwdQ + (2 * qb + t) * kTileBytes; };
  auto sK = [&](int st) { return base + kFwdKv + st * 2 * kTileBytes; };
  auto sV = [&](int st) { return base + kFwdKv + st * 2 * kTileBytes + kTileBytes; };
  const uint32_t bars = base + kFwdBar;
  auto q_full = [&](int qb) { return bars + 8u * qb; };
  auto q_empty = [&](int qb) { return bars + 8u * (2 + qb); };
  auto kv_full = [&](int st) { return bars + 8u * (4 + st); };
  auto kv_empty = [&](int st) { return bars + 8u * (7 + st); };
  auto s_full = [&](int t) { return bars + 8u * (10 + t); };
  auto s_free = [&](int t) { return bars + 8u * (12 + t); };
  auto p_full = [&](int t) { return bars + 8u * (14 + t); };
  auto pv_done = [&](int t) { return bars + 8u * (16 + t); };
  const uint32_t done_bar = bars + 8u * 18;
  const uint32_t tslot = bars + 8u * kFwdNumBars;
  uint32_t* tslot_ptr = reinterpret_cast<uint32_t*>(sp + kFwdBar + 8 * kFwdNumBars);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_qt = (a.S + kTile - 1) / kTile;
  const int n_pairs = (n_qt + 1) / 2;
  const int heads = a.H * a.B;
  const int U = n_pairs * heads;
  const int G = (int)gridDim.x, c = (int)blockIdx.x;
  // unit u: query-tile pair n_pairs - 1 - u / heads (varying slowest, so the
  // heaviest causal pairs come first), head u % heads
  struct Unit {
    int qt0, h, b, nk0, nk1, n_kv;
    bool has1;
  };
  auto unit = [&](int u) {
    Unit w;
    w.qt0 = 2 * (n_pairs - 1 - u / heads);
    w.has1 = w.qt0 + 1 < n_qt;
    const int hb = u % heads;
    w.h = hb % a.H;
    w.b = hb / a.H;
    // key tiles visited by query tile t
    w.nk0 = a.causal ? w.qt0 + 1 : n_qt;
    w.nk1 = w.has1 ? (a.causal ? w.qt0 + 2 : n_qt) : 0;
    w.n_kv = w.nk0 > w.nk1 ? w.nk0 : w.nk1;
    return w;
  };

  if (threadIdx.x == 0) {
    prefetch_tensormap(&tmQ);
    prefetch_tensormap(&tmK);
    prefetch_tensormap(&tmV);
    for (int qb = 0; qb < 2; ++qb) {
      mbar_init(q_full(qb), 1);
      mbar_init(q_empty(qb), 1);
    }
    for (int st = 0; st < kFwdStages; ++st) {
      mbar_init(kv_full(st), 1);
      mbar_init(kv_empty(st), 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(s_full(t), 1);
      mbar_init(s_free(t), 4);
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
  auto tP = [&](int t) { return tmem + 384u + (uint32_t)(t * kHd); };

  if (warp == 8) {
    if (lane == 0) {
      bool ok = true;
      int gk = 0;  // K/V tiles loaded so far (ring position)
      for (int r = 0; ok; ++r) {
        const int u = bw_unit(r, c, G, U);
        if (u < 0) break;
        const Unit w = unit(u);
        const int qb = r & 1;
        // Q buffer qb was last read by unit r-2
        if (!mbar_wait(q_empty(qb), (uint32_t)(((r >> 1) & 1) ^ 1), a.err)) { ok = false; break; }
        mbar_expect_tx(q_full(qb), (w.has1 ? 2 : 1) * kTileBytes);
        tma_load_4d(sQ(qb, 0), &tmQ, 0, w.qt0 * kTile, w.h, w.b, q_full(qb));
        if (w.has1) tma_load_4d(sQ(qb, 1), &tmQ, 0, (w.qt0 + 1) * kTile, w.h, w.b, q_full(qb));
        for (int j = 0; j < w.n_kv; ++j, ++gk) {
          const int st = gk % kFwdStages;
          if (!mbar_wait(kv_empty(st), (uint32_t)(((gk / kFwdStages) & 1) ^ 1), a.err)) {
            ok = false;
            break;
          }
          mbar_expect_tx(kv_full(st), 2 * kTileBytes);
          tma_load_4d(sK(st), &tmK, 0, j * kTile, w.h, w.b, kv_full(st));
          tma_load_4d(sV(st), &tmV, 0, j * kTile, w.h, w.b, kv_full(st));
        }
      }
      // every stage loaded above has been consumed before the producer leaves
      for (int k = gk; k < gk + kFwdStages && ok; ++k) {
        const int st = k % kFwdStages;
        if (!mbar_wait(kv_empty(st), (uint32_t)(((k / kFwdStages) & 1) ^ 1), a.err)) ok = false;
      }
    }
  } else if (warp == 9) {
    if (lane == 0) {
      constexpr uint32_t idS = idesc_bf16_f32(kTile, kTile, 0, 0);
      constexpr uint32_t idPV = idesc_bf16_f32(kTile, kHd, 0, 1);
      bool ok = true;
      int gk = 0;             // K/V tiles consumed so far
      int ns[2] = {0, 0};     // S_t issued so far (all units)
      int np[2] = {0, 0};     // PV_t issued so far
      // Descriptors are formed once; every instruction then adds an immediate
      // byte offset >> 4 (desc_add), which keeps the single issuing thread's
      // scalar work per tcgen05.mma to one add.
      const uint64_t dq0 = desc_k(sQ(0, 0)), dk0 = desc_k(sK(0)), dv0 = desc_mn(sV(0));
      // S_t of K/V tile at ring position kg, Q buffer qb; waits for S_t's
      // columns to be free (the previous S_t read by its warpgroup)
      auto issue_s = [&](int t, int qb, int kg) -> bool {
        if (ns[t] >= 1 && !mbar_wait(s_free(t), (uint32_t)((ns[t] - 1) & 1), a.err)) return false;
        const int st = kg % kFwdStages;
        if (!mbar_wait(kv_full(st), (uint32_t)((kg / kFwdStages) & 1), a.err)) return false;
        tc_fence_after();
        const uint64_t dq = desc_add(dq0, (uint32_t)(2 * qb + t) * kTileBytes);
        const uint64_t dk = desc_add(dk0, (uint32_t)st * 2 * kTileBytes);
        const uint32_t d = tS(t);
#pragma unroll
        for (int kk = 0; kk < kHd / 16; ++kk)
          mma_bf16_ss(d, desc_add(dq, kk * 32), desc_add(dk, kk * 32), idS, kk > 0 ? 1u : 0u);
        mma_commit(s_full(t));
        ++ns[t];
        return true;
      };
      auto issue_pv = [&](int t, int j, int kg) -> bool {
        if (!mbar_wait(p_full(t), (uint32_t)(np[t] & 1), a.err)) return false;
        tc_fence_after();
        const int st = kg % kFwdStages;
        const uint64_t dv = desc_add(dv0, (uint32_t)st * 2 * kTileBytes);
        const uint32_t d = tO(t), pa = tP(t);
        const uint32_t acc = j > 0 ? 1u : 0u;
#pragma unroll
        for (int kk = 0; kk < kTile / 16; ++kk)
          mma_bf16_ts(d, pa + kk * 8, desc_add(dv, kk * 2048), idPV, kk > 0 ? 1u : acc);
        mma_commit(pv_done(t));
        ++np[t];
        return true;
      };
      for (int r = 0; ok; ++r) {
        const int u = bw_unit(r, c, G, U);
        if (u < 0) break;
        const Unit w = unit(u);
        const int qb = r & 1;
        if (!mbar_wait(q_full(qb), (uint32_t)((r >> 1) & 1), a.err)) { ok = false; break; }
        if (w.n_kv > 0) {
          if (!issue_s(0, qb, gk)) { ok = false; break; }
          if (w.nk1 > 0 && !issue_s(1, qb, gk)) { ok = false; break; }
        }
        for (int j = 0; j < w.n_kv && ok; ++j) {
          for (int t = 0; t < 2 && ok; ++t) {
            const int nk = t ? w.nk1 : w.nk0;
            if (j >= nk) continue;
            // S_t(j+1) as soon as warpgroup t has read all of S_t(j)
            if (j + 1 < nk && !issue_s(t, qb, gk + j + 1)) { ok = false; break; }
            if (!issue_pv(t, j, gk + j)) { ok = false; break; }
          }
          if (ok) mma_commit(kv_empty((gk + j) % kFwdStages));
        }
        if (!ok) break;
        gk += w.n_kv;
        mma_commit(q_empty(qb));
      }
      mma_commit(done_bar);
      mbar_wait(done_bar, 0, a.err);
    }
  } else {
    // ---------------------------- softmax warpgroups ----------------------------
    const int t = warp >> 2;
    const int r_row = (warp & 3) * 32 + lane;
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t srow = tS(t) + lane_off;
    const uint32_t orow = tO(t) + lane_off;
    const uint32_t prow = tP(t) + lane_off;
    const float sl2 = a.scale * kLog2e;
    bool ok = true;
    int gs = 0;  // this warpgroup's steps over all its units (barrier phases)
    for (int r = 0; ok; ++r) {
    const int u = bw_unit(r, c, G, U);
    if (u < 0) break;
    const Unit w = unit(u);
    const int nk = t ? w.nk1 : w.nk0;
    const int qt = w.qt0 + t;
    const int qg = qt * kTile + r_row;
    float m_run = -INFINITY, l_run = 0.f;
    // The two warpgroups run their exponential passes concurrently (the
    // hardware interleaves their MUFU work with the other's FMA and TMEM
    // traffic; strict turn-taking between them measured 3% slower).
    for (int j = 0; j < nk; ++j, ++gs) {
      const int k0 = j * kTile;
      // Only the diagonal tile (causal) and a ragged last tile need masking;
      // every other tile takes the mask-free path (warp-uniform branch).
      const bool diag = a.causal && j == qt;
      const bool tail = k0 + kTile > a.S;
      const bool masked_tile = diag || tail;
      int lim = 127;  // last unmasked column of this row
      if (diag) lim = qg - k0;
      if (tail && a.S - 1 - k0 < lim) lim = a.S - 1 - k0;
      if (ok && !mbar_wait(s_full(t), (uint32_t)(gs & 1), a.err)) ok = false;
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
        // the previous PV_t has read P_t and added into O_t before either is
        // touched (at a unit's first step: the last PV_t of the unit before)
        if (gs >= 1 && !mbar_wait(pv_done(t), (uint32_t)((gs - 1) & 1), a.err)) ok = false;
        ok = __all_sync(0xffffffffu, ok);
        if (ok) {
          tc_fence_after();
          if (j == 0) {
            m_run = m_new == -INFINITY ? 0.f : m_new;
          } else if (__any_sync(0xffffffffu, m_new > m_run + kRescaleLog2)) {
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
      }
      // pass 2: P = exp2(S * scale * log2(e) - m) as BF16 pairs into P_t's
      // columns. The first half of the row is read from TMEM first, the rest
      // while the first is exponentiated; once the last column is read S_t's
      // columns are released for S_t(j+1).
      uint32_t va[2][32];
      if (ok) {
        tmem_ld32(srow, va[0]);
        tmem_ld32(srow + 32, va[1]);
        tmem_wait_ld();
        // The pass is issue-bound: the scaled arguments and the row sums are
        // formed two columns per instruction (packed F32 pairs; same rounding
        // per element as scalar FMA/add), the row sum in two pair
        // accumulators.
        unsigned long long rs2[2] = {0ull, 0ull};
        const unsigned long long sl22 = f2_pack(sl2, sl2), nm2 = f2_pack(-m_run, -m_run);
        // Exponentiates 32 columns starting at column c of S (v) into 16
        // packed BF16 pairs stored at P_t's columns [c/2, c/2 + 16).
        auto exp32 = [&](const uint32_t (&v)[32], int c) {
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            float x0, x1;
            f2_unpack(f2_fma(f2_pack(__uint_as_float(v[2 * e]), __uint_as_float(v[2 * e + 1])),
                             sl22, nm2), x0, x1);
            float p0 = ex2_approx(x0);
            float p1 = ex2_approx(x1);
            if (masked_tile) {
              if (c + 2 * e > lim) p0 = 0.f;
              if (c + 2 * e + 1 > lim) p1 = 0.f;
            }
            rs2[e & 1] = f2_add(rs2[e & 1], f2_pack(p0, p1));
            pk[e] = pack_bf16(p0, p1);
          }
          tmem_st16(prow + c / 2, pk);
        };
        uint32_t vb[32];
        exp32(va[0], 0);
        tmem_ld32(srow + 64, vb);  // lands while columns 32-63 are exponentiated
        exp32(va[1], 32);
        tmem_wait_ld();
        uint32_t vc[32];
        tmem_ld32(srow + 96, vc);
        exp32(vb, 64);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(s_free(t));  // all of S_t(j) is in registers
        exp32(vc, 96);
        {
          float a0, a1, b0, b1;
          f2_unpack(rs2[0], a0, a1);
          f2_unpack(rs2[1], b0, b1);
          l_run += (a0 + a1) + (b0 + b1);
        }
        tmem_wait_st();
      }
      if (ok) {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(p_full(t));
      }
    }
    if (ok && nk > 0 && !mbar_wait(pv_done(t), (uint32_t)((gs - 1) & 1), a.err)) ok = false;
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
        for (int cc = 0; cc < 32; ++cc) {
          of[cc] = __uint_as_float(o0[cc]);
          of[32 + cc] = __uint_as_float(o1[cc]);
        }
        const float inv = 1.0f / l_run;
        __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(a.o) + (int64_t)w.b * a.os0 +
                             (int64_t)w.h * a.os1 + (int64_t)qg * a.os2;
        store_global_row64(dst, of, inv);
        if (a.lse != nullptr)
          a.lse[((int64_t)w.b * a.H + w.h) * a.S + qg] = m_run * kLn2 + logf(l_run);
      }
    }
    }  // units
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
// Persistent: one CTA per SM walks a static list of work units (a key tile of
// one head), heaviest first, in a snake order over the CTAs (round r takes
// units r*G .. r*G+G-1, even rounds in CTA order, odd rounds reversed), which
// balances the causal units' unequal sizes to within a few per cent of the
// mean. Pipelines run on across units: the producer prefetches the next
// unit's K (double-buffered) and V (single, reloaded once the unit's last
// S^T/dP^T have read it) and its Q / dO stages while the current unit ends.
// Warps 0-7: element math, thread = key row (TMEM lane quarter warp % 4) x
// one half of the 128 query columns (warp / 4); warp 8: TMA producer, which
// also stages each query tile's row terms (lse in log2 units, delta); warp 9:
// TMEM allocator and MMA issuer; warp 10: sends the dQ partial tiles to the
// workspace with bulk copies.
constexpr int kBwThreads = 352;
constexpr int kBwQdoStages = 3;
constexpr int kBwK = 0;                                     // 2 buffers x 16 KB
constexpr int kBwV = 2 * kTileBytes;
constexpr int kBwQdo = 3 * kTileBytes;                      // 3 stages x (Q, dO)
constexpr int kBwDST = kBwQdo + kBwQdoStages * 2 * kTileBytes;  // 2 buffers x 32 KB
constexpr int kBwStats = kBwDST + 2 * 2 * kTileBytes;       // 3 stages x (lse2[128], delta[128])
constexpr int kBwBar = kBwStats + kBwQdoStages * 2 * kTile * 4;
// k_full[2], k_empty[2], v_full, v_empty, qdo_full[3], qdo_empty[3], stats_full[3],
// st_full, st_free, pds_full, pt_free, dq_full, dq_free, staged, stage_free,
// acc_full, acc_empty, final
constexpr int kBwNumBars = 26;
constexpr int kBwSmem = kBwBar + kBwNumBars * 8 + 16 + 1024;
static_assert(kBwSmem <= 232448, "backward shared memory");

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

// Pipeline over the CTA's query-tile iterations g = 0, 1, ... (across its
// units; TC = tensor-core issue order):
//   TC:    S(0) | S(g+1) dV(g) dK(g) dQ(g) | S(g+2) dV(g+1) ...
//   math:  load S^T, dP^T(g) -> [S^T/dP^T free] -> P^T, dS^T -> [ready]
//          -> drain dQ(g-1) -> load S^T, dP^T(g+1) -> ...   (and, after a
//          unit's last iteration, dV / dK of the unit -> [accumulators free])
// Each math thread loads its 64 columns of S^T and dP^T into registers and
// releases those TMEM columns at once (st_free), so S(g+1) and dP(g+1) run on
// the tensor cores while it computes P^T and dS^T of iteration g. P^T goes to
// its own 64 TMEM columns (BF16 pairs; the TMEM A operand of dV), dS^T to a
// double-buffered 128-byte-swizzled shared tile (the K-major A operand of dK
// and, read MN-major, of dQ). Once dQ(g) has completed, dS^T buffer g & 1 is
// free: the drain of dQ(g) writes the F32 partial tile there in the
// workspace layout and warp 10 sends it out with one bulk copy, releasing the
// buffer (stage_free) when the copy has read it; the dS^T of iteration g+2
// waits for that. The row terms of each query tile arrive with its Q / dO
// stage (stats_full). P^T's TMEM columns are rewritten one iteration later,
// after pt_free (committed after dV(g)); the single dQ accumulator is drained
// (dq_free) before dQ(g+1) is issued; a unit's first dV / dK wait until the
// previous unit's have been read out (acc_empty).
// TMEM columns: S^T [0,128), dP^T [128,256), dV [256,320), dK [320,384),
// dQ [384,448), P^T [448,512).
__global__ void __launch_bounds__(kBwThreads, 1)
attn_bwd_tc(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
            const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO,
            AttnTcArgs a, float* __restrict__ dq_part) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sp;
  const uint32_t base = align1024(smem_raw, &sp);
  auto sK = [&](int kb) { return base + kBwK + kb * kTileBytes; };
  const uint32_t sV = base + kBwV;
  auto sQ = [&](int st) { return base + kBwQdo + st * 2 * kTileBytes; };
  auto sdO = [&](int st) { return base + kBwQdo + st * 2 * kTileBytes + kTileBytes; };
  auto sDST = [&](int pb) { return base + kBwDST + pb * 2 * kTileBytes; };
  // row terms of stage st: lse (log2 units) [128], then delta [128]
  auto stats = [&](int st) { return reinterpret_cast<float*>(sp + kBwStats + st * 2 * kTile * 4); };
  const uint32_t bars = base + kBwBar;
  auto k_full = [&](int kb) { return bars + 8u * kb; };
  auto k_empty = [&](int kb) { return bars + 8u * (2 + kb); };
  const uint32_t v_full = bars + 8u * 4;
  const uint32_t v_empty = bars + 8u * 5;
  auto qdo_full = [&](int st) { return bars + 8u * (6 + st); };
  auto qdo_empty = [&](int st) { return bars + 8u * (9 + st); };
  auto stats_full = [&](int st) { return bars + 8u * (12 + st); };
  const uint32_t st_full = bars + 8u * 15;
  const uint32_t st_free = bars + 8u * 16;
  const uint32_t pds_full = bars + 8u * 17;
  const uint32_t pt_free = bars + 8u * 18;
  const uint32_t dq_full = bars + 8u * 19;
  const uint32_t dq_free = bars + 8u * 20;
  const uint32_t staged = bars + 8u * 21;
  const uint32_t stage_free = bars + 8u * 22;
  const uint32_t acc_full = bars + 8u * 23;
  const uint32_t acc_empty = bars + 8u * 24;
  const uint32_t final_bar = bars + 8u * 25;
  const uint32_t tslot = bars + 8u * kBwNumBars;
  uint32_t* tslot_ptr = reinterpret_cast<uint32_t*>(sp + kBwBar + 8 * kBwNumBars);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_t = (a.S + kTile - 1) / kTile;
  const int heads = a.H * a.B;
  const int U = n_t * heads;
  const int G = (int)gridDim.x, c = (int)blockIdx.x;
  // unit u: key tile u / heads (varying slowest: heaviest causal units first)
  struct Unit {
    int kt, h, b, first_q, n_it;
    int64_t bh;
  };
  auto unit = [&](int u) {
    Unit w;
    w.kt = u / heads;
    const int hb = u % heads;
    w.h = hb % a.H;
    w.b = hb / a.H;
    w.first_q = a.causal ? w.kt : 0;
    w.n_it = n_t - w.first_q;
    w.bh = (int64_t)w.b * a.H + w.h;
    return w;
  };

  if (threadIdx.x == 0) {
    prefetch_tensormap(&tmQ);
    prefetch_tensormap(&tmK);
    prefetch_tensormap(&tmV);
    prefetch_tensormap(&tmdO);
    for (int kb = 0; kb < 2; ++kb) {
      mbar_init(k_full(kb), 1);
      mbar_init(k_empty(kb), 1);
    }
    mbar_init(v_full, 1);
    mbar_init(v_empty, 1);
    for (int st = 0; st < kBwQdoStages; ++st) {
      mbar_init(qdo_full(st), 1);
      mbar_init(qdo_empty(st), 1);
      mbar_init(stats_full(st), 32);
    }
    mbar_init(st_full, 1);
    mbar_init(st_free, 8);
    mbar_init(pds_full, 8);
    mbar_init(pt_free, 1);
    mbar_init(dq_full, 1);
    mbar_init(dq_free, 8);
    mbar_init(staged, 8);
    mbar_init(stage_free, 1);
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 8);
    mbar_init(final_bar, 1);
    fence_barrier_init();
  }
  if (warp == 9) tmem_alloc(tslot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tslot_ptr);
  const uint32_t tST = tmem, tDPT = tmem + 128, tDV = tmem + 256, tDK = tmem + 320;
  const uint32_t tDQ = tmem + 384, tPT = tmem + 448;

  if (warp == 8) {
    // ------------------- TMA producer and row terms (whole warp) -------------------
    bool ok = true;
    int g = 0;
    for (int r = 0;; ++r) {
      const int u = bw_unit(r, c, G, U);
      if (u < 0) break;
      const Unit w = unit(u);
      const int kb = r & 1;
      if (lane == 0) {
        // K buffer kb was last read by unit r-2, V by unit r-1
        if (!mbar_wait(k_empty(kb), (uint32_t)(((r >> 1) & 1) ^ 1), a.err)) ok = false;
        if (ok) {
          mbar_expect_tx(k_full(kb), kTileBytes);
          tma_load_4d(sK(kb), &tmK, 0, w.kt * kTile, w.h, w.b, k_full(kb));
        }
        if (ok && !mbar_wait(v_empty, (uint32_t)((r & 1) ^ 1), a.err)) ok = false;
        if (ok) {
          mbar_expect_tx(v_full, kTileBytes);
          tma_load_4d(sV, &tmV, 0, w.kt * kTile, w.h, w.b, v_full);
        }
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      for (int it = 0; it < w.n_it && ok; ++it, ++g) {
        const int st = g % kBwQdoStages;
        const int q0 = (w.first_q + it) * kTile;
        if (!mbar_wait(qdo_empty(st), (uint32_t)(((g / kBwQdoStages) & 1) ^ 1), a.err)) ok = false;
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        if (lane == 0) {
          mbar_expect_tx(qdo_full(st), 2 * kTileBytes);
          tma_load_4d(sQ(st), &tmQ, 0, q0, w.h, w.b, qdo_full(st));
          tma_load_4d(sdO(st), &tmdO, 0, q0, w.h, w.b, qdo_full(st));
        }
        // -lse (log2 units; the addend of the exponent) and delta of query
        // rows q0 + 4 lane .. +3
        float* sts = stats(st);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int row = 4 * lane + k, qi = q0 + row;
          sts[row] = qi < a.S ? -(a.lse[w.bh * a.S + qi] * kLog2e) : -INFINITY;
          sts[kTile + row] = qi < a.S ? a.delta[w.bh * a.S + qi] : 0.f;
        }
        mbar_arrive(stats_full(st));
      }
      if (!ok) break;
    }
    if (lane == 0) {  // every stage loaded above has been consumed before the producer leaves
      for (int k = g; k < g + kBwQdoStages && ok; ++k) {
        const int st = k % kBwQdoStages;
        if (!mbar_wait(qdo_empty(st), (uint32_t)(((k / kBwQdoStages) & 1) ^ 1), a.err)) ok = false;
      }
    }
  } else if (warp == 10) {
    // ------------- dQ partial tiles: shared staging -> workspace -------------
    if (lane == 0) {
      bool ok = true;
      int g = 0;
      for (int r = 0; ok; ++r) {
        const int u = bw_unit(r, c, G, U);
        if (u < 0) break;
        const Unit w = unit(u);
        float* part_base = dq_part + w.bh * dq_slots(n_t, a.causal) * kDqTileFloats;
        for (int it = 0; it < w.n_it; ++it, ++g) {
          if (!mbar_wait(staged, (uint32_t)(g & 1), a.err)) { ok = false; break; }
          bulk_store(part_base + dq_slot(w.first_q + it, w.kt, n_t, a.causal) * kDqTileFloats,
                     sDST(g & 1), kDqTileFloats * 4);
          bulk_commit_group();
          bulk_wait_group_read<0>();
          mbar_arrive(stage_free);
        }
      }
      bulk_wait_group_all();  // the partials are in the workspace before exit
    }
  } else if (warp == 9) {
    if (lane == 0) {
      constexpr uint32_t idS = idesc_bf16_f32(kTile, kTile, 0, 0);
      constexpr uint32_t idG = idesc_bf16_f32(kTile, kHd, 0, 1);   // A K-major, B MN-major
      constexpr uint32_t idQ = idesc_bf16_f32(kTile, kHd, 1, 1);   // A MN-major (dS from dS^T)
      // Descriptors formed once; each instruction adds an immediate offset.
      const uint64_t dK_k0 = desc_k(sK(0)), dK_mn0 = desc_mn(sK(0)), dV_k = desc_k(sV);
      const uint64_t dQ_k0 = desc_k(sQ(0)), dO_k0 = desc_k(sdO(0));
      const uint64_t dQ_mn0 = desc_mn(sQ(0)), dO_mn0 = desc_mn(sdO(0));
      const uint64_t dS_k0 = desc_k(sDST(0));
      const uint64_t dS_mn0 = smem_desc_sw128(sDST(0), 16384, 1024);
      constexpr uint32_t kStage = 2 * kTileBytes;  // bytes between Q/dO stages, dS^T buffers
      auto issue_s = [&](int g, uint64_t dkk) -> bool {
        const int st = g % kBwQdoStages;
        if (!mbar_wait(qdo_full(st), (uint32_t)((g / kBwQdoStages) & 1), a.err)) return false;
        tc_fence_after();
        const uint64_t dq = desc_add(dQ_k0, st * kStage), dd = desc_add(dO_k0, st * kStage);
#pragma unroll
        for (int kk = 0; kk < kHd / 16; ++kk) {
          mma_bf16_ss(tST, desc_add(dkk, kk * 32), desc_add(dq, kk * 32), idS, kk > 0 ? 1u : 0u);
          mma_bf16_ss(tDPT, desc_add(dV_k, kk * 32), desc_add(dd, kk * 32), idS,
                      kk > 0 ? 1u : 0u);
        }
        mma_commit(st_full);
        return true;
      };
      bool ok = true;
      int g = 0;
      for (int r = 0; ok; ++r) {
        const int u = bw_unit(r, c, G, U);
        if (u < 0) break;
        const Unit w = unit(u);
        const int kb = r & 1;
        if (!mbar_wait(k_full(kb), (uint32_t)((r >> 1) & 1), a.err) ||
            !mbar_wait(v_full, (uint32_t)(r & 1), a.err)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t dkk = desc_add(dK_k0, kb * kTileBytes);
        const uint64_t dkmn = desc_add(dK_mn0, kb * kTileBytes);
        if (!issue_s(g, dkk)) { ok = false; break; }
        if (w.n_it == 1) mma_commit(v_empty);  // the unit's last S^T / dP^T read V
        for (int it = 0; it < w.n_it; ++it, ++g) {
          const int st = g % kBwQdoStages, pb = g & 1;
          // math(g) holds S^T / dP^T in registers: the next tile's go in
          if (!mbar_wait(st_free, (uint32_t)(g & 1), a.err)) { ok = false; break; }
          tc_fence_after();
          if (it + 1 < w.n_it) {
            if (!issue_s(g + 1, dkk)) { ok = false; break; }
            if (it + 2 == w.n_it) mma_commit(v_empty);
          }
          if (!mbar_wait(pds_full, (uint32_t)(g & 1), a.err)) { ok = false; break; }
          // the previous unit's dV / dK have been read out
          if (it == 0 && r >= 1 && !mbar_wait(acc_empty, (uint32_t)((r - 1) & 1), a.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // dV += P^T dO (P^T from TMEM), dK += dS^T Q (dS^T K-major from smem)
          const uint64_t dmn = desc_add(dO_mn0, st * kStage), qmn = desc_add(dQ_mn0, st * kStage);
          const uint64_t dsk = desc_add(dS_k0, pb * kStage);
#pragma unroll
          for (int kk = 0; kk < kTile / 16; ++kk) {
            const uint32_t acc = (it > 0 || kk > 0) ? 1u : 0u;
            mma_bf16_ts(tDV, tPT + kk * 8, desc_add(dmn, kk * 2048), idG, acc);
            mma_bf16_ss(tDK, desc_add(dsk, (kk >> 2) * 16384 + (kk & 3) * 32),
                        desc_add(qmn, kk * 2048), idG, acc);
          }
          mma_commit(qdo_empty(st));
          mma_commit(pt_free);
          // the single dQ accumulator: dQ(g-1) drained before dQ(g)
          if (g >= 1 && !mbar_wait(dq_free, (uint32_t)((g - 1) & 1), a.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // dQ_ij = dS K_j: A = dS^T read MN-major (query blocks of 64 are 16 KB
          // apart), B = K_j MN-major; 16 keys per step = 16 rows of 128 bytes.
          const uint64_t dsm = desc_add(dS_mn0, pb * kStage);
#pragma unroll
          for (int kk = 0; kk < kTile / 16; ++kk)
            mma_bf16_ss(tDQ, desc_add(dsm, kk * 2048), desc_add(dkmn, kk * 2048), idQ,
                        kk > 0 ? 1u : 0u);
          mma_commit(dq_full);
          if (it + 1 == w.n_it) {
            mma_commit(acc_full);     // the unit's dV / dK are final
            mma_commit(k_empty(kb));  // and its K has been read for the last time
          }
        }
      }
      mma_commit(final_bar);
      mbar_wait(final_bar, 0, a.err);
    }
  } else {
    // ------------------------------ element math ------------------------------
    const int quarter = warp & 3, half = warp >> 2;
    const int r_row = quarter * 32 + lane;  // key row within the tile / dQ row
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const int cbase = half * 64;            // this thread's query columns [cbase, cbase + 64)
    const float sl2 = a.scale * kLog2e;
    // Drains dQ(g) (row r_row, column groups 8*half .. +8) into dS^T buffer
    // g & 1, free since dQ(g) completed, in the partial-tile layout (float4
    // index (column / 4) * 128 + row); warp 10 sends it on.
    auto drain = [&](int g, bool ok) -> bool {
      if (ok && !mbar_wait(dq_full, (uint32_t)(g & 1), a.err)) ok = false;
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) return false;
      tc_fence_after();
      uint32_t v[32];
      tmem_ld32(tDQ + lane_off + half * 32, v);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(dq_free);
      const uint32_t stage = sDST(g & 1);
#pragma unroll
      for (int gg = 0; gg < 8; ++gg)
        st_shared_v4(stage + (uint32_t)(((half * 8 + gg) * kTile + r_row) * 16), v[4 * gg],
                     v[4 * gg + 1], v[4 * gg + 2], v[4 * gg + 3]);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(staged);
      return true;
    };
    bool ok = true;
    int g = 0;
    for (int r = 0;; ++r) {
      const int u = bw_unit(r, c, G, U);
      if (u < 0) break;
      const Unit w = unit(u);
      const int k0 = w.kt * kTile;
      const int kg = k0 + r_row;
      for (int it = 0; it < w.n_it; ++it, ++g) {
        const int st = g % kBwQdoStages, pb = g & 1;
        const int qt = w.first_q + it;
        const int q0 = qt * kTile;
        if (ok && !mbar_wait(st_full, (uint32_t)(g & 1), a.err)) ok = false;
        ok = __all_sync(0xffffffffu, ok);
        if (ok) {
          tc_fence_after();
          // this thread's 64 columns of S^T and dP^T, then the columns are free
          uint32_t vs0[32], vs1[32], vd0[32], vd1[32];
          tmem_ld32(tST + lane_off + cbase, vs0);
          tmem_ld32(tST + lane_off + cbase + 32, vs1);
          tmem_ld32(tDPT + lane_off + cbase, vd0);
          tmem_ld32(tDPT + lane_off + cbase + 32, vd1);
          tmem_wait_ld();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(st_free);
          // row terms of this tile; P^T's TMEM columns read by dV(g-1)
          if (!mbar_wait(stats_full(st), (uint32_t)((g / kBwQdoStages) & 1), a.err)) ok = false;
          if (g >= 1 && !mbar_wait(pt_free, (uint32_t)((g - 1) & 1), a.err)) ok = false;
          ok = __all_sync(0xffffffffu, ok);
          if (ok) {
            tc_fence_after();
            const float* lse_s = stats(st);  // -lse in log2 units
            const float* delta_s = lse_s + kTile;
            const unsigned long long sl22 = f2_pack(sl2, sl2);
            const bool diag = a.causal && qt == w.kt;
            const bool tail = q0 + kTile > a.S || k0 + kTile > a.S;
            // P^T (to TMEM) and dS^T (packed, kept in pd) for 32 of this
            // thread's query columns; the masked variant only runs on the
            // diagonal tile and a ragged edge.
            auto chunk = [&](auto masked_c, auto c_c, const uint32_t(&vs)[32],
                             const uint32_t(&vd)[32], uint32_t(&pd)[16]) {
              constexpr bool kMasked = decltype(masked_c)::value;
              constexpr int cc = decltype(c_c)::value;
              const int col = cbase + 32 * cc;
              const float4* l4 = reinterpret_cast<const float4*>(lse_s + col);
              const float4* d4 = reinterpret_cast<const float4*>(delta_s + col);
              uint32_t pp[16];
#pragma unroll
              for (int gg = 0; gg < 8; ++gg) {
                const float4 lv = l4[gg], dv4 = d4[gg];
                // P and dS two query columns per instruction (packed F32 pairs,
                // the same rounding per element as scalar FMA/sub/mul)
                const unsigned long long nl2[2] = {f2_pack(lv.x, lv.y), f2_pack(lv.z, lv.w)};
                const unsigned long long dl2[2] = {f2_pack(dv4.x, dv4.y), f2_pack(dv4.z, dv4.w)};
                float pe[4], de[4];
#pragma unroll
                for (int hp = 0; hp < 2; ++hp) {
                  const int e = 4 * gg + 2 * hp;
                  float x0, x1;
                  f2_unpack(f2_fma(f2_pack(__uint_as_float(vs[e]), __uint_as_float(vs[e + 1])),
                                   sl22, nl2[hp]), x0, x1);
                  pe[2 * hp] = ex2_approx(x0);
                  pe[2 * hp + 1] = ex2_approx(x1);
                  f2_unpack(f2_mul(f2_pack(pe[2 * hp], pe[2 * hp + 1]),
                                   f2_sub(f2_pack(__uint_as_float(vd[e]), __uint_as_float(vd[e + 1])),
                                          dl2[hp])),
                            de[2 * hp], de[2 * hp + 1]);
                }
#pragma unroll
                for (int uu = 0; uu < 4; ++uu) {
                  if (kMasked) {
                    const int qg = q0 + col + 4 * gg + uu;
                    if ((diag && qg < kg) || qg >= a.S || kg >= a.S) pe[uu] = de[uu] = 0.f;
                  }
                }
                pp[2 * gg] = pack_bf16(pe[0], pe[1]);
                pp[2 * gg + 1] = pack_bf16(pe[2], pe[3]);
                pd[2 * gg] = pack_bf16(de[0], de[1]);
                pd[2 * gg + 1] = pack_bf16(de[2], de[3]);
              }
              // P^T: queries [64 half + 32 cc, +32) = TMEM columns 32 half + 16 cc
              tmem_st16(tPT + lane_off + 32 * half + 16 * cc, pp);
            };
            using c0 = std::integral_constant<int, 0>;
            using c1 = std::integral_constant<int, 1>;
            uint32_t pd0[16], pd1[16];
            if (diag || tail) {
              chunk(std::true_type{}, c0{}, vs0, vd0, pd0);
              chunk(std::true_type{}, c1{}, vs1, vd1, pd1);
            } else {
              chunk(std::false_type{}, c0{}, vs0, vd0, pd0);
              chunk(std::false_type{}, c1{}, vs1, vd1, pd1);
            }
            // dS^T buffer pb was last the staging of dQ(g-2): its bulk copy has
            // read it (issued an iteration ago, so this wait is normally met)
            if (g >= 2 && !mbar_wait(stage_free, (uint32_t)(g & 1), a.err)) ok = false;
            ok = __all_sync(0xffffffffu, ok);
            if (ok) {
              store_row_packed(sDST(pb), r_row, cbase >> 5, pd0);
              store_row_packed(sDST(pb), r_row, (cbase >> 5) + 1, pd1);
            }
            tmem_wait_st();
            fence_proxy_async_smem();
            tc_fence_before();
            __syncwarp();
            if (ok && lane == 0) mbar_arrive(pds_full);
          }
        }
        if (g >= 1) ok = drain(g - 1, ok) && ok;
      }
      // the unit's dV and dK (dK scaled by the softmax scale)
      if (ok && !mbar_wait(acc_full, (uint32_t)(r & 1), a.err)) ok = false;
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      uint32_t v0[32], v1[32];
      tmem_ld32(tDV + lane_off + half * 32, v0);
      tmem_ld32(tDK + lane_off + half * 32, v1);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_empty);
      if (kg < a.S) {
        const int64_t off =
            (int64_t)w.b * a.qs0 + (int64_t)w.h * a.qs1 + (int64_t)kg * a.qs2 + half * 32;
        __nv_bfloat16* dvp = static_cast<__nv_bfloat16*>(a.dv) + off;
        __nv_bfloat16* dkp = static_cast<__nv_bfloat16*>(a.dk) + off;
#pragma unroll
        for (int gg = 0; gg < 4; ++gg) {
          uint4 uv, wk;
          uv.x = pack_bf16(__uint_as_float(v0[8 * gg + 0]), __uint_as_float(v0[8 * gg + 1]));
          uv.y = pack_bf16(__uint_as_float(v0[8 * gg + 2]), __uint_as_float(v0[8 * gg + 3]));
          uv.z = pack_bf16(__uint_as_float(v0[8 * gg + 4]), __uint_as_float(v0[8 * gg + 5]));
          uv.w = pack_bf16(__uint_as_float(v0[8 * gg + 6]), __uint_as_float(v0[8 * gg + 7]));
          wk.x = pack_bf16(__uint_as_float(v1[8 * gg + 0]) * a.scale,
                           __uint_as_float(v1[8 * gg + 1]) * a.scale);
          wk.y = pack_bf16(__uint_as_float(v1[8 * gg + 2]) * a.scale,
                           __uint_as_float(v1[8 * gg + 3]) * a.scale);
          wk.z = pack_bf16(__uint_as_float(v1[8 * gg + 4]) * a.scale,
                           __uint_as_float(v1[8 * gg + 5]) * a.scale);
          wk.w = pack_bf16(__uint_as_float(v1[8 * gg + 6]) * a.scale,
                           __uint_as_float(v1[8 * gg + 7]) * a.scale);
          reinterpret_cast<uint4*>(dvp)[gg] = uv;
          reinterpret_cast<uint4*>(dkp)[gg] = wk;
        }
      }
    }
    if (g >= 1) ok = drain(g - 1, ok) && ok;
    if (ok && !mbar_wait(final_bar, 0, a.err)) ok = false;
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
// of query tile i -> BF16 (caller's strided layout). One CTA per (i, h, b).
// Thread = one 4-column group of 8 rows: the partials of a group are read
// with every load of the key-tile loop issued before the additions (512
// contiguous bytes per warp load), the sums go to a row-major shared tile,
// and the BF16 rows leave as whole 128-byte row segments (8 threads x 16 B).
__global__ void __launch_bounds__(256)
attn_dq_reduce(const float* __restrict__ dq_part, __nv_bfloat16* __restrict__ dq, int S, int H,
               int causal, float scale, int64_t qs0, int64_t qs1, int64_t qs2) {
  __shared__ float sum_s[kTile][kHd + 4];  // row pitch 68 floats: conflict-free float4 rows
  const int n_t = (S + kTile - 1) / kTile;
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int64_t bh = (int64_t)b * H + h;
  const float4* base = reinterpret_cast<const float4*>(dq_part + bh * dq_slots(n_t, causal) *
                                                                     kDqTileFloats);
  const int j_end = causal ? qt + 1 : n_t;
  const int64_t slot0 = dq_slot(qt, 0, n_t, causal);  // a query tile's slots are consecutive
  constexpr int kGroups = kDqTileFloats / 4;             // float4 groups per tile
#pragma unroll 1
  for (int g = threadIdx.x; g < kGroups; g += blockDim.x) {
    const int row = g % kTile, col = (g / kTile) * 4;  // column-group-major tiles
    float4 t[8];
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j0 = 0; j0 < j_end; j0 += 8) {
      const int nj = j_end - j0 < 8 ? j_end - j0 : 8;
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if (k < nj) t[k] = base[(slot0 + j0 + k) * kGroups + g];
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if (k < nj) {
          acc.x += t[k].x;
          acc.y += t[k].y;
          acc.z += t[k].z;
          acc.w += t[k].w;
        }
    }
    *reinterpret_cast<float4*>(&sum_s[row][col]) = acc;
  }
  __syncthreads();
  // rows of 64 columns: 8 threads x 8 columns per row, 32 rows per pass
  const int cg = threadIdx.x & 7;
#pragma unroll 1
  for (int row = threadIdx.x >> 3; row < kTile; row += blockDim.x >> 3) {
    const int q = qt * kTile + row;
    if (q >= S) continue;
    const float4 lo = *reinterpret_cast<const float4*>(&sum_s[row][8 * cg]);
    const float4 hi = *reinterpret_cast<const float4*>(&sum_s[row][8 * cg + 4]);
    uint4 u;
    u.x = pack_bf16(lo.x * scale, lo.y * scale);
    u.y = pack_bf16(lo.z * scale, lo.w * scale);
    u.z = pack_bf16(hi.x * scale, hi.y * scale);
    u.w = pack_bf16(hi.z * scale, hi.w * scale);
    *reinterpret_cast<uint4*>(dq + (int64_t)b * qs0 + (int64_t)h * qs1 + (int64_t)q * qs2 +
                              8 * cg) = u;
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
  // persistent: one CTA per SM over the query-tile pairs of every head
  const int64_t units = ceil_div(ceil_div(S, kTile), 2) * H * B;
  const int ctas = (int)(units < num_sms() ? units : num_sms());
  attn_fwd_tc<<<ctas, kFwdThreads, kFwdSmem, s>>>(mq, mk, mv, a);
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
  if (ws_bytes >= dbytes + attention_bwd_tc_partials_bytes(B, H, S, causal) &&
      aligned16(workspace)) {
    float* part = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + dbytes);
    if (magma_status_t st = set_smem_attr<3>(attn_bwd_tc, kBwSmem)) return st;
    // persistent: one CTA per SM over the n_t * H * B key-tile units
    const int64_t units = ceil_div(S, kTile) * H * B;
    const int ctas = (int)(units < num_sms() ? units : num_sms());
    attn_bwd_tc<<<ctas, kBwThreads, kBwSmem, s>>>(mq, mk, mv, mdo, a, part);
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
