// C-ABI entry points for causal attention: argument checks and dispatch
// between the tcgen05 BF16 kernels (head_dim 64) and the F32-accurate SIMT
// kernels (F32 inputs, other head sizes).
#include "common.cuh"

namespace magma {
magma_status_t attention_fwd_simt(const void* q, const void* k, const void* v, void* o,
                                  float* lse, int64_t batch, int64_t heads, int64_t seq,
                                  int64_t hd, const int64_t* qs, const int64_t* os, float scale,
                                  int causal, magma_dtype_t dtype, cudaStream_t s);
magma_status_t attention_bwd_simt(const void* q, const void* k, const void* v, const void* o,
                                  const void* d_o, const float* lse, void* dq, void* dk, void* dv,
                                  float* delta, int64_t batch, int64_t heads, int64_t seq,
                                  int64_t hd, const int64_t* qs, const int64_t* os, float scale,
                                  int causal, magma_dtype_t dtype, cudaStream_t s);
bool attention_tc_supported(const void* q, const void* k, const void* v, const void* o,
                            int64_t hd, const int64_t* qs, const int64_t* os,
                            magma_dtype_t dtype, int64_t batch, int64_t heads, int64_t seq);
magma_status_t attention_fwd_tc(const void* q, const void* k, const void* v, void* o, float* lse,
                                int64_t B, int64_t H, int64_t S, const int64_t* qs,
                                const int64_t* os, float scale, int causal, cudaStream_t s);
size_t attention_bwd_tc_partials_bytes(int64_t B, int64_t H, int64_t S, int causal);
size_t attention_bwd_tc_delta_bytes(int64_t B, int64_t H, int64_t S);
magma_status_t attention_bwd_tc(const void* q, const void* k, const void* v, const void* o,
                                const void* d_o, const float* lse, void* dq, void* dk, void* dv,
                                void* workspace, size_t ws_bytes, int64_t B, int64_t H, int64_t S,
                                const int64_t* qs, const int64_t* os, float scale, int causal,
                                cudaStream_t s);
}  // namespace magma

using namespace magma;

namespace {

magma_status_t check_geometry(const char* fn, int64_t batch, int64_t heads, int64_t seq,
                              int64_t hd, const int64_t* qs, const int64_t* os,
                              magma_dtype_t dtype) {
  MAGMA_REQUIRE(batch >= 0 && heads >= 0 && seq >= 0, "%s: negative size", fn);
  MAGMA_REQUIRE(batch < 65536 && heads < 65536, "%s: batch and heads must be < 65536", fn);
  MAGMA_REQUIRE(hd >= 1 && hd <= 128, "%s: head_dim %lld outside [1, 128]", fn, (long long)hd);
  MAGMA_REQUIRE(dtype == MAGMA_DTYPE_F32 || dtype == MAGMA_DTYPE_BF16,
                "%s: dtype must be F32 or BF16", fn);
  MAGMA_REQUIRE(qs != nullptr && os != nullptr, "%s: NULL strides", fn);
  for (int i = 0; i < 3; ++i)
    MAGMA_REQUIRE(qs[i] >= 0 && os[i] >= 0, "%s: negative stride", fn);
  return MAGMA_OK;
}

}  // namespace

extern "C" {

magma_status_t magma_attention_fwd(const void* q, const void* k, const void* v, void* o,
                                   float* lse, int64_t batch, int64_t heads, int64_t seq,
                                   int64_t head_dim, const int64_t* qkv_strides,
                                   const int64_t* o_strides, float scale, int32_t causal,
                                   magma_dtype_t dtype, void* stream) {
  if (magma_status_t st = check_geometry("magma_attention_fwd", batch, heads, seq, head_dim,
                                         qkv_strides, o_strides, dtype))
    return st;
  if (batch == 0 || heads == 0 || seq == 0) return MAGMA_OK;
  MAGMA_REQUIRE(q && k && v && o, "magma_attention_fwd: NULL pointer");
  if (attention_tc_supported(q, k, v, o, head_dim, qkv_strides, o_strides, dtype, batch, heads,
                             seq))
    return attention_fwd_tc(q, k, v, o, lse, batch, heads, seq, qkv_strides, o_strides, scale,
                            causal, (cudaStream_t)stream);
  return attention_fwd_simt(q, k, v, o, lse, batch, heads, seq, head_dim, qkv_strides, o_strides,
                            scale, causal, dtype, (cudaStream_t)stream);
}

size_t magma_attention_bwd_workspace_size(int64_t batch, int64_t heads, int64_t seq,
                                          int64_t head_dim, magma_dtype_t dtype) {
  if (batch <= 0 || heads <= 0 || seq <= 0) return 0;
  const size_t delta = attention_bwd_tc_delta_bytes(batch, heads, seq);
  // BF16 head_dim 64 runs the fused tensor-core backward, which also keeps one
  // F32 dQ partial tile per (query tile, key tile) pair (the non-causal count,
  // an upper bound for causal); capped at 4 GiB, beyond which it falls back to
  // the two-pass kernels that need only delta.
  if (dtype == MAGMA_DTYPE_BF16 && head_dim == 64) {
    const size_t part = attention_bwd_tc_partials_bytes(batch, heads, seq, 0);
    if (part <= (4ull << 30)) return delta + part;
  }
  return delta;
}

magma_status_t magma_attention_bwd(const void* q, const void* k, const void* v, const void* o,
                                   const void* d_o, const float* lse, void* dq, void* dk, void* dv,
                                   int64_t batch, int64_t heads, int64_t seq, int64_t head_dim,
                                   const int64_t* qkv_strides, const int64_t* o_strides,
                                   float scale, int32_t causal, magma_dtype_t dtype,
                                   void* workspace, size_t workspace_bytes, void* stream) {
  if (magma_status_t st = check_geometry("magma_attention_bwd", batch, heads, seq, head_dim,
                                         qkv_strides, o_strides, dtype))
    return st;
  if (batch == 0 || heads == 0 || seq == 0) return MAGMA_OK;
  MAGMA_REQUIRE(q && k && v && o && d_o && lse && dq && dk && dv,
                "magma_attention_bwd: NULL pointer");
  // Minimum: the row terms delta (two-pass kernels); the size the query
  // returns also lets BF16 head_dim 64 take the fused kernel.
  const size_t need = attention_bwd_tc_delta_bytes(batch, heads, seq);
  MAGMA_REQUIRE(workspace != nullptr && workspace_bytes >= need,
                "magma_attention_bwd: workspace of at least %zu bytes needed, %zu given", need,
                workspace_bytes);
  if (attention_tc_supported(q, k, v, o, head_dim, qkv_strides, o_strides, dtype, batch, heads,
                             seq) &&
      aligned16(d_o) && aligned16(dq) && aligned16(dk) && aligned16(dv))
    return attention_bwd_tc(q, k, v, o, d_o, lse, dq, dk, dv, workspace, workspace_bytes, batch,
                            heads, seq, qkv_strides, o_strides, scale, causal,
                            (cudaStream_t)stream);
  return attention_bwd_simt(q, k, v, o, d_o, lse, dq, dk, dv, (float*)workspace, batch, heads, seq,
                            head_dim, qkv_strides, o_strides, scale, causal, dtype,
                            (cudaStream_t)stream);
}

}  // extern "C"
