// Shared helpers for libmagma_cuda.so: status/last-error plumbing, dtype
// traits, BF16 packing, warp reductions and the device-side error word.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stddef.h>

#include "../../include/magma_cuda.h"

namespace magma {

// Records a printf-style message as the calling thread's last error and
// returns `code` (the PJRT shim's "copy the message, return the code" rule,
// PJRTSimpleWrapper.h:86-99).
magma_status_t fail(magma_status_t code, const char* fmt, ...);

// Maps a CUDA runtime error to a status + message; MAGMA_OK if err == success.
magma_status_t cuda_status(cudaError_t err, const char* what);

// Checks the launch that just happened on this thread.
inline magma_status_t check_launch(const char* what) {
  return cuda_status(cudaGetLastError(), what);
}

// SM count of the current device (cached per device ordinal).
int num_sms();

// Device address of the error word that bounded waits set on timeout
// (one per device, found once per device with cudaGetSymbolAddress).
int* device_error_word();

// Error codes kernels write into the device error word.
enum DeviceErrorCode : int {
  kDevErrNone = 0,
  kDevErrWaitTimeout = 1,   // an mbarrier/flag wait exceeded its iteration cap
  kDevErrBadIndex = 2,      // a token id / target outside [0, vocab)
};

inline size_t dtype_size(magma_dtype_t t) {
  switch (t) {
    case MAGMA_DTYPE_F32: return 4;
    case MAGMA_DTYPE_BF16: return 2;
    case MAGMA_DTYPE_S32: return 4;
    case MAGMA_DTYPE_S64: return 8;
    default: return 0;
  }
}

inline bool is_float_dtype(magma_dtype_t t) {
  return t == MAGMA_DTYPE_F32 || t == MAGMA_DTYPE_BF16;
}

inline const char* dtype_name(magma_dtype_t t) {
  switch (t) {
    case MAGMA_DTYPE_F32: return "F32";
    case MAGMA_DTYPE_BF16: return "BF16";
    case MAGMA_DTYPE_S32: return "S32";
    case MAGMA_DTYPE_S64: return "S64";
    default: return "UNSUPPORTED";
  }
}

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---- element load/store as F32 -------------------------------------------
__device__ __forceinline__ float to_f32(float x) { return x; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}

// Loads 8 consecutive elements (16 B for BF16, 32 B for F32) as F32.
// The address must be aligned to the vector size.
__device__ __forceinline__ void load8(const float* p, float (&v)[8]) {
  float4 a = *reinterpret_cast<const float4*>(p);
  float4 b = *reinterpret_cast<const float4*>(p + 4);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&v)[8]) {
  uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ void store8(float* p, const float (&v)[8]) {
  *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  *reinterpret_cast<float4*>(p + 4) = make_float4(v[4], v[5], v[6], v[7]);
}
__device__ __forceinline__ void store8(__nv_bfloat16* p, const float (&v)[8]) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = u;
}

// Four consecutive elements (16 B for F32, 8 B for BF16), aligned to that.
__device__ __forceinline__ void load4(const float* p, float (&v)[4]) {
  const float4 a = *reinterpret_cast<const float4*>(p);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
}
__device__ __forceinline__ void load4(const __nv_bfloat16* p, float (&v)[4]) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const float2 lo = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
  const float2 hi = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
  v[0] = lo.x; v[1] = lo.y; v[2] = hi.x; v[3] = hi.y;
}
__device__ __forceinline__ void store4(float* p, const float (&v)[4]) {
  *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
}
__device__ __forceinline__ void store4(__nv_bfloat16* p, const float (&v)[4]) {
  uint2 u;
  *reinterpret_cast<__nv_bfloat162*>(&u.x) = __floats2bfloat162_rn(v[0], v[1]);
  *reinterpret_cast<__nv_bfloat162*>(&u.y) = __floats2bfloat162_rn(v[2], v[3]);
  *reinterpret_cast<uint2*>(p) = u;
}

// Two consecutive elements (an 8-B F32 pair or a 4-B BF16 pair).
__device__ __forceinline__ void load2(const float* p, float& a, float& b) {
  const float2 v = *reinterpret_cast<const float2*>(p);
  a = v.x;
  b = v.y;
}
__device__ __forceinline__ void load2(const __nv_bfloat16* p, float& a, float& b) {
  const float2 v = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
  a = v.x;
  b = v.y;
}
__device__ __forceinline__ void store2(float* p, float a, float b) {
  *reinterpret_cast<float2*>(p) = make_float2(a, b);
}
__device__ __forceinline__ void store2(__nv_bfloat16* p, float a, float b) {
  *reinterpret_cast<__nv_bfloat162*>(p) = __floats2bfloat162_rn(a, b);
}

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}
__device__ __forceinline__ float warp_max(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
  return x;
}

// Records the first device-side error (later errors keep the first code).
__device__ __forceinline__ void set_device_error(int* word, int code) {
  if (word != nullptr) atomicCAS(word, 0, code);
}

// GELU, tanh form, in the op order of StableHLOEmitter.swift:804-816:
//   x3 = x*(x*x); inner = x + 0.044715*x3; t = tanh(0.7978845608*inner);
//   y = 0.5*(x*(1+t)).
__device__ __forceinline__ float gelu_f(float x) {
  float x3 = __fmul_rn(x, __fmul_rn(x, x));
  float inner = __fadd_rn(x, __fmul_rn(0.044715f, x3));
  float t = tanhf(__fmul_rn(0.7978845608f, inner));
  return __fmul_rn(0.5f, __fmul_rn(x, __fadd_rn(1.0f, t)));
}
// GELU derivative, Autodiff.swift:401-418:
//   u = c*(x + a*x^3); t = tanh(u); u' = c*(1 + 3a*x^2);
//   g' = 0.5*(1+t) + 0.5*x*(1-t*t)*u'.
__device__ __forceinline__ float gelu_grad_f(float x) {
  const float c = 0.7978845608f, a = 0.044715f;
  float x2 = __fmul_rn(x, x);
  float u = __fmul_rn(c, __fadd_rn(x, __fmul_rn(a, __fmul_rn(x2, x))));
  float t = tanhf(u);
  float up = __fmul_rn(c, __fadd_rn(1.0f, __fmul_rn(__fmul_rn(3.0f, a), x2)));
  float left = __fmul_rn(0.5f, __fadd_rn(1.0f, t));
  float right = __fmul_rn(__fmul_rn(__fmul_rn(0.5f, x), __fsub_rn(1.0f, __fmul_rn(t, t))), up);
  return __fadd_rn(left, right);
}

// Hardware tanh approximation (max relative error ~2^-11): used where the
// result is rounded to BF16 anyway.
__device__ __forceinline__ float tanh_approx(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// GELU / GELU' with the hardware tanh, same op order as gelu_f / gelu_grad_f.
__device__ __forceinline__ float gelu_fast(float x) {
  float inner = x + 0.044715f * (x * (x * x));
  float t = tanh_approx(0.7978845608f * inner);
  return 0.5f * (x * (1.0f + t));
}
__device__ __forceinline__ float gelu_grad_fast(float x) {
  const float c = 0.7978845608f, a = 0.044715f;
  float x2 = x * x;
  float t = tanh_approx(c * (x + a * (x2 * x)));
  float up = c * (1.0f + (3.0f * a) * x2);
  return 0.5f * (1.0f + t) + ((0.5f * x) * (1.0f - t * t)) * up;
}

// Pairs of F32 values in one 64-bit register for the sm_100 packed F32 ops
// (fma/mul/add .rn.f32x2: two independent IEEE operations per instruction).
__device__ __forceinline__ unsigned long long f2_pack(float a, float b) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2_unpack(unsigned long long v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ unsigned long long f2_fma(unsigned long long a, unsigned long long b,
                                                     unsigned long long c) {
  unsigned long long d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ unsigned long long f2_mul(unsigned long long a, unsigned long long b) {
  unsigned long long d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ unsigned long long f2_add(unsigned long long a, unsigned long long b) {
  unsigned long long d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ unsigned long long f2_sub(unsigned long long a, unsigned long long b) {
  unsigned long long d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// GELU and GELU' of two values for BF16 outputs, on packed F32 pairs, with
// the hardware tanh. The tanh argument is formed as x * (c + (a*c) * x^2)
// (the same quantity as c * (x + a * x^3), in fewer roundings), then
//   gelu  = x * (0.5 + 0.5 * t),
//   gelu' = (0.5 + 0.5 * t) + (0.5 * x * (1 - t^2)) * (c + 3ac * x^2);
// the difference from gelu_fast / gelu_grad_fast is far below a BF16 ulp.
__device__ __forceinline__ void gelu_pair_fast(float& y0, float& y1, float x0, float x1) {
  const float c = 0.7978845608f, ac = 0.044715f * 0.7978845608f;
  const unsigned long long X = f2_pack(x0, x1);
  const unsigned long long P = f2_fma(f2_mul(X, X), f2_pack(ac, ac), f2_pack(c, c));
  float u0, u1;
  f2_unpack(f2_mul(X, P), u0, u1);
  const unsigned long long T = f2_pack(tanh_approx(u0), tanh_approx(u1));
  const unsigned long long H = f2_fma(T, f2_pack(0.5f, 0.5f), f2_pack(0.5f, 0.5f));
  f2_unpack(f2_mul(X, H), y0, y1);
}
__device__ __forceinline__ void gelu_grad_pair_fast(float& g0, float& g1, float x0, float x1) {
  const float c = 0.7978845608f, ac = 0.044715f * 0.7978845608f;
  const unsigned long long X = f2_pack(x0, x1);
  const unsigned long long X2 = f2_mul(X, X);
  const unsigned long long P = f2_fma(X2, f2_pack(ac, ac), f2_pack(c, c));
  float u0, u1;
  f2_unpack(f2_mul(X, P), u0, u1);
  const unsigned long long T = f2_pack(tanh_approx(u0), tanh_approx(u1));
  const unsigned long long Q = f2_fma(X2, f2_pack(3.0f * ac, 3.0f * ac), f2_pack(c, c));
  const unsigned long long M = f2_fma(T, T, f2_pack(-1.0f, -1.0f));            // t^2 - 1
  const unsigned long long R = f2_mul(f2_mul(X, f2_pack(-0.5f, -0.5f)), M);   // 0.5 x (1 - t^2)
  const unsigned long long H = f2_fma(T, f2_pack(0.5f, 0.5f), f2_pack(0.5f, 0.5f));
  f2_unpack(f2_fma(R, Q, H), g0, g1);
}

// GELU variants by output precision: the accurate form for F32 outputs, the
// hardware-tanh form when the result is stored as BF16.
template <typename T> __device__ __forceinline__ float gelu_t(float x) { return gelu_f(x); }
template <> __device__ __forceinline__ float gelu_t<__nv_bfloat16>(float x) { return gelu_fast(x); }
template <typename T> __device__ __forceinline__ float gelu_grad_t(float x) { return gelu_grad_f(x); }
template <> __device__ __forceinline__ float gelu_grad_t<__nv_bfloat16>(float x) {
  return gelu_grad_fast(x);
}

}  // namespace magma

// Argument-check helper used at the top of every entry point.
#define MAGMA_REQUIRE(cond, ...)                                   \
  do {                                                             \
    if (!(cond)) return ::magma::fail(MAGMA_INVALID_ARGUMENT, __VA_ARGS__); \
  } while (0)
