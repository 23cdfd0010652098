// Runtime part of the C ABI: last-error plumbing, device selection, streams,
// memory and the device-side error word. Mirrors the client/buffer surface of
// Magma's PJRT shim (Sources/CXLARuntime/PJRTSimpleWrapper.c: PJRT_CreateClient
// :248, PJRT_CreateBuffer :551, PJRT_BufferToHost :714) without XLA: buffers are
// raw device pointers and the caller owns them.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "common.cuh"

namespace {

thread_local std::string t_last_error;
thread_local bool t_has_error = false;

constexpr int kMaxDevices = 64;
int g_sm_count[kMaxDevices] = {0};
int* g_error_word[kMaxDevices] = {nullptr};
std::mutex g_device_mu;

}  // namespace

// One error word per device; kernels with bounded waits write it on timeout.
__device__ int g_magma_device_error_word;

namespace magma {

magma_status_t fail(magma_status_t code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error.assign(buf);
  t_has_error = true;
  return code;
}

magma_status_t cuda_status(cudaError_t err, const char* what) {
  if (err == cudaSuccess) return MAGMA_OK;
  magma_status_t code = MAGMA_INTERNAL;
  if (err == cudaErrorMemoryAllocation) code = MAGMA_RESOURCE_EXHAUSTED;
  else if (err == cudaErrorInvalidValue || err == cudaErrorInvalidDevicePointer ||
           err == cudaErrorInvalidConfiguration)
    code = MAGMA_INVALID_ARGUMENT;
  else if (err == cudaErrorNoDevice || err == cudaErrorInsufficientDriver ||
           err == cudaErrorInvalidDevice)
    code = MAGMA_UNAVAILABLE;
  return fail(code, "%s: %s (%s)", what, cudaGetErrorString(err), cudaGetErrorName(err));
}

int num_sms() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
  if (g_sm_count[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    g_sm_count[dev] = n;
  }
  return g_sm_count[dev];
}

int* device_error_word() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  if (g_error_word[dev] == nullptr) {
    std::lock_guard<std::mutex> lock(g_device_mu);
    if (g_error_word[dev] == nullptr) {
      void* p = nullptr;
      if (cudaGetSymbolAddress(&p, g_magma_device_error_word) != cudaSuccess) return nullptr;
      g_error_word[dev] = static_cast<int*>(p);
    }
  }
  return g_error_word[dev];
}

}  // namespace magma

using namespace magma;

extern "C" {

const char* magma_get_last_error_message(void) {
  return t_has_error ? t_last_error.c_str() : nullptr;
}

void magma_clear_last_error_message(void) {
  t_last_error.clear();
  t_has_error = false;
}

int32_t magma_abi_version(void) { return 100; /* 0.1.0 */ }

magma_status_t magma_device_count(int32_t* count) {
  MAGMA_REQUIRE(count != nullptr, "magma_device_count: count is NULL");
  int n = 0;
  cudaError_t err = cudaGetDeviceCount(&n);
  if (err == cudaErrorNoDevice || err == cudaErrorInsufficientDriver) {
    cudaGetLastError();
    *count = 0;
    return MAGMA_OK;
  }
  if (magma_status_t s = cuda_status(err, "cudaGetDeviceCount")) return s;
  *count = n;
  return MAGMA_OK;
}

magma_status_t magma_init(int32_t device_ordinal) {
  int n = 0;
  cudaError_t err = cudaGetDeviceCount(&n);
  if (err != cudaSuccess) {
    cudaGetLastError();
    return fail(MAGMA_UNAVAILABLE, "magma_init: no CUDA device available (%s)",
                cudaGetErrorString(err));
  }
  if (device_ordinal < 0 || device_ordinal >= n || device_ordinal >= kMaxDevices)
    return fail(MAGMA_INVALID_ARGUMENT, "magma_init: device ordinal %d out of range [0, %d)",
                device_ordinal, n);
  if (magma_status_t s = cuda_status(cudaSetDevice(device_ordinal), "cudaSetDevice")) return s;
  cudaDeviceProp prop;
  if (magma_status_t s = cuda_status(cudaGetDeviceProperties(&prop, device_ordinal),
                                     "cudaGetDeviceProperties"))
    return s;
  if (prop.major != 10)
    return fail(MAGMA_FAILED_PRECONDITION,
                "magma_init: device %d is sm_%d%d (%s); this library is built for sm_100a only",
                device_ordinal, prop.major, prop.minor, prop.name);
  g_sm_count[device_ordinal] = prop.multiProcessorCount;
  if (device_error_word() == nullptr)
    return fail(MAGMA_INTERNAL, "magma_init: cannot resolve the device error word");
  return MAGMA_OK;
}

magma_status_t magma_stream_create(void** stream) {
  MAGMA_REQUIRE(stream != nullptr, "magma_stream_create: stream is NULL");
  cudaStream_t s = nullptr;
  if (magma_status_t st = cuda_status(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking),
                                      "cudaStreamCreate"))
    return st;
  *stream = s;
  return MAGMA_OK;
}

magma_status_t magma_stream_destroy(void* stream) {
  MAGMA_REQUIRE(stream != nullptr, "magma_stream_destroy: stream is NULL");
  return cuda_status(cudaStreamDestroy(static_cast<cudaStream_t>(stream)), "cudaStreamDestroy");
}

magma_status_t magma_stream_synchronize(void* stream) {
  return cuda_status(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)),
                     "cudaStreamSynchronize");
}

magma_status_t magma_malloc(void** ptr, size_t bytes) {
  MAGMA_REQUIRE(ptr != nullptr, "magma_malloc: ptr is NULL");
  *ptr = nullptr;
  if (bytes == 0) return MAGMA_OK;
  return cuda_status(cudaMalloc(ptr, bytes), "cudaMalloc");
}

magma_status_t magma_free(void* ptr) {
  if (ptr == nullptr) return MAGMA_OK;
  return cuda_status(cudaFree(ptr), "cudaFree");
}

magma_status_t magma_memcpy_h2d(void* dst, const void* src, size_t bytes, void* stream) {
  if (bytes == 0) return MAGMA_OK;
  MAGMA_REQUIRE(dst != nullptr && src != nullptr, "magma_memcpy_h2d: NULL pointer");
  return cuda_status(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice,
                                     static_cast<cudaStream_t>(stream)),
                     "cudaMemcpyAsync(H2D)");
}

magma_status_t magma_memcpy_d2h(void* dst, const void* src, size_t bytes, void* stream) {
  if (bytes == 0) return MAGMA_OK;
  MAGMA_REQUIRE(dst != nullptr && src != nullptr, "magma_memcpy_d2h: NULL pointer");
  return cuda_status(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost,
                                     static_cast<cudaStream_t>(stream)),
                     "cudaMemcpyAsync(D2H)");
}

magma_status_t magma_memset(void* dst, int32_t value, size_t bytes, void* stream) {
  if (bytes == 0) return MAGMA_OK;
  MAGMA_REQUIRE(dst != nullptr, "magma_memset: NULL pointer");
  return cuda_status(cudaMemsetAsync(dst, value, bytes, static_cast<cudaStream_t>(stream)),
                     "cudaMemsetAsync");
}

magma_status_t magma_device_error_check(void* stream, int32_t* code) {
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (magma_status_t st = cuda_status(cudaStreamSynchronize(s), "cudaStreamSynchronize"))
    return st;
  int* word = device_error_word();
  if (word == nullptr) return fail(MAGMA_INTERNAL, "device error word unavailable");
  int host = 0;
  if (magma_status_t st = cuda_status(cudaMemcpy(&host, word, sizeof(int), cudaMemcpyDeviceToHost),
                                      "read device error word"))
    return st;
  if (code != nullptr) *code = host;
  if (host != kDevErrNone) {
    int zero = 0;
    cudaMemcpy(word, &zero, sizeof(int), cudaMemcpyHostToDevice);
    if (host == kDevErrWaitTimeout)
      return fail(MAGMA_DEADLINE_EXCEEDED, "a device-side wait exceeded its iteration limit");
    if (host == kDevErrBadIndex)
      return fail(MAGMA_OUT_OF_RANGE, "a kernel met an index outside its table");
    return fail(MAGMA_INTERNAL, "device error code %d", host);
  }
  return MAGMA_OK;
}

}  // extern "C"
