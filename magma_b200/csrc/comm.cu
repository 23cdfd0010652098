// Collectives and events of the C ABI: the data-parallel exchange of a
// training step, over NCCL (NVLink / NVSwitch within one box).
//
// The reference runs a replicated step through PJRT_ExecuteMultiDevice
// (Sources/CXLARuntime/PJRTSimpleWrapper.c:1412) with the gradient mean traced
// as crossReplicaMean (Sources/Core/Distributed.swift:59-64), lowered to an
// all_reduce add followed by a multiply by 1/n
// (Sources/StableHLO/Builder/MLIRBuilder.swift:923-929). Here the caller holds
// one communicator per GPU (one process per GPU, or one process driving all of
// them) and issues the collectives on its own streams; the 1/n multiply is
// left to the consumer (the Adam kernels take it as grad_scale).
//
// NCCL is opened at run time (dlopen of libnccl.so.2: in a process that
// already loaded NCCL, such as one running PyTorch, the same library is used),
// so the shared library carries no link-time NCCL dependency and reports
// MAGMA_UNAVAILABLE where NCCL is missing. Communicators are created
// non-blocking, so that initialisation and every enqueue wait a bounded time:
// a peer that never joins, or has died, ends the call with
// MAGMA_DEADLINE_EXCEEDED (the communicator is then aborted) instead of a hang.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>

#include "common.cuh"

namespace magma {
namespace {

struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*);
  ncclResult_t (*comm_init_rank_config)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*);
  ncclResult_t (*comm_init_all)(ncclComm_t*, int, const int*);
  ncclResult_t (*comm_finalize)(ncclComm_t);
  ncclResult_t (*comm_destroy)(ncclComm_t);
  ncclResult_t (*comm_abort)(ncclComm_t);
  ncclResult_t (*comm_get_async_error)(ncclComm_t, ncclResult_t*);
  ncclResult_t (*comm_count)(const ncclComm_t, int*);
  ncclResult_t (*comm_user_rank)(const ncclComm_t, int*);
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t);
  ncclResult_t (*reduce_scatter)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t,
                                 ncclComm_t, cudaStream_t);
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                             cudaStream_t);
  ncclResult_t (*group_start)();
  ncclResult_t (*group_end)();
  const char* (*get_error_string)(ncclResult_t);
  ncclResult_t (*get_version)(int*);
};

NcclApi g_nccl;
bool g_nccl_ok = false;
std::string g_nccl_why;
std::once_flag g_nccl_once;

template <typename F>
bool sym(void* h, const char* name, F* out) {
  *out = reinterpret_cast<F>(dlsym(h, name));
  return *out != nullptr;
}

void open_nccl() {
  void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (h == nullptr) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
  if (h == nullptr) {
    const char* e = dlerror();
    g_nccl_why = std::string("cannot open libnccl.so.2: ") + (e ? e : "not found");
    return;
  }
  NcclApi a;
  const bool ok =
      sym(h, "ncclGetUniqueId", &a.get_unique_id) &&
      sym(h, "ncclCommInitRankConfig", &a.comm_init_rank_config) &&
      sym(h, "ncclCommInitAll", &a.comm_init_all) && sym(h, "ncclCommFinalize", &a.comm_finalize) &&
      sym(h, "ncclCommDestroy", &a.comm_destroy) && sym(h, "ncclCommAbort", &a.comm_abort) &&
      sym(h, "ncclCommGetAsyncError", &a.comm_get_async_error) &&
      sym(h, "ncclCommCount", &a.comm_count) && sym(h, "ncclCommUserRank", &a.comm_user_rank) &&
      sym(h, "ncclAllReduce", &a.all_reduce) && sym(h, "ncclReduceScatter", &a.reduce_scatter) &&
      sym(h, "ncclAllGather", &a.all_gather) && sym(h, "ncclGroupStart", &a.group_start) &&
      sym(h, "ncclGroupEnd", &a.group_end) && sym(h, "ncclGetErrorString", &a.get_error_string) &&
      sym(h, "ncclGetVersion", &a.get_version);
  if (!ok) {
    g_nccl_why = "libnccl.so.2 lacks a required entry point (NCCL >= 2.18 needed)";
    return;
  }
  g_nccl = a;
  g_nccl_ok = true;
}

magma_status_t nccl() {
  std::call_once(g_nccl_once, open_nccl);
  if (!g_nccl_ok) return fail(MAGMA_UNAVAILABLE, "NCCL unavailable: %s", g_nccl_why.c_str());
  return MAGMA_OK;
}

magma_status_t nccl_status(ncclResult_t r, const char* what) {
  if (r == ncclSuccess) return MAGMA_OK;
  magma_status_t code = MAGMA_INTERNAL;
  if (r == ncclInvalidArgument || r == ncclInvalidUsage) code = MAGMA_INVALID_ARGUMENT;
  else if (r == ncclSystemError || r == ncclRemoteError) code = MAGMA_UNAVAILABLE;
  return fail(code, "%s: %s (ncclResult %d)", what, g_nccl.get_error_string(r), (int)r);
}

// Default bound on a communicator operation's host-side wait.
constexpr int64_t kDefaultTimeoutMs = 120000;

// Polls a non-blocking communicator until its pending operation leaves
// ncclInProgress; past the deadline the communicator is aborted.
magma_status_t wait_comm(ncclComm_t comm, ncclResult_t r, int64_t timeout_ms, const char* what) {
  if (r != ncclSuccess && r != ncclInProgress) return nccl_status(r, what);
  const auto deadline = std::chrono::steady_clock::now() +
                        std::chrono::milliseconds(timeout_ms > 0 ? timeout_ms : kDefaultTimeoutMs);
  for (;;) {
    ncclResult_t st = ncclSuccess;
    ncclResult_t q = g_nccl.comm_get_async_error(comm, &st);
    if (q != ncclSuccess) return nccl_status(q, "ncclCommGetAsyncError");
    if (st == ncclSuccess) return MAGMA_OK;
    if (st != ncclInProgress) return nccl_status(st, what);
    if (std::chrono::steady_clock::now() > deadline) {
      g_nccl.comm_abort(comm);
      return fail(MAGMA_DEADLINE_EXCEEDED, "%s: no progress within %lld ms; communicator aborted",
                  what, (long long)(timeout_ms > 0 ? timeout_ms : kDefaultTimeoutMs));
    }
    std::this_thread::sleep_for(std::chrono::microseconds(200));
  }
}

bool nccl_dtype(magma_dtype_t dt, ncclDataType_t* out) {
  switch (dt) {
    case MAGMA_DTYPE_F32: *out = ncclFloat32; return true;
    case MAGMA_DTYPE_BF16: *out = ncclBfloat16; return true;
    case MAGMA_DTYPE_S32: *out = ncclInt32; return true;
    case MAGMA_DTYPE_S64: *out = ncclInt64; return true;
    default: return false;
  }
}

bool nccl_op(int32_t op, ncclRedOp_t* out) {
  switch (op) {
    case MAGMA_REDUCE_SUM: *out = ncclSum; return true;
    case MAGMA_REDUCE_MAX: *out = ncclMax; return true;
    case MAGMA_REDUCE_MIN: *out = ncclMin; return true;
    case MAGMA_REDUCE_AVG: *out = ncclAvg; return true;
    default: return false;
  }
}

}  // namespace
}  // namespace magma

using namespace magma;

extern "C" {

magma_status_t magma_comm_unique_id(uint8_t* id, size_t bytes) {
  MAGMA_REQUIRE(id != nullptr && bytes >= MAGMA_COMM_ID_BYTES,
                "magma_comm_unique_id: a buffer of %d bytes is needed", MAGMA_COMM_ID_BYTES);
  if (magma_status_t st = nccl()) return st;
  ncclUniqueId u;
  if (magma_status_t st = nccl_status(g_nccl.get_unique_id(&u), "ncclGetUniqueId")) return st;
  static_assert(sizeof(u) == MAGMA_COMM_ID_BYTES, "NCCL unique id size");
  memcpy(id, &u, sizeof(u));
  return MAGMA_OK;
}

magma_status_t magma_comm_init_rank(void** comm, int32_t nranks, int32_t rank, const uint8_t* id,
                                    int64_t timeout_ms) {
  MAGMA_REQUIRE(comm != nullptr && id != nullptr, "magma_comm_init_rank: NULL pointer");
  MAGMA_REQUIRE(nranks >= 1 && rank >= 0 && rank < nranks,
                "magma_comm_init_rank: rank %d of %d", rank, nranks);
  *comm = nullptr;
  if (magma_status_t st = nccl()) return st;
  ncclUniqueId u;
  memcpy(&u, id, sizeof(u));
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  ncclComm_t c = nullptr;
  ncclResult_t r = g_nccl.comm_init_rank_config(&c, nranks, u, rank, &cfg);
  if (c == nullptr) return nccl_status(r == ncclSuccess ? ncclInternalError : r,
                                       "ncclCommInitRankConfig");
  if (magma_status_t st = wait_comm(c, r, timeout_ms, "magma_comm_init_rank")) return st;
  *comm = c;
  return MAGMA_OK;
}

magma_status_t magma_comm_init_all(int32_t ndev, const int32_t* devices, void** comms) {
  MAGMA_REQUIRE(ndev >= 1 && comms != nullptr, "magma_comm_init_all: bad arguments");
  if (magma_status_t st = nccl()) return st;
  return nccl_status(g_nccl.comm_init_all(reinterpret_cast<ncclComm_t*>(comms), ndev, devices),
                     "ncclCommInitAll");
}

magma_status_t magma_comm_destroy(void* comm) {
  if (comm == nullptr) return MAGMA_OK;
  if (magma_status_t st = nccl()) return st;
  ncclComm_t c = static_cast<ncclComm_t>(comm);
  magma_status_t st = wait_comm(c, g_nccl.comm_finalize(c), kDefaultTimeoutMs,
                                "magma_comm_destroy (finalize)");
  if (st == MAGMA_DEADLINE_EXCEEDED) return st;  // aborted (and freed) by wait_comm
  ncclResult_t r = g_nccl.comm_destroy(c);
  return st != MAGMA_OK ? st : nccl_status(r, "ncclCommDestroy");
}

magma_status_t magma_comm_abort(void* comm) {
  if (comm == nullptr) return MAGMA_OK;
  if (magma_status_t st = nccl()) return st;
  return nccl_status(g_nccl.comm_abort(static_cast<ncclComm_t>(comm)), "ncclCommAbort");
}

magma_status_t magma_comm_size(void* comm, int32_t* nranks) {
  MAGMA_REQUIRE(comm != nullptr && nranks != nullptr, "magma_comm_size: NULL pointer");
  if (magma_status_t st = nccl()) return st;
  int n = 0;
  if (magma_status_t st = nccl_status(g_nccl.comm_count(static_cast<ncclComm_t>(comm), &n),
                                      "ncclCommCount"))
    return st;
  *nranks = n;
  return MAGMA_OK;
}

magma_status_t magma_comm_rank(void* comm, int32_t* rank) {
  MAGMA_REQUIRE(comm != nullptr && rank != nullptr, "magma_comm_rank: NULL pointer");
  if (magma_status_t st = nccl()) return st;
  int r = 0;
  if (magma_status_t st = nccl_status(g_nccl.comm_user_rank(static_cast<ncclComm_t>(comm), &r),
                                      "ncclCommUserRank"))
    return st;
  *rank = r;
  return MAGMA_OK;
}

magma_status_t magma_comm_check(void* comm) {
  MAGMA_REQUIRE(comm != nullptr, "magma_comm_check: NULL communicator");
  if (magma_status_t st = nccl()) return st;
  ncclResult_t st = ncclSuccess;
  if (magma_status_t s = nccl_status(
          g_nccl.comm_get_async_error(static_cast<ncclComm_t>(comm), &st), "ncclCommGetAsyncError"))
    return s;
  if (st == ncclSuccess || st == ncclInProgress) return MAGMA_OK;
  return nccl_status(st, "communicator error");
}

magma_status_t magma_allreduce(const void* send, void* recv, int64_t count, magma_dtype_t dtype,
                               int32_t op, void* comm, void* stream) {
  MAGMA_REQUIRE(count >= 0 && comm != nullptr, "magma_allreduce: bad arguments");
  MAGMA_REQUIRE(count == 0 || (send && recv), "magma_allreduce: NULL buffer");
  ncclDataType_t t;
  ncclRedOp_t o;
  MAGMA_REQUIRE(nccl_dtype(dtype, &t), "magma_allreduce: unsupported dtype %s", dtype_name(dtype));
  MAGMA_REQUIRE(nccl_op(op, &o), "magma_allreduce: unknown reduction %d", op);
  if (magma_status_t st = nccl()) return st;
  ncclComm_t c = static_cast<ncclComm_t>(comm);
  return wait_comm(c, g_nccl.all_reduce(send, recv, (size_t)count, t, o, c, (cudaStream_t)stream),
                   kDefaultTimeoutMs, "magma_allreduce");
}

magma_status_t magma_reduce_scatter(const void* send, void* recv, int64_t recv_count,
                                    magma_dtype_t dtype, int32_t op, void* comm, void* stream) {
  MAGMA_REQUIRE(recv_count >= 0 && comm != nullptr, "magma_reduce_scatter: bad arguments");
  MAGMA_REQUIRE(recv_count == 0 || (send && recv), "magma_reduce_scatter: NULL buffer");
  ncclDataType_t t;
  ncclRedOp_t o;
  MAGMA_REQUIRE(nccl_dtype(dtype, &t), "magma_reduce_scatter: unsupported dtype %s",
                dtype_name(dtype));
  MAGMA_REQUIRE(nccl_op(op, &o), "magma_reduce_scatter: unknown reduction %d", op);
  if (magma_status_t st = nccl()) return st;
  ncclComm_t c = static_cast<ncclComm_t>(comm);
  return wait_comm(c, g_nccl.reduce_scatter(send, recv, (size_t)recv_count, t, o, c,
                                            (cudaStream_t)stream),
                   kDefaultTimeoutMs, "magma_reduce_scatter");
}

magma_status_t magma_all_gather(const void* send, void* recv, int64_t send_count,
                                magma_dtype_t dtype, void* comm, void* stream) {
  MAGMA_REQUIRE(send_count >= 0 && comm != nullptr, "magma_all_gather: bad arguments");
  MAGMA_REQUIRE(send_count == 0 || (send && recv), "magma_all_gather: NULL buffer");
  ncclDataType_t t;
  MAGMA_REQUIRE(nccl_dtype(dtype, &t), "magma_all_gather: unsupported dtype %s",
                dtype_name(dtype));
  if (magma_status_t st = nccl()) return st;
  ncclComm_t c = static_cast<ncclComm_t>(comm);
  return wait_comm(c, g_nccl.all_gather(send, recv, (size_t)send_count, t, c,
                                        (cudaStream_t)stream),
                   kDefaultTimeoutMs, "magma_all_gather");
}

magma_status_t magma_group_start(void) {
  if (magma_status_t st = nccl()) return st;
  return nccl_status(g_nccl.group_start(), "ncclGroupStart");
}

magma_status_t magma_group_end(void) {
  if (magma_status_t st = nccl()) return st;
  ncclResult_t r = g_nccl.group_end();
  return r == ncclInProgress ? MAGMA_OK : nccl_status(r, "ncclGroupEnd");
}

// ---- events --------------------------------------------------------------
magma_status_t magma_event_create(void** event, int32_t enable_timing) {
  MAGMA_REQUIRE(event != nullptr, "magma_event_create: NULL pointer");
  cudaEvent_t e = nullptr;
  if (magma_status_t st = cuda_status(
          cudaEventCreateWithFlags(&e, enable_timing ? cudaEventDefault : cudaEventDisableTiming),
          "cudaEventCreate"))
    return st;
  *event = e;
  return MAGMA_OK;
}

magma_status_t magma_event_destroy(void* event) {
  if (event == nullptr) return MAGMA_OK;
  return cuda_status(cudaEventDestroy(static_cast<cudaEvent_t>(event)), "cudaEventDestroy");
}

magma_status_t magma_event_record(void* event, void* stream) {
  MAGMA_REQUIRE(event != nullptr, "magma_event_record: NULL event");
  return cuda_status(cudaEventRecord(static_cast<cudaEvent_t>(event), (cudaStream_t)stream),
                     "cudaEventRecord");
}

magma_status_t magma_stream_wait_event(void* stream, void* event) {
  MAGMA_REQUIRE(event != nullptr, "magma_stream_wait_event: NULL event");
  return cuda_status(cudaStreamWaitEvent((cudaStream_t)stream, static_cast<cudaEvent_t>(event), 0),
                     "cudaStreamWaitEvent");
}

magma_status_t magma_event_synchronize(void* event) {
  MAGMA_REQUIRE(event != nullptr, "magma_event_synchronize: NULL event");
  return cuda_status(cudaEventSynchronize(static_cast<cudaEvent_t>(event)),
                     "cudaEventSynchronize");
}

magma_status_t magma_event_query(void* event, int32_t* done) {
  MAGMA_REQUIRE(event != nullptr && done != nullptr, "magma_event_query: NULL pointer");
  cudaError_t e = cudaEventQuery(static_cast<cudaEvent_t>(event));
  if (e == cudaErrorNotReady) {
    cudaGetLastError();
    *done = 0;
    return MAGMA_OK;
  }
  *done = 1;
  return cuda_status(e, "cudaEventQuery");
}

magma_status_t magma_event_elapsed_ms(void* start, void* end, float* ms) {
  MAGMA_REQUIRE(start && end && ms, "magma_event_elapsed_ms: NULL pointer");
  return cuda_status(cudaEventElapsedTime(ms, static_cast<cudaEvent_t>(start),
                                          static_cast<cudaEvent_t>(end)),
                     "cudaEventElapsedTime");
}

}  // extern "C"
