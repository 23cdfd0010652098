// Host-side TMA descriptor encoding via the driver entry point that the CUDA
// runtime resolves (cuTensorMapEncodeTiled), cached once per process.
#include <cudaTypedefs.h>

#include <mutex>

#include "sm100.cuh"

namespace magma {
namespace {

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;
cudaError_t g_encode_err = cudaSuccess;

PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    g_encode_err = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (g_encode_err == cudaSuccess && q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  return g_encode;
}

}  // namespace

magma_status_t encode_tensor_map_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base,
                                    uint64_t inner, uint64_t outer, uint64_t row_stride_bytes,
                                    uint32_t box_inner, uint32_t box_outer,
                                    CUtensorMapSwizzle swizzle) {
  auto enc = get_encode();
  if (enc == nullptr)
    return fail(MAGMA_UNAVAILABLE, "cuTensorMapEncodeTiled unavailable (%s)",
                cudaGetErrorString(g_encode_err));
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(MAGMA_INVALID_ARGUMENT,
                "cuTensorMapEncodeTiled failed (%d): dims=(%llu,%llu) stride=%llu box=(%u,%u)",
                (int)r, (unsigned long long)inner, (unsigned long long)outer,
                (unsigned long long)row_stride_bytes, box_inner, box_outer);
  return MAGMA_OK;
}

magma_status_t encode_tensor_map_3d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base,
                                    const uint64_t dims_in[3], const uint64_t strides_bytes[2],
                                    const uint32_t box_in[3], CUtensorMapSwizzle swizzle) {
  auto enc = get_encode();
  if (enc == nullptr)
    return fail(MAGMA_UNAVAILABLE, "cuTensorMapEncodeTiled unavailable (%s)",
                cudaGetErrorString(g_encode_err));
  cuuint64_t dims[3] = {dims_in[0], dims_in[1], dims_in[2]};
  cuuint64_t strides[2] = {strides_bytes[0], strides_bytes[1]};
  cuuint32_t box[3] = {box_in[0], box_in[1], box_in[2]};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, dtype, 3, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(MAGMA_INVALID_ARGUMENT, "cuTensorMapEncodeTiled (3-D) failed (%d)", (int)r);
  return MAGMA_OK;
}

magma_status_t encode_tensor_map_nd(CUtensorMap* map, CUtensorMapDataType dtype, const void* base,
                                    int rank, const uint64_t* dims_in,
                                    const uint64_t* strides_bytes, const uint32_t* box_in,
                                    CUtensorMapSwizzle swizzle) {
  auto enc = get_encode();
  if (enc == nullptr)
    return fail(MAGMA_UNAVAILABLE, "cuTensorMapEncodeTiled unavailable (%s)",
                cudaGetErrorString(g_encode_err));
  if (rank < 1 || rank > 5) return fail(MAGMA_INVALID_ARGUMENT, "tensor map rank %d", rank);
  cuuint64_t dims[5], strides[4];
  cuuint32_t box[5], estr[5];
  for (int i = 0; i < rank; ++i) {
    dims[i] = dims_in[i];
    box[i] = box_in[i];
    estr[i] = 1;
    if (i + 1 < rank) strides[i] = strides_bytes[i];
  }
  CUresult r = enc(map, dtype, (cuuint32_t)rank, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(MAGMA_INVALID_ARGUMENT, "cuTensorMapEncodeTiled (%d-D) failed (%d)", rank, (int)r);
  return MAGMA_OK;
}

}  // namespace magma
