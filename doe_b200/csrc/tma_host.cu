// tma_host.cu -- tensor-map encoding for the TMA kernels (host side).
#include <mutex>

#include "tma.cuh"

namespace doe {

namespace {
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::mutex g_encode_mu;

int get_encoder(const char* who) {
  std::lock_guard<std::mutex> lock(g_encode_mu);
  if (g_encode) return DOE_OK;
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
  if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || fn == nullptr) {
    cudaGetLastError();
    set_op_error("%s: cuTensorMapEncodeTiled is not available from the driver", who);
    return DOE_CUDA_ERROR;
  }
  g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  return DOE_OK;
}
}  // namespace

int encode_rows_map(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, uint32_t elem_bytes,
                    uint64_t inner, uint64_t heads, uint64_t rows, uint32_t box_inner, uint32_t box_rows,
                    const char* who) {
  int rc = get_encoder(who);
  if (rc != DOE_OK) return rc;
  const cuuint64_t dims[3] = {inner, heads, rows};
  const cuuint64_t strides[2] = {inner * elem_bytes, heads * inner * elem_bytes};
  const cuuint32_t box[3] = {box_inner, 1, box_rows};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(map, dtype, 3, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_op_error("%s: cuTensorMapEncodeTiled failed (%d)", who, (int)r);
    return DOE_CUDA_ERROR;
  }
  return DOE_OK;
}

}  // namespace doe
