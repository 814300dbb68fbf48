// Host side of the tensor-core path: TMA tensor-map encoding through the
// runtime's driver entry point, so the library needs no link against libcuda.
#include <mutex>

#include "tc_common.cuh"

namespace msa {
namespace tc {

namespace {
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_once;
cudaError_t g_status = cudaSuccess;
}  // namespace

int encode_tensor_map(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base, const uint64_t* dims,
                      const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle) {
  std::call_once(g_once, [] {
    cudaDriverEntryPointQueryResult q;
    void* fn = nullptr;
    g_status = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (g_status == cudaSuccess && q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (!g_encode) return set_error(MSA_ERR_CUDA, "cuTensorMapEncodeTiled unavailable (%s)", cudaGetErrorString(g_status));
  cuuint64_t gdim[5], gstride[4];
  cuuint32_t bdim[5], estride[5];
  for (int i = 0; i < rank; ++i) {
    gdim[i] = dims[i];
    bdim[i] = box[i];
    estride[i] = 1;
    if (i + 1 < rank) gstride[i] = strides_bytes[i];
  }
  CUresult r = g_encode(map, dtype, (cuuint32_t)rank, const_cast<void*>(base), gdim, gstride, bdim, estride,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(MSA_ERR_CUDA, "cuTensorMapEncodeTiled failed (CUresult %d)", (int)r);
  return MSA_OK;
}

}  // namespace tc
}  // namespace msa
