// Host helpers for the tcgen05 kernels: tensor-map creation through the
// driver entry point, so the library needs no link-time libcuda dependency.
#include <cudaTypedefs.h>

#include "tc_common.cuh"

namespace b2 {

int make_tensor_map(CUtensorMap *map, CUtensorMapDataType dtype, int rank, const void *base,
                    const uint64_t *dims, const uint64_t *strides_bytes, const uint32_t *box,
                    CUtensorMapSwizzle swizzle) {
  static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  if (encode == nullptr) {
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    B2_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
    if (fn == nullptr || q != cudaDriverEntryPointSuccess)
      B2_FAIL(B2_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  cuuint32_t elem_strides[5] = {1, 1, 1, 1, 1};
  cuuint64_t d[5], s[4];
  cuuint32_t b[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    if (i + 1 < rank) s[i] = strides_bytes[i];
  }
  const CUresult r = encode(map, dtype, (cuuint32_t)rank, const_cast<void *>(base), d, s, b,
                            elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) B2_FAIL(B2_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return B2_OK;
}

} // namespace b2
