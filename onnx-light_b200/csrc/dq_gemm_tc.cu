// FLOAT16/BFLOAT16 fused dequant GEMM on tcgen05 tensor cores (M > 8).
#include "dq_matmul.cuh"

namespace b2 {

bool dq_tc_supported(const DqMmParams &) { return false; }
size_t dq_tc_workspace(const DqMmParams &) { return 0; }
int dq_tc_launch(const DqMmParams &, void *, cudaStream_t) {
  B2_FAIL(B2_ERR_UNSUPPORTED, "tensor-core dequant GEMM not built");
}

} // namespace b2
