// MatMulInteger / QLinearMatMul on tcgen05 kind::i8 tensor cores.
#include "imma.cuh"

namespace b2 {

bool imma_tc_supported(const ImmaParams &) { return false; }
size_t imma_tc_workspace(const ImmaParams &) { return 0; }
int imma_tc_launch(const ImmaParams &, void *, cudaStream_t) {
  B2_FAIL(B2_ERR_UNSUPPORTED, "tensor-core integer GEMM not built");
}

} // namespace b2
