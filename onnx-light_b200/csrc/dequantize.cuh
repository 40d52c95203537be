// DequantizeLinear parameters and validation shared with the fused kernels.
#pragma once
#include "b2_common.cuh"

namespace b2 {

struct DqParams {
  const uint8_t *x;
  const uint8_t *scale; // FLOAT or FLOAT16 storage
  const uint8_t *zp;    // nullable, dtype == x dtype
  void *y;
  int64_t n;
  int64_t inner, alen, s_alen, block;
  int layout; // 0 per-tensor, 1 per-axis, 2 blocked
  int xdt;
  int f16;    // scale/output FLOAT16
  uint32_t use32; // n < 2^31: 32-bit index math
  FastDiv div_inner, div_alen, div_block;
};

// Validates a DequantizeLinear call in the reference's order
// (kernel_dequantizelinear.cc:332-693) and fills everything but the pointers.
int dq_validate(const b2_tensor *x, const b2_tensor *s, const b2_tensor *zp, int64_t axis,
                int32_t out_dtype, const std::vector<int64_t> &out_shape, DqParams &p);
int dq_launch(const DqParams &p, cudaStream_t stream);

} // namespace b2
