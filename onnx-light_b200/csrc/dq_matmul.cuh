// Parameters of the fused DequantizeLinear -> [Cast] -> MatMul kernels.
#pragma once
#include "b2_common.cuh"
#include "dequantize.cuh"

namespace b2 {

// Where the scale (and zero point) of weight element (k, n) of W[K, N] lives.
enum ScaleLayout : int {
  kScaleTensor = 0,     // one scale
  kScaleAxis0Block = 1, // blocked along K: s[k / block][n]
  kScaleAxis0 = 2,      // per-axis along K: s[k]
  kScaleAxis1Block = 3, // blocked along N: s[k][n / block]
  kScaleAxis1 = 4       // per-axis along N: s[n]
};

struct DqMmParams {
  const void *a;        // activations [M, K] (FLOAT / FLOAT16 / BFLOAT16)
  const uint8_t *w;     // packed quantized weight [K, N]
  const uint8_t *scale; // FLOAT or FLOAT16
  const uint8_t *zp;    // nullable, dtype of w
  void *y;              // [M, N], dtype of a
  int64_t M, K, N;
  int64_t block, s_alen;
  FastDiv fdiv_block;   // k / block (and n / block) in 32-bit arithmetic
  int wdt;
  int s_f16;    // scale (and DequantizeLinear output) is FLOAT16
  int cast_dt;  // 0 or the Cast target dtype
  int ydt;
  int slayout;
  int64_t kchunk;
  int ksplit;
  int gemv_nkb;       // scale rows staged per CTA (GEMV fast path)
  float *partials;    // split-K workspace
  uint32_t *counters; // split-K arrival counters (zero between calls)
  // Column-sharded output over a multi-GPU group (b2_dequantize_matmul_peer):
  // world > 1 sends every output value to each rank's full buffer.
  int world, rank;
  int64_t n_full, col_off;
  void *peer_full[8];
  uint32_t *peer_flags[8];
  uint32_t *pctr;
  int wait_input;
};

// Tensor-core path (dq_gemm_tc.cu).
bool dq_tc_eligible(const DqMmParams &p);  // shape/type constraints only
bool dq_tc_supported(const DqMmParams &p); // eligible and chosen by default
size_t dq_tc_workspace(const DqMmParams &p);
// wait_ns bounds every device-side wait; no_loads (self-test only) issues no
// TMA, so the first data wait runs out and the time-out path runs.
int dq_tc_launch(const DqMmParams &p, void *workspace, cudaStream_t stream,
                 uint64_t wait_ns = kWaitNs, bool no_loads = false);
int dq_tc_ksplit(const DqMmParams &p); // split-K factor of the plan
int status_read_dq_gemm_tc(int reset); // time-out word of dq_gemm_tc (-1: read failed)

// Decode path on register-level MMA (dq_gemv_mma.cu): M <= 16, INT4/UINT4
// weights, FLOAT16 scales, activations and output.
bool dq_mma_eligible(const DqMmParams &p); // shape/type constraints
bool dq_mma_aligned(const DqMmParams &p);  // pointer alignment TMA needs
size_t dq_mma_workspace(const DqMmParams &p);
int dq_mma_launch(const DqMmParams &p, void *workspace, cudaStream_t stream);
// Several projections of the same activations in one launch (1..4 of them,
// same M, K, weight type and scale layout, each eligible and aligned).
bool dq_mma_group_eligible(const DqMmParams *ps, int count);
size_t dq_mma_group_workspace(const DqMmParams *ps, int count);
int dq_mma_launch_group(const DqMmParams *ps, int count, void *workspace, cudaStream_t stream);

// Decode path with the reference's exact fp16 weights (dq_gemv_x.cu): M <= 64,
// INT4/UINT4 weights, FLOAT16 scales, activations and output.
bool dq_x_eligible(const DqMmParams &p); // shape/type constraints (pointer alignment: dq_mma_aligned)
size_t dq_x_workspace(const DqMmParams &p);
int dq_x_launch(const DqMmParams &p, void *workspace, cudaStream_t stream);

// Decode path on narrow column tiles without split-K (dq_gemv_n.cu): M <= 64,
// INT4/UINT4 weights, FLOAT16 scales, activations and output; no workspace.
bool dq_n_eligible(const DqMmParams &p); // shape/type constraints (pointer alignment: dq_mma_aligned)
int dq_n_launch(const DqMmParams &p, cudaStream_t stream);

// Decode path split along K inside thread-block clusters (dq_gemv_c.cu): M <=
// 32, INT4/UINT4 weights, FLOAT16 scales, activations and output; no workspace.
bool dq_c_eligible(const DqMmParams &p); // shape/type constraints (pointer alignment: dq_mma_aligned)
int dq_c_launch(const DqMmParams &p, cudaStream_t stream, bool exact);

// FLOAT-activation path on CUDA cores (dq_gemm_f32.cu): INT4 / UINT4 / INT8 /
// UINT8 weights, per-tensor, per-column or K-blocked scales, FLOAT output.
bool dq_f32_eligible(const DqMmParams &p); // shape/type constraints
bool dq_f32_aligned(const DqMmParams &p);  // pointer alignment of its vector loads
size_t dq_f32_workspace(const DqMmParams &p);
int dq_f32_launch(const DqMmParams &p, void *workspace, cudaStream_t stream);

} // namespace b2
