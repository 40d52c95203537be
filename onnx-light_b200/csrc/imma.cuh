// Shared parameters and the exact integer / requantisation epilogue of
// MatMulInteger and QLinearMatMul.
#pragma once
#include "b2_common.cuh"

namespace b2 {

constexpr int kImmaMaxBatchRank = 8;
enum ImmaMode : int { kImmaInteger = 0, kImmaQLinear = 1 };

struct ImmaParams {
  const uint8_t *a, *b;        // [batch..][M, K], [batch..][K, N]
  const uint8_t *a_zp, *b_zp;  // nullable; scalar or per-row [M] / per-column [N]
  const uint8_t *y_zp;         // QLinearMatMul
  const void *scale_ptr[3];    // QLinearMatMul a/b/y scales (device)
  int scale_f16[3];
  float comb_scale;            // a_s * b_s / y_s in fp32, evaluated as the reference does
  void *y;
  int64_t M, K, N;
  int64_t a_zp_n, b_zp_n;
  int adt, bdt, ydt;
  int mode;
  int batch_rank;
  int64_t batch;
  int64_t out_prefix[kImmaMaxBatchRank];
  int64_t a_bstride[kImmaMaxBatchRank], b_bstride[kImmaMaxBatchRank];
};

__device__ __forceinline__ int32_t rd_byte(int dt, const uint8_t *p, int64_t i) {
  return dt == kInt8 ? (int32_t)(int8_t)p[i] : (int32_t)p[i];
}

// Writes y for one output element given sum_k a*b (exact, int64), sum_k a
// (row) and sum_k b (column).
__device__ __forceinline__ void imma_epilogue(const ImmaParams &p, int64_t bt, int64_t m, int64_t n,
                                              int64_t ab, int64_t rowsum, int64_t colsum) {
  const int64_t za = p.a_zp ? rd_byte(p.adt, p.a_zp, p.a_zp_n > 1 ? m : 0) : 0;
  const int64_t zb = p.b_zp ? rd_byte(p.bdt, p.b_zp, p.b_zp_n > 1 ? n : 0) : 0;
  const int64_t acc = ab - zb * rowsum - za * colsum + p.K * za * zb;
  const int64_t yi = (bt * p.M + m) * p.N + n;
  if (p.mode == kImmaInteger) {
    reinterpret_cast<int32_t *>(p.y)[yi] = (int32_t)(uint32_t)(uint64_t)acc; // int32 wraparound
    return;
  }
  // QLinearMatMul (kernel_qlinearmatmul.cc:115-127, 201-213)
  float v = __fmul_rn(__ll2float_rn(acc), p.comb_scale);
  v = __fadd_rn(rintf(v), (float)rd_byte(p.ydt, p.y_zp, 0));
  const float lo = p.ydt == kInt8 ? -128.0f : 0.0f, hi = p.ydt == kInt8 ? 127.0f : 255.0f;
  if (v < lo) v = lo;
  else if (v > hi) v = hi;
  const int32_t q = (v != v) ? 0 : (int32_t)v; // x86 cvttss2si of NaN -> 0x80000000, low byte 0
  reinterpret_cast<uint8_t *>(p.y)[yi] = (uint8_t)(q & 0xff);
}

// tcgen05 path (imma_tc.cu)
bool imma_tc_supported(const ImmaParams &p);
size_t imma_tc_workspace(const ImmaParams &p);
int imma_tc_launch(const ImmaParams &p, void *workspace, cudaStream_t stream);

} // namespace b2
