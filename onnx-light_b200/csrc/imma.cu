// MatMulInteger and QLinearMatMul on sm_100a, bit-exact with onnx-light's CPU
// kernels:
//   kernel::MatMulInteger (onnx_light/onnx_extensions/kernels/kernels/math/kernel_matmul_integer.cc:89-234)
//   kernel::QLinearMatMul (onnx_light/onnx_extensions/kernels/kernels/quantization/kernel_qlinearmatmul.cc:115-267)
//
// Zero points are applied in the epilogue:
//   sum_k (a - za)(b - zb) = sum ab - zb * sum_k a - za * sum_k b + K * za * zb
// which is exact in int32 wraparound arithmetic (MatMulInteger's int32
// accumulator) and, evaluated in int64, equals QLinearMatMul's int64
// accumulator.  Raw products are accumulated per 64-deep K tile in int32 (at
// most 64 * 255 * 255 < 2^31) and summed across tiles in int64, so any K is
// exact.  Row sums of A and column sums of B come from the same shared-memory
// tiles.
//
// mmi_tc (imma_tc.cu) runs the large 2-D shapes on tcgen05 kind::i8 tensor
// cores; this file holds the validation, the CUDA-core kernel used for every
// other shape (batched broadcasting, tiny or ragged matrices), and the
// requantisation epilogue shared by both.
#include "b2_common.cuh"
#include "imma.cuh"

namespace b2 {

constexpr int IM_BM = 64, IM_BN = 64, IM_BK = 64, IM_THREADS = 256;

template <bool AS, bool BS>
__device__ __forceinline__ int dp4a(uint32_t a, uint32_t b, int c) {
  int d;
  if (AS && BS) asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  else if (AS && !BS) asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  else if (!AS && BS) asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  else asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

__device__ __forceinline__ int64_t batch_offset(const ImmaParams &p, int64_t bt, const int64_t *st) {
  int64_t off = 0;
  for (int d = p.batch_rank - 1; d >= 0; --d) {
    const int64_t c = bt % p.out_prefix[d];
    bt /= p.out_prefix[d];
    off += c * st[d];
  }
  return off;
}

template <bool AS, bool BS>
__global__ void __launch_bounds__(IM_THREADS) imma_simt(const ImmaParams p) {
  // A tile stored k-contiguous per row, B tile transposed to k-contiguous per column,
  // so both dp4a operands are 4 consecutive k.
  __shared__ __align__(16) uint8_t As[IM_BM][IM_BK + 4];
  __shared__ __align__(16) uint8_t Bs[IM_BN][IM_BK + 4];
  __shared__ int64_t rowsum[IM_BM], colsum[IM_BN];
  const int tid = threadIdx.x;
  const int tx = tid % 16, ty = tid / 16; // 16 x 16 threads, 4 x 4 outputs each
  const int64_t m0 = (int64_t)blockIdx.y * IM_BM, n0 = (int64_t)blockIdx.x * IM_BN;
  const int64_t bt = blockIdx.z;
  const uint8_t *A = p.a + batch_offset(p, bt, p.a_bstride);
  const uint8_t *Bm = p.b + batch_offset(p, bt, p.b_bstride);
  if (tid < IM_BM) rowsum[tid] = 0;
  if (tid < IM_BN) colsum[tid] = 0;
  int64_t acc[4][4] = {};
  int rs_part = 0, cs_part = 0;
  for (int64_t k0 = 0; k0 < p.K; k0 += IM_BK) {
    __syncthreads();
    for (int e = tid; e < IM_BM * IM_BK; e += IM_THREADS) {
      const int mm = e / IM_BK, kk = e % IM_BK;
      const int64_t gm = m0 + mm, gk = k0 + kk;
      As[mm][kk] = (gm < p.M && gk < p.K) ? A[gm * p.K + gk] : 0;
    }
    for (int e = tid; e < IM_BN * IM_BK; e += IM_THREADS) {
      const int kk = e / IM_BN, nn = e % IM_BN;
      const int64_t gn = n0 + nn, gk = k0 + kk;
      Bs[nn][kk] = (gn < p.N && gk < p.K) ? Bm[gk * p.N + gn] : 0;
    }
    __syncthreads();
    int tacc[4][4] = {};
#pragma unroll 4
    for (int kk = 0; kk < IM_BK; kk += 4) {
      uint32_t av[4], bv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) av[i] = *reinterpret_cast<const uint32_t *>(&As[ty * 4 + i][kk]);
#pragma unroll
      for (int j = 0; j < 4; ++j) bv[j] = *reinterpret_cast<const uint32_t *>(&Bs[tx * 4 + j][kk]);
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) tacc[i][j] = dp4a<AS, BS>(av[i], bv[j], tacc[i][j]);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] += tacc[i][j];
    // row / column sums of this tile (threads 0..63 rows, 64..127 columns)
    if (tid < IM_BM) {
      int s = 0;
      for (int kk = 0; kk < IM_BK; kk += 4)
        s = dp4a<AS, false>(*reinterpret_cast<const uint32_t *>(&As[tid][kk]), 0x01010101u, s);
      rs_part = s;
      rowsum[tid] += rs_part;
    } else if (tid < IM_BM + IM_BN) {
      int s = 0;
      for (int kk = 0; kk < IM_BK; kk += 4)
        s = dp4a<BS, false>(*reinterpret_cast<const uint32_t *>(&Bs[tid - IM_BM][kk]), 0x01010101u, s);
      cs_part = s;
      colsum[tid - IM_BM] += cs_part;
    }
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t gm = m0 + ty * 4 + i, gn = n0 + tx * 4 + j;
      if (gm < p.M && gn < p.N)
        imma_epilogue(p, bt, gm, gn, acc[i][j], rowsum[ty * 4 + i], colsum[tx * 4 + j]);
    }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

static bool is_byte_int(int dt) { return dt == kInt8 || dt == kUint8; }

// MatMul shape rules (matmul_shape_utils.h:24-108).
static int plan_shapes(const b2_tensor *a, const b2_tensor *b, const char *name, ImmaParams &p,
                       std::vector<int64_t> &out_shape) {
  B2_ENFORCE(a->ndim >= 1 && b->ndim >= 1, "%s: rank-0 inputs are not accepted.", name);
  std::vector<int64_t> a2 = shape_of(a), b2 = shape_of(b);
  if (a2.size() == 1) a2.insert(a2.begin(), 1);
  if (b2.size() == 1) b2.push_back(1);
  B2_ENFORCE(a2.back() == b2[b2.size() - 2], "%s: incompatible inner dimensions.", name);
  const int ap = (int)a2.size() - 2, bp = (int)b2.size() - 2;
  const int r = ap > bp ? ap : bp;
  B2_ENFORCE(r <= kImmaMaxBatchRank, "%s: too many batch dimensions", name);
  std::vector<int64_t> outp(r);
  for (int i = 0; i < r; ++i) {
    const int64_t da = i + ap >= r ? a2[i - (r - ap)] : 1;
    const int64_t db = i + bp >= r ? b2[i - (r - bp)] : 1;
    if (da == db || da == 1) outp[i] = db;
    else if (db == 1) outp[i] = da;
    else B2_FAIL(B2_ERR_INVALID_ARGUMENT, "%s: inputs are not broadcast-compatible on batch dimensions.", name);
  }
  out_shape = outp;
  if (a->ndim != 1) out_shape.push_back(a2[a2.size() - 2]);
  if (b->ndim != 1) out_shape.push_back(b2.back());
  p.M = a2[a2.size() - 2];
  p.K = a2.back();
  p.N = b2.back();
  p.batch_rank = r;
  p.batch = 1;
  // element strides of each operand's batch dims (0 where broadcast)
  int64_t ast = p.M * p.K, bst = p.K * p.N;
  std::vector<int64_t> as(r, 0), bs(r, 0);
  for (int d = r - 1; d >= 0; --d) {
    if (d + ap >= r) {
      const int ad = d - (r - ap);
      as[d] = a2[ad] == 1 ? 0 : ast;
      ast *= a2[ad];
    }
    if (d + bp >= r) {
      const int bd = d - (r - bp);
      bs[d] = b2[bd] == 1 ? 0 : bst;
      bst *= b2[bd];
    }
  }
  for (int d = 0; d < r; ++d) {
    p.out_prefix[d] = outp[d];
    p.a_bstride[d] = as[d];
    p.b_bstride[d] = bs[d];
    p.batch *= outp[d];
  }
  return B2_OK;
}

static int launch(const ImmaParams &p, void *ws, cudaStream_t st) {
  if (p.M == 0 || p.N == 0 || p.batch == 0) return B2_OK;
  if (imma_tc_supported(p)) return imma_tc_launch(p, ws, st);
  dim3 grid((unsigned)((p.N + IM_BN - 1) / IM_BN), (unsigned)((p.M + IM_BM - 1) / IM_BM),
            (unsigned)p.batch);
  const bool as = p.adt == kInt8, bs = p.bdt == kInt8;
  if (as && bs) imma_simt<true, true><<<grid, IM_THREADS, 0, st>>>(p);
  else if (as) imma_simt<true, false><<<grid, IM_THREADS, 0, st>>>(p);
  else if (bs) imma_simt<false, true><<<grid, IM_THREADS, 0, st>>>(p);
  else imma_simt<false, false><<<grid, IM_THREADS, 0, st>>>(p);
  B2_LAUNCH_CHECK();
  return B2_OK;
}

// Zero-point tensor rules of MatMulInteger (kernel_matmul_integer.cc:40-70).
static int zp_count(const b2_tensor *t, int dt, int64_t expected, const char *name, int64_t &count) {
  if (t == nullptr) { count = 0; return B2_OK; }
  B2_ENFORCE(t->dtype == dt, "kernel::MatMulInteger: '%s' dtype must match its data input.", name);
  B2_ENFORCE(t->ndim <= 1, "kernel::MatMulInteger: '%s' must be a scalar or a 1-D tensor.", name);
  const int64_t n = numel(t);
  B2_ENFORCE(n == 1 || n == expected,
             "kernel::MatMulInteger: '%s' must be a scalar, a one-element 1-D tensor, or a 1-D tensor "
             "whose size matches the corresponding matrix dimension.", name);
  count = n;
  return B2_OK;
}

} // namespace b2

using namespace b2;

extern "C" int b2_matmul_integer(const b2_tensor *a, const b2_tensor *b, const b2_tensor *a_zp,
                                 const b2_tensor *b_zp, b2_tensor *y, void *workspace,
                                 size_t *workspace_bytes, void *stream) {
  if (!a || !b || !y) B2_FAIL(B2_ERR_INVALID_ARGUMENT, "kernel::MatMulInteger: null tensor");
  B2_ENFORCE(is_byte_int(a->dtype), "kernel::MatMulInteger: A must be INT8 or UINT8.");
  B2_ENFORCE(is_byte_int(b->dtype), "kernel::MatMulInteger: B must be INT8 or UINT8.");
  B2_ENFORCE(y->dtype == kInt32, "kernel::MatMulInteger: output dtype must be INT32.");
  ImmaParams p{};
  std::vector<int64_t> out;
  int rc = plan_shapes(a, b, "kernel::MatMulInteger", p, out);
  if (rc) return rc;
  B2_ENFORCE(shape_of(y) == out, "kernel::MatMulInteger: preallocated output has invalid shape.");
  int64_t na = 0, nb = 0;
  if ((rc = zp_count(a_zp, a->dtype, p.M, "a_zero_point", na))) return rc;
  if ((rc = zp_count(b_zp, b->dtype, p.N, "b_zero_point", nb))) return rc;
  p.mode = kImmaInteger;
  p.adt = a->dtype;
  p.bdt = b->dtype;
  p.a = static_cast<const uint8_t *>(a->data);
  p.b = static_cast<const uint8_t *>(b->data);
  p.a_zp = na ? static_cast<const uint8_t *>(a_zp->data) : nullptr;
  p.b_zp = nb ? static_cast<const uint8_t *>(b_zp->data) : nullptr;
  p.a_zp_n = na;
  p.b_zp_n = nb;
  p.y = y->data;
  const size_t need = imma_tc_supported(p) ? imma_tc_workspace(p) : 0;
  rc = workspace_check(workspace, workspace_bytes, need);
  if (rc < 0) return rc;
  if (rc == 1) return B2_OK;
  return launch(p, workspace, static_cast<cudaStream_t>(stream));
}

extern "C" int b2_qlinear_matmul(const b2_tensor *a, const b2_tensor *a_scale,
                                 const b2_tensor *a_zp, const b2_tensor *b,
                                 const b2_tensor *b_scale, const b2_tensor *b_zp,
                                 const b2_tensor *y_scale, const b2_tensor *y_zp, b2_tensor *y,
                                 void *workspace, size_t *workspace_bytes, void *stream) {
  if (!a || !a_scale || !a_zp || !b || !b_scale || !b_zp || !y_scale || !y_zp || !y)
    B2_FAIL(B2_ERR_INVALID_ARGUMENT, "kernel::QLinearMatMul: null tensor");
  B2_ENFORCE(is_byte_int(a->dtype), "kernel::QLinearMatMul: a must be INT8 or UINT8.");
  B2_ENFORCE(is_byte_int(b->dtype), "kernel::QLinearMatMul: b must be INT8 or UINT8.");
  B2_ENFORCE(is_byte_int(y_zp->dtype), "kernel::QLinearMatMul: y_zero_point must be INT8 or UINT8.");
  B2_ENFORCE(a_zp->dtype == a->dtype, "kernel::QLinearMatMul: a_zero_point dtype must match a.");
  B2_ENFORCE(b_zp->dtype == b->dtype, "kernel::QLinearMatMul: b_zero_point dtype must match b.");
  B2_ENFORCE(y->dtype == y_zp->dtype, "kernel::QLinearMatMul: output dtype must match y_zero_point.");
  ImmaParams p{};
  std::vector<int64_t> out;
  int rc = plan_shapes(a, b, "kernel::QLinearMatMul", p, out);
  if (rc) return rc;
  B2_ENFORCE(shape_of(y) == out, "kernel::QLinearMatMul: preallocated output has invalid shape.");
  B2_ENFORCE(numel(a_zp) == 1, "kernel::QLinearMatMul: 'a_zero_point' must be a scalar.");
  B2_ENFORCE(numel(b_zp) == 1, "kernel::QLinearMatMul: 'b_zero_point' must be a scalar.");
  B2_ENFORCE(numel(y_zp) == 1, "kernel::QLinearMatMul: 'y_zero_point' must be a scalar.");
  const b2_tensor *sc[3] = {a_scale, b_scale, y_scale};
  const char *sn[3] = {"a_scale", "b_scale", "y_scale"};
  for (int i = 0; i < 3; ++i) {
    B2_ENFORCE(numel(sc[i]) == 1, "kernel::QLinearMatMul: '%s' must be a scalar.", sn[i]);
    B2_ENFORCE(sc[i]->dtype == kFloat || sc[i]->dtype == kFloat16,
               "kernel::QLinearMatMul: '%s' must be a FLOAT or FLOAT16 scalar for the reference kernel.",
               sn[i]);
  }
  p.mode = kImmaQLinear;
  p.adt = a->dtype;
  p.bdt = b->dtype;
  p.ydt = y->dtype;
  p.a = static_cast<const uint8_t *>(a->data);
  p.b = static_cast<const uint8_t *>(b->data);
  p.a_zp = static_cast<const uint8_t *>(a_zp->data);
  p.b_zp = static_cast<const uint8_t *>(b_zp->data);
  p.y_zp = static_cast<const uint8_t *>(y_zp->data);
  p.a_zp_n = 1;
  p.b_zp_n = 1;
  for (int i = 0; i < 3; ++i) {
    p.scale_ptr[i] = sc[i]->data;
    p.scale_f16[i] = sc[i]->dtype == kFloat16;
  }
  p.y = y->data;
  const size_t need = imma_tc_supported(p) ? imma_tc_workspace(p) : 0;
  rc = workspace_check(workspace, workspace_bytes, need);
  if (rc < 0) return rc;
  if (rc == 1) return B2_OK;
  // The three scalar scales are read back to the host: the reference rejects
  // y_scale == 0 (kernel_qlinearmatmul.cc:264) and evaluates the combined
  // scale a_s * b_s / y_s once in fp32 (:156); doing both here keeps the error
  // and the rounding identical.  This synchronizes with `stream`.
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  float sv[3];
  for (int i = 0; i < 3; ++i) {
    if (p.scale_f16[i]) {
      uint16_t h = 0;
      B2_CUDA(cudaMemcpyAsync(&h, p.scale_ptr[i], 2, cudaMemcpyDeviceToHost, st));
      B2_CUDA(cudaStreamSynchronize(st));
      sv[i] = __half2float(__ushort_as_half(h));
    } else {
      B2_CUDA(cudaMemcpyAsync(&sv[i], p.scale_ptr[i], 4, cudaMemcpyDeviceToHost, st));
      B2_CUDA(cudaStreamSynchronize(st));
    }
  }
  B2_ENFORCE(sv[2] != 0.0f, "kernel::QLinearMatMul: y_scale must be non-zero.");
  volatile float ab = sv[0] * sv[1];
  p.comb_scale = ab / sv[2];
  return launch(p, workspace, st);
}
