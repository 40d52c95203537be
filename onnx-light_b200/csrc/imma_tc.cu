// MatMulInteger / QLinearMatMul on tcgen05 kind::i8 tensor cores (sm_100a).
//
// y = sum_k (a - za)(b - zb) is computed as
//   S - zb * sum_k a' - za' * sum_k b + K * za' * zb,   S = sum_k a' b,
// with a' = a - 128 for UINT8 A (a byte XOR 0x80 read as int8) and a' = a for
// INT8 A, za' the matching shift of the zero point.  For the common
// symmetric UINT8 activation (za = 128) za' = 0 and the column sums of B are
// never needed.  S is accumulated by the tensor cores in int32 TMEM (exact:
// K < 65536 so |S| < 2^31), the zero-point terms and the QLinearMatMul
// requantisation run in the epilogue.
//
// Kernel structure (one CTA per 128 x 256 output tile, 192 threads):
//   warp 0     one elected thread issues TMA loads of A' [128 x 128 bytes] and
//              B [128 x 256 bytes] (two 128-byte-wide boxes) into a 4-stage
//              shared-memory ring, both with 128-byte swizzling;
//   warp 1     allocates 256 TMEM columns and one elected thread issues
//              tcgen05.mma.kind::i8 (M=128, N=256, K=32; A K-major, B MN-major,
//              straight from the row-major [K, N] B) and tcgen05.commit to
//              release each stage;
//   warps 2-5  read the accumulator tile from TMEM (tcgen05.ld 32x32b) and
//              write y.
// Every wait is bounded; a wait that gives up records the failure in the
// device word g_imma_tc_status (read by b2_kernel_status) and the CTA skips
// the rest of its work, after letting its own copies in flight land.
#include "imma.cuh"
#include "tc_common.cuh"

namespace b2 {

// Two CTAs per SM (2 x 96 KB of ring, 2 x 256 TMEM columns): one CTA's epilogue
// and prologue overlap the other's streaming, and config 2's 172 tiles fit in
// one wave of 296 slots instead of two of 148 (+29 % measured).
constexpr int IT_BM = 128, IT_BN = 256, IT_BK = 128, IT_STAGES = 2, IT_THREADS = 192;
constexpr uint32_t IT_A_BYTES = IT_BM * IT_BK;  // 16 KB
constexpr uint32_t IT_B_BYTES = IT_BK * IT_BN;  // 32 KB
constexpr uint32_t IT_STAGE_BYTES = IT_A_BYTES + IT_B_BYTES;
constexpr size_t IT_SMEM = (size_t)IT_STAGES * IT_STAGE_BYTES + 1024 + 256;

struct ImmaTcArgs {
  ImmaParams p;
  const int32_t *rowsum; // [M] sum_k a'
  const int32_t *colsum; // [N] sum_k b, written only when some za' != 0
  uint8_t *a_shift;      // workspace copy of a' (UINT8 A only)
};

// Time-out code of the last launch that gave up (0 = none); read and cleared
// by b2_kernel_status().
__device__ int g_imma_tc_status;

__device__ __forceinline__ int32_t zp_shifted(const ImmaParams &p, int64_t m) {
  const int32_t za = p.a_zp ? rd_byte(p.adt, p.a_zp, p.a_zp_n > 1 ? m : 0) : 0;
  return p.adt == kUint8 ? za - 128 : za;
}

// Row sums of A' (and the UINT8 -> int8 shifted copy of A), then column sums
// of B when some shifted A zero point is non-zero.
__global__ void __launch_bounds__(256) imma_prep(const ImmaTcArgs args, int a_blocks) {
  const ImmaParams &p = args.p;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if ((int)blockIdx.x < a_blocks) {
    const int64_t m = (int64_t)blockIdx.x * 8 + warp;
    if (m >= p.M) return;
    const uint32_t *src = reinterpret_cast<const uint32_t *>(p.a + m * p.K);
    uint32_t *dst = args.a_shift ? reinterpret_cast<uint32_t *>(args.a_shift + m * p.K) : nullptr;
    int sum = 0;
    for (int64_t i = lane; i < p.K / 4; i += 32) {
      uint32_t w = src[i];
      if (dst) {
        w ^= 0x80808080u;
        dst[i] = w;
      }
      int d;
      asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(w), "r"(0x01010101u), "r"(sum));
      sum = d;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) const_cast<int32_t *>(args.rowsum)[m] = sum;
    return;
  }
  // column sums, only when needed
  bool need = false;
  const int64_t nz = p.a_zp ? (p.a_zp_n > 1 ? p.M : 1) : 1;
  for (int64_t m = 0; m < nz && !need; ++m) need = zp_shifted(p, m) != 0;
  if (!need) return;
  const int64_t n4 = ((int64_t)(blockIdx.x - a_blocks) * 256 + threadIdx.x) * 4;
  if (n4 >= p.N) return;
  int s0 = 0, s1 = 0, s2 = 0, s3 = 0;
  const bool bs = p.bdt == kInt8;
  for (int64_t k = 0; k < p.K; ++k) {
    const uint32_t w = *reinterpret_cast<const uint32_t *>(p.b + k * p.N + n4);
    if (bs) {
      s0 += (int8_t)(w & 0xff); s1 += (int8_t)((w >> 8) & 0xff);
      s2 += (int8_t)((w >> 16) & 0xff); s3 += (int8_t)(w >> 24);
    } else {
      s0 += (int)(w & 0xff); s1 += (int)((w >> 8) & 0xff);
      s2 += (int)((w >> 16) & 0xff); s3 += (int)(w >> 24);
    }
  }
  int32_t *cs = const_cast<int32_t *>(args.colsum);
  cs[n4] = s0; cs[n4 + 1] = s1; cs[n4 + 2] = s2; cs[n4 + 3] = s3;
}

__device__ __forceinline__ void imma_tc_store(const ImmaTcArgs &args, int64_t m, int64_t n0,
                                              const uint32_t (&r)[32]) {
  const ImmaParams &p = args.p;
  const int32_t zas = zp_shifted(p, m);
  const int32_t rs = args.rowsum[m];
  if (p.mode == kImmaInteger) {
    int32_t out[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int64_t n = n0 + j;
      const int32_t zb = (p.b_zp && n < p.N) ? rd_byte(p.bdt, p.b_zp, p.b_zp_n > 1 ? n : 0) : 0;
      const int32_t cs = (zas != 0 && n < p.N) ? args.colsum[n] : 0;
      // int32 wraparound arithmetic, as the reference accumulator
      const uint32_t v = r[j] - (uint32_t)zb * (uint32_t)rs - (uint32_t)zas * (uint32_t)cs +
                         (uint32_t)p.K * (uint32_t)zas * (uint32_t)zb;
      out[j] = (int32_t)v;
    }
    int32_t *y = reinterpret_cast<int32_t *>(p.y) + m * p.N + n0;
    if (n0 + 32 <= p.N && (p.N % 4) == 0) {
#pragma unroll
      for (int j = 0; j < 32; j += 4)
        *reinterpret_cast<int4 *>(y + j) = make_int4(out[j], out[j + 1], out[j + 2], out[j + 3]);
    } else {
      for (int j = 0; j < 32; ++j)
        if (n0 + j < p.N) y[j] = out[j];
    }
    return;
  }
  // QLinearMatMul: exact int64 accumulator, then the reference's requantisation.
  uint8_t out[32];
  const float lo = p.ydt == kInt8 ? -128.0f : 0.0f, hi = p.ydt == kInt8 ? 127.0f : 255.0f;
  const float yz = (float)rd_byte(p.ydt, p.y_zp, 0);
  const int64_t zb = rd_byte(p.bdt, p.b_zp, 0);
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const int64_t n = n0 + j;
    const int64_t cs = (zas != 0 && n < p.N) ? args.colsum[n] : 0;
    const int64_t acc = (int64_t)(int32_t)r[j] - zb * rs - (int64_t)zas * cs + p.K * (int64_t)zas * zb;
    float v = __fmul_rn(__ll2float_rn(acc), p.comb_scale);
    v = __fadd_rn(rintf(v), yz);
    if (v < lo) v = lo;
    else if (v > hi) v = hi;
    const int32_t q = (v != v) ? 0 : (int32_t)v;
    out[j] = (uint8_t)(q & 0xff);
  }
  uint8_t *y = reinterpret_cast<uint8_t *>(p.y) + m * p.N + n0;
  if (n0 + 32 <= p.N && (p.N % 16) == 0) {
    const uint32_t *o = reinterpret_cast<const uint32_t *>(out);
    *reinterpret_cast<uint4 *>(y) = make_uint4(o[0], o[1], o[2], o[3]);
    *reinterpret_cast<uint4 *>(y + 16) = make_uint4(o[4], o[5], o[6], o[7]);
  } else {
    for (int j = 0; j < 32; ++j)
      if (n0 + j < p.N) y[j] = out[j];
  }
}

__global__ void __launch_bounds__(IT_THREADS, 2)
    imma_tc_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                   const ImmaTcArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + IT_STAGES * IT_STAGE_BYTES);
  uint64_t *empty = full + IT_STAGES;
  uint64_t *done = empty + IT_STAGES;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);
  __shared__ volatile int abort_flag;
  __shared__ int issued; // k stages the producer filled (for the drain after a give-up)
  const ImmaParams &p = args.p;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m_tile = blockIdx.x, n_tile = blockIdx.y;
  const int kt_count = (int)((p.K + IT_BK - 1) / IT_BK);

  if (threadIdx.x == 0) {
    abort_flag = 0;
    issued = 0;
    for (int s = 0; s < IT_STAGES; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    tc::mbar_init(done, 1);
    tc::fence_barrier_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, 256);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (tc::elect_one()) {
      tc::prefetch_tensormap(&map_a);
      tc::prefetch_tensormap(&map_b);
      for (int kt = 0; kt < kt_count; ++kt) {
        const int s = kt % IT_STAGES;
        if (kt >= IT_STAGES && !tc::mbar_wait(&empty[s], ((kt / IT_STAGES) - 1) & 1)) {
          atomicExch(&g_imma_tc_status, tc::kTimeoutEmpty);
          abort_flag = 1;
          break;
        }
        if (abort_flag) break;
        issued = kt + 1;
        uint8_t *st = smem + s * IT_STAGE_BYTES;
        tc::mbar_expect_tx(&full[s], IT_STAGE_BYTES);
        tc::tma_load_2d(st, &map_a, &full[s], kt * IT_BK, m_tile * IT_BM);
        tc::tma_load_2d(st + IT_A_BYTES, &map_b, &full[s], n_tile * IT_BN, kt * IT_BK);
        tc::tma_load_2d(st + IT_A_BYTES + IT_B_BYTES / 2, &map_b, &full[s], n_tile * IT_BN + 128,
                        kt * IT_BK);
      }
    }
  } else if (warp == 1) {
    if (tc::elect_one()) {
      constexpr uint32_t kIdescSS = tc::idesc(2, 1, 1, 0, 1, IT_BM, IT_BN);
      constexpr uint32_t kIdescSU = tc::idesc(2, 1, 0, 0, 1, IT_BM, IT_BN);
      const uint32_t id = p.bdt == kInt8 ? kIdescSS : kIdescSU;
      int kt = 0;
      for (; kt < kt_count; ++kt) {
        const int s = kt % IT_STAGES;
        if (!tc::mbar_wait(&full[s], (kt / IT_STAGES) & 1)) {
          atomicExch(&g_imma_tc_status, tc::kTimeoutFull);
          abort_flag = 1;
          break;
        }
        tc::tc_fence_after();
        const uint32_t a_base = tc::smem_u32(smem + s * IT_STAGE_BYTES);
        const uint32_t b_base = a_base + IT_A_BYTES;
#pragma unroll
        for (int kk = 0; kk < IT_BK / 32; ++kk) {
          const uint64_t ad = tc::sdesc_sw128(a_base + kk * 32, 16, 1024);
          const uint64_t bd = tc::sdesc_sw128(b_base + kk * 32 * 128, IT_B_BYTES / 2, 1024);
          tc::mma_i8(tmem, ad, bd, id, (kt > 0 || kk > 0) ? 1u : 0u);
        }
        tc::tc_commit(&empty[s]);
      }
      tc::tc_commit(done);
    }
  } else {
    // epilogue warps 2..5 -> TMEM lane groups 2, 3, 0, 1
    const int g = warp & 3;
    const bool ok = tc::mbar_wait(done, 0, 2 * kWaitNs);
    if (!ok) {
      atomicExch(&g_imma_tc_status, tc::kTimeoutMma);
      abort_flag = 1;
    }
    tc::tc_fence_after();
    const int64_t m = (int64_t)m_tile * IT_BM + g * 32 + lane;
    if (ok && !abort_flag) {
#pragma unroll 1
      for (int ch = 0; ch < IT_BN / 32; ++ch) {
        uint32_t r[32];
        tc::tmem_ld32(tmem + ((uint32_t)(g * 32) << 16) + (uint32_t)(ch * 32), r);
        tc::tmem_ld_wait();
        const int64_t n0 = (int64_t)n_tile * IT_BN + ch * 32;
        if (m < p.M && n0 < p.N) imma_tc_store(args, m, n0, r);
      }
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 1) tc::tmem_dealloc(tmem, 256);
  if (abort_flag && threadIdx.x == 0) {
    // A wait gave up: let this CTA's own copies in flight land before it
    // exits (the last fill of each stage; bounded again).
    const int n = issued;
    for (int kt = n > IT_STAGES ? n - IT_STAGES : 0; kt < n; ++kt)
      tc::mbar_wait(&full[kt % IT_STAGES], (kt / IT_STAGES) & 1, kWaitNs / 4);
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

bool imma_tc_supported(const ImmaParams &p) {
  return p.batch == 1 && p.M >= 64 && p.N >= 128 && p.K >= 128 && p.K < 65536 &&
         p.K % 16 == 0 && p.N % 16 == 0;
}

static size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

size_t imma_tc_workspace(const ImmaParams &p) {
  size_t bytes = kCounterBytes;
  if (p.adt == kUint8) bytes += align256((size_t)p.M * p.K);
  bytes += align256((size_t)p.M * 4) + align256((size_t)p.N * 4);
  return bytes;
}

int imma_tc_launch(const ImmaParams &p, void *workspace, cudaStream_t st) {
  ImmaTcArgs args{};
  args.p = p;
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  size_t off = kCounterBytes;
  if (p.adt == kUint8) {
    args.a_shift = ws + off;
    off += align256((size_t)p.M * p.K);
  }
  args.rowsum = reinterpret_cast<int32_t *>(ws + off);
  off += align256((size_t)p.M * 4);
  args.colsum = reinterpret_cast<int32_t *>(ws + off);
  // 1) row sums (+ shifted A copy) and, if needed, column sums
  const int a_blocks = (int)((p.M + 7) / 8);
  const int b_blocks = (int)((p.N / 4 + 255) / 256);
  if ((p.K % 4) != 0) B2_FAIL(B2_ERR_UNSUPPORTED, "imma_tc: K must be a multiple of 4");
  imma_prep<<<a_blocks + b_blocks, 256, 0, st>>>(args, a_blocks);
  B2_LAUNCH_CHECK();
  // 2) tensor maps: A' [M, K] int8 (K innermost), B [K, N] (N innermost)
  CUtensorMap map_a, map_b;
  const void *a_src = args.a_shift ? args.a_shift : p.a;
  {
    const uint64_t dims[2] = {(uint64_t)p.K, (uint64_t)p.M};
    const uint64_t strides[1] = {(uint64_t)p.K};
    const uint32_t box[2] = {IT_BK, IT_BM};
    int rc = make_tensor_map(&map_a, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, a_src, dims, strides, box,
                             CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  {
    const uint64_t dims[2] = {(uint64_t)p.N, (uint64_t)p.K};
    const uint64_t strides[1] = {(uint64_t)p.N};
    const uint32_t box[2] = {128, IT_BK};
    int rc = make_tensor_map(&map_b, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, p.b, dims, strides, box,
                             CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  B2_CUDA(cudaFuncSetAttribute(imma_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)IT_SMEM));
  dim3 grid((unsigned)((p.M + IT_BM - 1) / IT_BM), (unsigned)((p.N + IT_BN - 1) / IT_BN));
  imma_tc_kernel<<<grid, IT_THREADS, IT_SMEM, st>>>(map_a, map_b, args);
  B2_LAUNCH_CHECK();
  return B2_OK;
}

int status_read_imma_tc(int reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_imma_tc_status, sizeof(int)) != cudaSuccess) return -1;
  if (reset) {
    const int z = 0;
    if (cudaMemcpyToSymbol(g_imma_tc_status, &z, sizeof(int)) != cudaSuccess) return -1;
  }
  return v;
}

} // namespace b2
