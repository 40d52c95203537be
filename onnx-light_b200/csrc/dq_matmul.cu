// Fused DequantizeLinear -> [Cast] -> MatMul (weight-only quantization).
//
// Replaces the node pair kernel::DequantizeLinear
// (onnx_light/onnx_extensions/kernels/kernels/quantization/kernel_dequantizelinear.cc:522-693)
// feeding kernel::MatMul (onnx_light/onnx_extensions/kernels/kernels/math/kernel_matmul.cc:181-223).
// The dequantized weight never exists in HBM: packed weights are read once,
// dequantized in registers with the reference's rounding (fp32 (q-zp)*s, then
// RNE to the DequantizeLinear output type and to the Cast type), and
// multiplied with fp32 accumulation.
//
// Kernels
//  * dq_gemv  — decode shapes (M <= 4 activation rows).  HBM-bound: each warp
//    streams 128-byte row segments of the packed weight with 16-byte loads
//    (8 lanes per row, 4 rows per load instruction), scales for the CTA's
//    K-range are staged in shared memory by the bulk-copy (TMA) engine, lanes
//    reduce across rows with warp shuffles, warps through shared memory and
//    CTAs (split-K) through a deterministic last-CTA reduction of partials.
//  * dq_gemm_simt — any shape / layout / dtype; tiled CUDA-core GEMM with the
//    dequantization fused into the B-tile load.  Used for FLOAT activations
//    (fp32 accumulation parity, 1e-5) and for layouts the fast paths skip.
//  * dq_gemm_tc (dq_gemm_tc.cu) — FLOAT16/BFLOAT16 activations with M > 8 on
//    tcgen05 tensor cores.
#include "b2_common.cuh"
#include "dq_matmul.cuh"
#include "tc_common.cuh"

#include <cstdlib>
#include <cstring>

namespace b2 {

// ---------------------------------------------------------------------------
// Dequantized weight element with the reference's rounding chain.
// ---------------------------------------------------------------------------

__device__ __forceinline__ float round_to(float v, int dt) {
  if (dt == kFloat16) return __half2float(__ushort_as_half(f32_to_f16_bits(v)));
  if (dt == kBfloat16) return __uint_as_float((uint32_t)f32_to_bf16_bits(v) << 16);
  return v;
}

__device__ __forceinline__ int64_t w_scale_index(const DqMmParams &p, int64_t k, int64_t n) {
  switch (p.slayout) {
  case kScaleTensor: return 0;
  case kScaleAxis0Block: return (int64_t)p.fdiv_block.div((uint32_t)k) * p.N + n;
  case kScaleAxis0: return k;
  case kScaleAxis1Block: return k * p.s_alen + p.fdiv_block.div((uint32_t)n);
  default: return n; // kScaleAxis1
  }
}

__device__ __forceinline__ float w_element(const DqMmParams &p, int64_t k, int64_t n) {
  const int64_t i = k * p.N + n;
  const float q = qval(p.wdt, p.w, i);
  const int64_t si = w_scale_index(p, k, n);
  const float s = p.s_f16 ? f16_bits_to_f32(reinterpret_cast<const uint16_t *>(p.scale)[si])
                          : reinterpret_cast<const float *>(p.scale)[si];
  const float z = p.zp ? qval(p.wdt, p.zp, si) : 0.0f;
  float v = x86_mul(x86_sub(q, z), s);
  v = round_to(v, p.s_f16 ? kFloat16 : kFloat); // DequantizeLinear output type
  if (p.cast_dt) v = round_to(v, p.cast_dt);    // optional Cast node
  return v;
}

template <typename T> __device__ __forceinline__ float act_load(const void *a, int64_t i);
template <> __device__ __forceinline__ float act_load<float>(const void *a, int64_t i) {
  return reinterpret_cast<const float *>(a)[i];
}
template <> __device__ __forceinline__ float act_load<__half>(const void *a, int64_t i) {
  return __half2float(reinterpret_cast<const __half *>(a)[i]);
}
template <> __device__ __forceinline__ float act_load<__nv_bfloat16>(const void *a, int64_t i) {
  return __uint_as_float((uint32_t)reinterpret_cast<const uint16_t *>(a)[i] << 16);
}

__device__ __forceinline__ void store_out(void *y, int dt, int64_t i, float v) {
  if (dt == kFloat) reinterpret_cast<float *>(y)[i] = v;
  else if (dt == kFloat16) reinterpret_cast<uint16_t *>(y)[i] = f32_to_f16_bits(v);
  else reinterpret_cast<uint16_t *>(y)[i] = f32_to_bf16_bits(v);
}

// ---------------------------------------------------------------------------
// Split-K finalisation shared by the CUDA-core kernels.
//
// Workspace layout: [ksplit][M][N] fp32 partials, then one uint32 arrival
// counter per output tile.  Each CTA writes its partial tile, then bumps the
// tile's counter; the CTA that arrives last sums the partials in split order
// (deterministic), writes y and resets the counter to 0, so the counters are
// zero again for the next call.
// ---------------------------------------------------------------------------

// Time-out code of the last CUDA-core GEMV launch that gave up (0 = none);
// read and cleared by b2_kernel_status().
__device__ int g_dq_gemv_status;

int status_read_dq_gemv(int reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_dq_gemv_status, sizeof(int)) != cudaSuccess) return -1;
  if (reset) {
    const int z = 0;
    if (cudaMemcpyToSymbol(g_dq_gemv_status, &z, sizeof(int)) != cudaSuccess) return -1;
  }
  return v;
}

__device__ __forceinline__ bool arrive_last(uint32_t *counter, int expected) {
  __shared__ bool last;
  __syncthreads(); // all partial stores of this CTA issued
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t prev = atomicAdd(counter, 1u);
    last = (prev + 1 == (uint32_t)expected);
    if (last) {
      __threadfence();
      *counter = 0u;
    }
  }
  __syncthreads();
  return last;
}

// ---------------------------------------------------------------------------
// dq_gemm_simt: C[M,N] = A[M,K] * Wdeq[K,N]
// ---------------------------------------------------------------------------

constexpr int SIMT_BM = 32, SIMT_BN = 128, SIMT_BK = 32;

template <typename T>
__global__ void __launch_bounds__(256) dq_gemm_simt(const DqMmParams p) {
  __shared__ float As[SIMT_BK][SIMT_BM + 1];
  __shared__ float Bs[SIMT_BK][SIMT_BN];
  const int tid = threadIdx.x;
  const int tn = tid % 32, tm = tid / 32;
  const int64_t n0 = (int64_t)blockIdx.x * SIMT_BN;
  const int64_t m0 = (int64_t)blockIdx.y * SIMT_BM;
  const int split = blockIdx.z;
  const int64_t kbeg = (int64_t)split * p.kchunk;
  const int64_t kend = min((int64_t)p.K, kbeg + p.kchunk);
  float acc[4][4] = {};
  for (int64_t k0 = kbeg; k0 < kend; k0 += SIMT_BK) {
    // A tile: 32 x 32, 4 per thread
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int e = tid + r * 256;
      const int mm = e / SIMT_BK, kk = e % SIMT_BK;
      const int64_t gm = m0 + mm, gk = k0 + kk;
      As[kk][mm] = (gm < p.M && gk < kend) ? act_load<T>(p.a, gm * p.K + gk) : 0.0f;
    }
    // B tile: 32 x 128, dequantized, 16 per thread
#pragma unroll 4
    for (int r = 0; r < 16; ++r) {
      const int e = tid + r * 256;
      const int kk = e / SIMT_BN, nn = e % SIMT_BN;
      const int64_t gk = k0 + kk, gn = n0 + nn;
      Bs[kk][nn] = (gk < kend && gn < p.N) ? w_element(p, gk, gn) : 0.0f;
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < SIMT_BK; ++kk) {
      float av[4], bv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) av[i] = As[kk][tm * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) bv[j] = Bs[kk][tn + 32 * j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();
  }
  if (p.ksplit == 1) {
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int64_t gm = m0 + tm * 4 + i, gn = n0 + tn + 32 * j;
        if (gm < p.M && gn < p.N) store_out(p.y, p.ydt, gm * p.N + gn, acc[i][j]);
      }
    return;
  }
  float *part = p.partials + (int64_t)split * p.M * p.N;
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t gm = m0 + tm * 4 + i, gn = n0 + tn + 32 * j;
      if (gm < p.M && gn < p.N) part[gm * p.N + gn] = acc[i][j];
    }
  const int tile = blockIdx.y * gridDim.x + blockIdx.x;
  if (!arrive_last(p.counters + tile, p.ksplit)) return;
  for (int e = tid; e < SIMT_BM * SIMT_BN; e += 256) {
    const int64_t gm = m0 + e / SIMT_BN, gn = n0 + e % SIMT_BN;
    if (gm >= p.M || gn >= p.N) continue;
    float s = 0.0f;
    for (int sp = 0; sp < p.ksplit; ++sp) s += __ldcg(p.partials + ((int64_t)sp * p.M + gm) * p.N + gn);
    store_out(p.y, p.ydt, gm * p.N + gn, s);
  }
}

// ---------------------------------------------------------------------------
// dq_gemv: decode-shaped fused kernel (M <= 8).
// ---------------------------------------------------------------------------

// Decodes the 32 (int4/fp4: 16 bytes) or 32 (8-bit: 32 bytes) consecutive
// quantized values a lane owns in one weight row.
template <int BITS>
__device__ __forceinline__ void gemv_load(const uint8_t *row, uint4 (&raw)[BITS / 4]) {
  const uint4 *src = reinterpret_cast<const uint4 *>(row);
#pragma unroll
  for (int i = 0; i < BITS / 4; ++i) raw[i] = __ldcs(src + i);
}

template <int BITS>
__device__ __forceinline__ float gemv_q(int wdt, const uint4 (&raw)[BITS / 4], int j) {
  if (BITS == 4) {
    const uint32_t word = j < 8 ? raw[0].x : j < 16 ? raw[0].y : j < 24 ? raw[0].z : raw[0].w;
    const uint32_t nib = (word >> (4 * (j & 7))) & 0xfu;
    if (wdt == kInt4) return (float)((int)nib - ((nib & 8u) ? 16 : 0));
    if (wdt == kUint4) return (float)nib;
    return dec_f4e2m1(nib);
  } else {
    const uint4 &r = raw[j >> 4];
    const int jj = j & 15;
    const uint32_t word = jj < 4 ? r.x : jj < 8 ? r.y : jj < 12 ? r.z : r.w;
    const uint32_t b = (word >> (8 * (jj & 3))) & 0xffu;
    switch (wdt) {
    case kUint8: return (float)b;
    case kInt8: return (float)(int8_t)b;
    case kF8E4M3FN: return dec_f8e4m3fn(b);
    case kF8E4M3FNUZ: return dec_f8e4m3fnuz(b);
    case kF8E5M2: return dec_f8e5m2(b);
    default: return dec_f8e5m2fnuz(b);
    }
  }
}

constexpr int GEMV_THREADS = 256;
constexpr int GEMV_TN = 256; // columns per CTA (8 lanes x 32)

// Fast dequantisation of 8 signed/unsigned int4 values (one 32-bit word) into
// fp16 pairs, multiplied by fp16 scales: the fp16 product of a 4-bit integer
// and an fp16 scale is the correctly rounded fp16 of the exact product, i.e.
// FloatToFloat16Bits((q - 0) * s) of the reference.
__device__ __forceinline__ void int4x8_times_scale_f16(uint32_t w, bool is_signed,
                                                       const __half2 (&s2)[4], __half2 (&out)[4]) {
  // Element j of the word is nibble j.  Pairs are formed as (j, j+4): bits
  // [4j, 4j+4) go to the low half, bits [4j+16, 4j+20) to the high half.
  const uint32_t x = is_signed ? (w ^ 0x88888888u) : w;
  const __half2 bias = __halves2half2(__ushort_as_half(is_signed ? 0x6408 : 0x6400),
                                      __ushort_as_half(is_signed ? 0x6408 : 0x6400));
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t h = ((x >> (4 * j)) & 0x000f000fu) | 0x64006400u; // 1024 + code
    const __half2 q = __hsub2(*reinterpret_cast<const __half2 *>(&h), bias);
    __half2 r;
    asm("mul.rn.f16x2 %0, %1, %2;"
        : "=r"(*reinterpret_cast<uint32_t *>(&r))
        : "r"(*reinterpret_cast<const uint32_t *>(&q)), "r"(*reinterpret_cast<const uint32_t *>(&s2[j])));
    out[j] = r;
  }
}

__device__ __forceinline__ float act_load_rt(const DqMmParams &p, int64_t i) {
  if (p.ydt == kFloat) return act_load<float>(p.a, i);
  if (p.ydt == kFloat16) return act_load<__half>(p.a, i);
  return act_load<__nv_bfloat16>(p.a, i);
}

// Reduction epilogue shared by the GEMV kernels: acc[m][j] holds this lane's
// partial sums for columns ncol..ncol+31 of row group r.  Lanes r = 0..3 are
// summed with shuffles, warps through shared memory, CTAs (split-K) through
// the workspace partials and the last-arriving CTA.
template <int MT>
__device__ __forceinline__ void gemv_reduce(const DqMmParams &p, float (&acc)[MT][32], float *red,
                                            int64_t n0, int split) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c = lane & 7, r = lane >> 3;
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      acc[m][j] += __shfl_xor_sync(0xffffffffu, acc[m][j], 8);
      acc[m][j] += __shfl_xor_sync(0xffffffffu, acc[m][j], 16);
    }
  __syncthreads(); // red may alias staging buffers
  if (r == 0) {
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
      for (int j = 0; j < 32; ++j) red[(warp * MT + m) * GEMV_TN + c * 32 + j] = acc[m][j];
  }
  __syncthreads();
  float *part = p.ksplit > 1 ? p.partials + (int64_t)split * p.M * p.N : nullptr;
  for (int e = threadIdx.x; e < MT * GEMV_TN; e += GEMV_THREADS) {
    const int m = e / GEMV_TN, nn = e % GEMV_TN;
    float s = 0.0f;
#pragma unroll
    for (int w = 0; w < GEMV_THREADS / 32; ++w) s += red[(w * MT + m) * GEMV_TN + nn];
    const int64_t gn = n0 + nn;
    if (m < p.M && gn < p.N) {
      if (part) part[(int64_t)m * p.N + gn] = s;
      else store_out(p.y, p.ydt, (int64_t)m * p.N + gn, s);
    }
  }
  if (!part) return;
  if (!arrive_last(p.counters + blockIdx.x, p.ksplit)) return;
  for (int e = threadIdx.x; e < MT * GEMV_TN; e += GEMV_THREADS) {
    const int m = e / GEMV_TN;
    const int64_t gn = n0 + e % GEMV_TN;
    if (m >= p.M || gn >= p.N) continue;
    float s = 0.0f;
    for (int sp = 0; sp < p.ksplit; ++sp)
      s += __ldcg(p.partials + ((int64_t)sp * p.M + m) * p.N + gn);
    store_out(p.y, p.ydt, (int64_t)m * p.N + gn, s);
  }
}

// fp32 += fp16 * fp16 with one rounding (mixed-precision FMA, sm_100).
__device__ __forceinline__ float fma_f16(uint16_t a, uint16_t b, float c) {
  asm("fma.rn.f32.f16 %0, %1, %2, %0;" : "+f"(c) : "h"(a), "h"(b));
  return c;
}

// Generic decode GEMV: any 4-/8-bit weight type, zero points, FLOAT/FLOAT16
// scales, any activation type; "column" scale layouts only.
template <int MT, int BITS>
__global__ void __launch_bounds__(GEMV_THREADS) dq_gemv(const DqMmParams p) {
  extern __shared__ float smem[];
  float *a_s = smem;                  // [MT][kchunk] fp32 activations
  float *red = smem + MT * p.kchunk;  // [8][MT][256] reduction
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c = lane & 7, r = lane >> 3;
  const int64_t n0 = (int64_t)blockIdx.x * GEMV_TN;
  const int64_t ncol = n0 + c * 32;
  const int split = blockIdx.y;
  const int64_t kbeg = (int64_t)split * p.kchunk;
  const int64_t kend = min((int64_t)p.K, kbeg + p.kchunk);
  const int64_t klen = kend - kbeg;
  for (int e = threadIdx.x; e < MT * p.kchunk; e += GEMV_THREADS) {
    const int mm = e / p.kchunk;
    const int64_t kk = e % p.kchunk;
    a_s[e] = (mm < p.M && kk < klen) ? act_load_rt(p, (int64_t)mm * p.K + kbeg + kk) : 0.0f;
  }
  __syncthreads();
  float acc[MT][32];
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int j = 0; j < 32; ++j) acc[m][j] = 0.0f;
  const bool col_ok = ncol + 32 <= p.N;
  float sc[32], zc[32];
  int64_t cur_kb = -1;
  const int64_t row_bytes = p.N * BITS / 8;
  const uint8_t *wcol = p.w + ncol * BITS / 8;
  constexpr int U = 4;
  for (int64_t kk0 = warp * 4 + r; col_ok && kk0 < klen; kk0 += 32 * U) {
    uint4 raw[U][BITS / 4];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t kk = kk0 + 32 * u;
      if (kk < klen) gemv_load<BITS>(wcol + (kbeg + kk) * row_bytes, raw[u]);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t kk = kk0 + 32 * u;
      if (kk >= klen) break;
      const int64_t k = kbeg + kk;
      const int64_t kb = p.slayout == kScaleAxis0Block ? (int64_t)p.fdiv_block.div((uint32_t)k) : 0;
      if (kb != cur_kb) {
        cur_kb = kb;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int64_t si = p.slayout == kScaleTensor ? 0
                             : p.slayout == kScaleAxis0Block ? kb * p.N + ncol + j
                                                             : ncol + j;
          sc[j] = p.s_f16 ? f16_bits_to_f32(reinterpret_cast<const uint16_t *>(p.scale)[si])
                          : reinterpret_cast<const float *>(p.scale)[si];
          zc[j] = p.zp ? qval(p.wdt, p.zp, si) : 0.0f;
        }
      }
      float wv[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        float v = x86_mul(x86_sub(gemv_q<BITS>(p.wdt, raw[u], j), zc[j]), sc[j]);
        v = round_to(v, p.s_f16 ? kFloat16 : kFloat);
        if (p.cast_dt) v = round_to(v, p.cast_dt);
        wv[j] = v;
      }
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        const float av = a_s[m * p.kchunk + kk];
#pragma unroll
        for (int j = 0; j < 32; ++j) acc[m][j] = fmaf(av, wv[j], acc[m][j]);
      }
    }
  }
  gemv_reduce<MT>(p, acc, red, n0, split);
}

// Decode GEMV fast path: INT4/UINT4 weights, FLOAT16 scales (blocked along K
// with block % 32 == 0, per-tensor, or per-column), no zero point, FLOAT16
// activations and output.
//
// The packed weight rows of the CTA's [kchunk x 256] tile stream through an
// 8-stage shared-memory ring (32 rows x 128 bytes per stage) filled by TMA
// from a dedicated producer warp, so 32 KB per CTA stay in flight whatever
// the consumers are doing.  The CTA's scale rows are staged once with bulk
// copies.  Each consumer lane takes one weight row segment of 32 nibbles per
// stage: magic-number nibble -> fp16 conversion, fp16 product with the scale
// (the correctly rounded fp16 of the exact product, i.e. the reference's
// FloatToFloat16Bits((q - 0) * s)), and fp32 accumulation with the
// mixed-precision FMA.
constexpr int GV_STAGES = 8, GV_ROWS = 32, GV_CONSUMERS = 256, GV_THREADS = 288;
constexpr uint32_t GV_STAGE_BYTES = GV_ROWS * 128;

template <int MT>
__global__ void __launch_bounds__(GV_THREADS, MT == 1 ? 2 : 1)
    dq_gemv_i4h(const __grid_constant__ CUtensorMap map_w, const DqMmParams p) {
  extern __shared__ __align__(1024) uint8_t gsm[];
  uint8_t *ring = gsm;                                                 // [S][32][128]
  __half *s_s = reinterpret_cast<__half *>(gsm + GV_STAGES * GV_STAGE_BYTES); // [nkb][256]
  __half *a_s = s_s + (size_t)p.gemv_nkb * GEMV_TN;                    // [MT][kchunk]
  uint64_t *full = reinterpret_cast<uint64_t *>(
      (reinterpret_cast<uintptr_t>(a_s + (size_t)MT * p.kchunk) + 15) & ~uintptr_t(15));
  uint64_t *empty = full + GV_STAGES;
  uint64_t *sbar = empty + GV_STAGES;
  float *red = reinterpret_cast<float *>(gsm);                         // reuses the ring
  __shared__ volatile int abort_flag;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c = lane & 7, r = lane >> 3;
  const int64_t n0 = (int64_t)blockIdx.x * GEMV_TN;
  const int split = blockIdx.y;
  const int64_t kbeg = (int64_t)split * p.kchunk;
  const int64_t kend = min((int64_t)p.K, kbeg + p.kchunk);
  const int64_t klen = kend - kbeg;
  const int ntiles = (int)((klen + GV_ROWS - 1) / GV_ROWS);
  const int64_t kb0 = p.slayout == kScaleAxis0Block ? kbeg / p.block : 0;
  const int nrows_s = p.slayout == kScaleAxis0Block ? (int)((kend - 1) / p.block - kb0 + 1) : 1;
  int *status = &g_dq_gemv_status;
  __shared__ int issued; // ring stages the producer filled (for the drain after a give-up)

  if (threadIdx.x == 0) {
    abort_flag = 0;
    issued = 0;
    for (int i = 0; i < GV_STAGES; ++i) {
      tc::mbar_init(&full[i], 1);
      tc::mbar_init(&empty[i], GV_CONSUMERS / 32);
    }
    tc::mbar_init(sbar, 1);
    tc::fence_barrier_init();
  }
  // Activations of this K range, staged by every thread before the roles
  // split (no block-wide barrier may follow the split until both roles are
  // done, or the producer's ring waits would deadlock against it).
  for (int e = threadIdx.x; e < MT * p.kchunk; e += GV_THREADS) {
    const int mm = e / p.kchunk;
    const int64_t kk = e % p.kchunk;
    a_s[e] = (mm < p.M && kk < klen)
                 ? reinterpret_cast<const __half *>(p.a)[(int64_t)mm * p.K + kbeg + kk]
                 : __ushort_as_half(0);
  }
  __syncthreads();

  if (warp == GV_CONSUMERS / 32) {
    // ---------------- producer warp ----------------
    if (tc::elect_one()) {
      tc::prefetch_tensormap(&map_w);
      if (p.slayout == kScaleTensor) {
        const __half v = reinterpret_cast<const __half *>(p.scale)[0];
        for (int i = 0; i < GEMV_TN; ++i) s_s[i] = v;
        tc::mbar_arrive(sbar); // release semantics publish the stores above
      } else {
        tc::mbar_expect_tx(sbar, (uint32_t)(nrows_s * GEMV_TN * 2));
        for (int i = 0; i < nrows_s; ++i) {
          const int64_t srow = p.slayout == kScaleAxis0Block ? kb0 + i : 0;
          const uint8_t *src = p.scale + (srow * p.N + n0) * 2;
          asm volatile(
              "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
              ::"r"(tc::smem_u32(s_s + (size_t)i * GEMV_TN)), "l"(src), "r"(GEMV_TN * 2),
              "r"(tc::smem_u32(sbar))
              : "memory");
        }
      }
      for (int t = 0; t < ntiles; ++t) {
        const int s = t % GV_STAGES;
        if (t >= GV_STAGES && !tc::mbar_wait(&empty[s], ((t / GV_STAGES) - 1) & 1)) {
          atomicExch(status, tc::kTimeoutEmpty);
          abort_flag = 1;
          break;
        }
        if (abort_flag) break;
        issued = t + 1;
        tc::mbar_expect_tx(&full[s], GV_STAGE_BYTES);
        tc::tma_load_2d(ring + s * GV_STAGE_BYTES, &map_w, &full[s], (int32_t)(n0 / 2),
                        (int32_t)(kbeg + (int64_t)t * GV_ROWS));
      }
    }
    __syncwarp();
  }
  float acc[MT][32];
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int j = 0; j < 32; ++j) acc[m][j] = 0.0f;

  if (warp < GV_CONSUMERS / 32) {
    bool ok = tc::mbar_wait(sbar, 0);
    if (!ok) {
      atomicExch(status, tc::kTimeoutFull);
      abort_flag = 1;
    }
    const bool is_signed = p.wdt == kInt4;
    const uint32_t flip = is_signed ? 0x88888888u : 0u;
    const uint32_t bias_bits = is_signed ? 0x64086408u : 0x64006400u;
    const int row = warp * 4 + r; // row within a stage
    uint32_t s2[16];
    int cur_sr = -1;
    for (int t = 0; t < ntiles && ok; ++t) {
      const int s = t % GV_STAGES;
      if (!tc::mbar_wait(&full[s], (t / GV_STAGES) & 1)) {
        atomicExch(status, tc::kTimeoutFull);
        abort_flag = 1;
        break;
      }
      const int64_t kk = (int64_t)t * GV_ROWS + row;
      const uint4 raw = *reinterpret_cast<const uint4 *>(ring + s * GV_STAGE_BYTES + row * 128 + c * 16);
      if (kk >= klen) {
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&empty[s]);
        continue;
      }
      const int sr = p.slayout == kScaleAxis0Block
                         ? (int)(p.fdiv_block.div((uint32_t)(kbeg + kk)) - (uint32_t)kb0)
                         : 0;
      if (sr != cur_sr) {
        cur_sr = sr;
        const uint4 *sp = reinterpret_cast<const uint4 *>(s_s + (size_t)sr * GEMV_TN + c * 32);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint4 v = sp[q]; // halves q*8 .. q*8+7
          s2[q * 4 + 0] = __byte_perm(v.x, v.z, 0x5410); // (0, 4)
          s2[q * 4 + 1] = __byte_perm(v.x, v.z, 0x7632); // (1, 5)
          s2[q * 4 + 2] = __byte_perm(v.y, v.w, 0x5410); // (2, 6)
          s2[q * 4 + 3] = __byte_perm(v.y, v.w, 0x7632); // (3, 7)
        }
      }
      uint16_t av[MT];
#pragma unroll
      for (int m = 0; m < MT; ++m) av[m] = __half_as_ushort(a_s[m * p.kchunk + kk]);
      const uint32_t words[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint32_t x = words[q] ^ flip;
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          const uint32_t h = ((x >> (4 * jj)) & 0x000f000fu) | 0x64006400u;
          uint32_t qh, w2;
          asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(qh) : "r"(h), "r"(bias_bits));
          asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(w2) : "r"(qh), "r"(s2[q * 4 + jj]));
          const uint16_t wl = (uint16_t)(w2 & 0xffffu), wh = (uint16_t)(w2 >> 16);
#pragma unroll
          for (int m = 0; m < MT; ++m) {
            acc[m][q * 8 + jj] = fma_f16(av[m], wl, acc[m][q * 8 + jj]);
            acc[m][q * 8 + jj + 4] = fma_f16(av[m], wh, acc[m][q * 8 + jj + 4]);
          }
        }
      }
      // Release the stage only after its data has been consumed: the next TMA
      // fill of this slot must not overtake a shared-memory read in flight.
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&empty[s]);
    }
    // reduce the 4 row-lanes (r) sharing a column chunk
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        acc[m][j] += __shfl_xor_sync(0xffffffffu, acc[m][j], 8);
        acc[m][j] += __shfl_xor_sync(0xffffffffu, acc[m][j], 16);
      }
  }
  __syncthreads();
  if (abort_flag && threadIdx.x == 0) {
    // A wait gave up: let the copies in flight (scale rows, the last fill of
    // each ring stage) land before the ring is reused or the CTA exits.
    tc::mbar_wait(sbar, 0, kWaitNs / 4);
    const int n = issued;
    for (int t = n > GV_STAGES ? n - GV_STAGES : 0; t < n; ++t)
      tc::mbar_wait(&full[t % GV_STAGES], (t / GV_STAGES) & 1, kWaitNs / 4);
  }
  __syncthreads(); // the ring is free: reuse it for the cross-warp reduction
  if (warp < GV_CONSUMERS / 32 && r == 0) {
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
      for (int j = 0; j < 32; ++j) red[(warp * MT + m) * GEMV_TN + c * 32 + j] = acc[m][j];
  }
  __syncthreads();
  float *part = p.ksplit > 1 ? p.partials + (int64_t)split * p.M * p.N : nullptr;
  for (int e = threadIdx.x; e < MT * GEMV_TN; e += GV_THREADS) {
    const int m = e / GEMV_TN, nn = e % GEMV_TN;
    float sum = 0.0f;
#pragma unroll
    for (int w = 0; w < GV_CONSUMERS / 32; ++w) sum += red[(w * MT + m) * GEMV_TN + nn];
    const int64_t gn = n0 + nn;
    if (m < p.M && gn < p.N && !abort_flag) {
      if (part) part[(int64_t)m * p.N + gn] = sum;
      else store_out(p.y, p.ydt, (int64_t)m * p.N + gn, sum);
    }
  }
  if (!part) return;
  // Last contributor merges, unless one of them gave up (partials not valid).
  __shared__ bool gv_last, gv_skip;
  __syncthreads();
  if (threadIdx.x == 0) {
    bool gave_up = false;
    gv_last = arrive_marked(p.counters + blockIdx.x, (uint32_t)p.ksplit, abort_flag != 0, &gave_up);
    gv_skip = gave_up;
  }
  __syncthreads();
  if (!gv_last || gv_skip) return;
  for (int e = threadIdx.x; e < MT * GEMV_TN; e += GV_THREADS) {
    const int m = e / GEMV_TN;
    const int64_t gn = n0 + e % GEMV_TN;
    if (m >= p.M || gn >= p.N) continue;
    float sum = 0.0f;
    for (int sp = 0; sp < p.ksplit; ++sp)
      sum += __ldcg(p.partials + ((int64_t)sp * p.M + m) * p.N + gn);
    store_out(p.y, p.ydt, (int64_t)m * p.N + gn, sum);
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

static int dq_mm_validate(const b2_tensor *a, const b2_tensor *w, const b2_tensor *s,
                          const b2_tensor *zp, int64_t axis, int32_t cast_dt, const b2_tensor *y,
                          DqMmParams &p) {
  B2_ENFORCE(a && w && s && y, "kernel::MatMul: null tensor");
  B2_ENFORCE(w->ndim == 2, "b2_dequantize_matmul: the quantized weight must be rank-2 [K, N]");
  B2_ENFORCE(s->dtype == kFloat || s->dtype == kFloat16,
             "kernel::DequantizeLinear: x_scale must be FLOAT or FLOAT16.");
  const int dq_out = s->dtype;
  const int wdt_eff = cast_dt ? cast_dt : dq_out;
  if (cast_dt)
    B2_ENFORCE(cast_dt == kFloat || cast_dt == kFloat16 || cast_dt == kBfloat16,
               "b2_dequantize_matmul: cast_dtype must be FLOAT, FLOAT16 or BFLOAT16");
  B2_ENFORCE(a->dtype == wdt_eff, "kernel::MatMul inputs must share the same dtype.");
  B2_ENFORCE(a->dtype == kFloat || a->dtype == kFloat16 || a->dtype == kBfloat16,
             "kernel::MatMul: unsupported data type %d", a->dtype);
  // DequantizeLinear layout rules (kernel_dequantizelinear.cc:528-565).
  DqParams dqp{};
  std::vector<int64_t> wshape = shape_of(w);
  int rc = dq_validate(w, s, zp, axis, dq_out, wshape, dqp);
  if (rc) return rc;
  // MatMul shape rules (matmul_shape_utils.h:86-106) with a rank-2 right operand.
  B2_ENFORCE(a->ndim >= 1, "kernel::MatMul does not accept rank-0 inputs.");
  const int64_t K = w->shape[0], N = w->shape[1];
  const int64_t Ka = a->shape[a->ndim - 1];
  B2_ENFORCE(Ka == K, "kernel::MatMul got incompatible inner dimensions.");
  int64_t M = 1;
  for (int i = 0; i < a->ndim - 1; ++i) M *= a->shape[i];
  std::vector<int64_t> out(a->shape, a->shape + a->ndim - 1);
  out.push_back(N);
  B2_ENFORCE(y->dtype == a->dtype, "kernel::MatMul preallocated output must have the same dtype as input A.");
  B2_ENFORCE(shape_of(y) == out, "kernel::MatMul preallocated output has an invalid shape.");
  p.M = M;
  p.K = K;
  p.N = N;
  p.wdt = w->dtype;
  p.s_f16 = s->dtype == kFloat16;
  p.cast_dt = cast_dt;
  p.ydt = a->dtype;
  if (dqp.layout == 0) p.slayout = kScaleTensor;
  else if (axis == 0) p.slayout = dqp.layout == 2 ? kScaleAxis0Block : kScaleAxis0;
  else p.slayout = dqp.layout == 2 ? kScaleAxis1Block : kScaleAxis1;
  p.block = dqp.block;
  p.s_alen = dqp.s_alen;
  B2_ENFORCE(K < (int64_t(1) << 31) && N < (int64_t(1) << 31),
             "b2_dequantize_matmul: K and N must be below 2^31");
  p.fdiv_block = FastDiv((uint32_t)(p.block > 0 ? p.block : 1));
  return B2_OK;
}

struct Plan {
  int kind = 0; // 0 simt, 1 gemv, 2 tensor core, 3 register-MMA decode
  int ksplit = 1;
  int64_t kchunk = 0;
  dim3 grid;
  size_t smem = 0;
  int mt = 1;
  int bits = 4;
  bool fast16 = false;
  int nkb = 0;
  size_t ws = 0;
};

static int wbits(int dt) {
  if (dt == kInt4 || dt == kUint4 || dt == kF4E2M1) return 4;
  if (dt == kInt8 || dt == kUint8 || is_f8(dt)) return 8;
  return 0;
}

// Kernel selection.  ONNXL_B200_DQ_KERNEL=tc|gemv|simt|mma|f32|x|n|c|cx
// forces one family (tests use it to exercise every kernel on the same
// shapes); the default picks, for int4 / fp16, the register-MMA decode
// kernels up to 64 rows (split-K magic-number kernel, or narrow tiles, by the
// rule below), the tensor-core kernel for other 16-bit activations, the
// CUDA-core GEMV for one or two rows, dq_gemm_f32 for FLOAT activations with
// integer weights, and the generic CUDA-core GEMM for the rest.
enum DqPath { kPathAuto = 0, kPathTc = 1, kPathGemv = 2, kPathSimt = 3, kPathMma = 4, kPathF32 = 5,
              kPathX = 6, kPathN = 7, kPathC = 8, kPathCX = 9 };

static DqPath forced_path() {
  const char *e = getenv("ONNXL_B200_DQ_KERNEL");
  if (!e) return kPathAuto;
  if (!strcmp(e, "tc")) return kPathTc;
  if (!strcmp(e, "gemv")) return kPathGemv;
  if (!strcmp(e, "simt")) return kPathSimt;
  if (!strcmp(e, "mma")) return kPathMma;
  if (!strcmp(e, "f32")) return kPathF32;
  if (!strcmp(e, "x")) return kPathX;
  if (!strcmp(e, "n")) return kPathN;
  if (!strcmp(e, "c")) return kPathC;
  if (!strcmp(e, "cx")) return kPathCX;
  return kPathAuto;
}

static Plan make_plan(const DqMmParams &p) {
  Plan pl;
  const int sms = sm_count();
  const int bits = wbits(p.wdt);
  const bool col_layout = p.slayout == kScaleTensor || p.slayout == kScaleAxis0Block ||
                          p.slayout == kScaleAxis1;
  const bool fast16 = (p.wdt == kInt4 || p.wdt == kUint4) && p.s_f16 && p.zp == nullptr &&
                      p.ydt == kFloat16 && (p.cast_dt == 0 || p.cast_dt == kFloat16) &&
                      p.N % GEMV_TN == 0;
  const bool gemv_ok = p.M <= (fast16 ? 4 : 2) && bits && col_layout && p.N % 32 == 0 &&
                       (p.slayout != kScaleAxis0Block || p.block % 32 == 0) &&
                       ((p.N * bits / 8) % 16 == 0);
  const DqPath forced = forced_path();
  if ((forced == kPathC || forced == kPathCX) && dq_c_eligible(p)) {
    pl.kind = forced == kPathC ? 7 : 8;
    pl.ws = 0;
    return pl;
  }
  if (forced == kPathN && dq_n_eligible(p)) {
    pl.kind = 6;
    pl.ws = 0;
    return pl;
  }
  if (forced == kPathX && dq_x_eligible(p)) {
    pl.kind = 5;
    pl.ws = dq_x_workspace(p);
    return pl;
  }
  // Default decode choice for the int4 / fp16 family, by batch (measured on
  // the config-3 projection shapes): up to 8 rows the magic-number split-K
  // kernel; 9 to 16 rows the narrow-tile kernel (no split-K; its
  // dequantization is shared by all activation tiles) when its 32-column
  // tiles fit one wave and K is short (4096 x 4096: 8.2 us against 11.8 us),
  // else the split-K kernel (4096 x 11008: 18.2 against 23.5 us; 11008 x
  // 4096: 17.7 against 20.4 us); 17 to 64 rows the narrow-tile kernel (at 64
  // rows 12.3 / 35.8 / 29.6 us against 31.5 / 47.2 / 49.5 us for the exact
  // kernel with two row passes, kept for M <= 64 outside its reach).
  if (forced == kPathAuto && p.M > 8 && p.M <= 64) {
    const bool narrow_fits = (p.N + 31) / 32 <= sm_count() && p.K <= 8192;
    if (dq_n_eligible(p) && (p.M > 16 || narrow_fits)) {
      pl.kind = 6;
      pl.ws = 0;
      return pl;
    }
    if (p.M > 16 && dq_x_eligible(p)) {
      pl.kind = 5;
      pl.ws = dq_x_workspace(p);
      return pl;
    }
  }
  if ((forced == kPathAuto || forced == kPathMma) && dq_mma_eligible(p)) {
    pl.kind = 3;
    pl.ws = dq_mma_workspace(p);
    return pl;
  }
  if ((forced == kPathAuto && dq_tc_supported(p)) || (forced == kPathTc && dq_tc_eligible(p))) {
    pl.kind = 2;
    pl.ws = dq_tc_workspace(p);
    return pl;
  }
  if (gemv_ok && (forced == kPathAuto || forced == kPathGemv || forced == kPathTc)) {
    pl.kind = 1;
    pl.bits = bits;
    pl.mt = p.M <= 1 ? 1 : p.M <= 2 ? 2 : 4;
    pl.fast16 = fast16;
    const int64_t ntiles = (p.N + GEMV_TN - 1) / GEMV_TN;
    // about two CTAs per SM in one wave
    int64_t want = (2 * sms + ntiles - 1) / ntiles;
    int64_t kchunk = (p.K + want - 1) / want;
    const int64_t align = p.slayout == kScaleAxis0Block ? std::max<int64_t>(32, p.block) : 32;
    kchunk = (kchunk + align - 1) / align * align;
    if (kchunk < 32) kchunk = 32;
    pl.kchunk = kchunk;
    pl.ksplit = (int)((p.K + kchunk - 1) / kchunk);
    if (pl.ksplit > 1 && ntiles > (int64_t)kMaxCounters) {
      pl.kchunk = p.K;
      pl.ksplit = 1;
    }
    pl.grid = dim3((unsigned)ntiles, (unsigned)pl.ksplit, 1);
    const size_t red = (size_t)(GEMV_THREADS / 32) * pl.mt * GEMV_TN * 4;
    if (fast16) {
      pl.nkb = p.slayout == kScaleAxis0Block ? (int)(pl.kchunk / p.block) + 1 : 1;
      pl.smem = (size_t)GV_STAGES * GV_STAGE_BYTES + (size_t)pl.nkb * GEMV_TN * 2 +
                (size_t)pl.mt * pl.kchunk * 2 + 16 + (2 * GV_STAGES + 1) * 8 + 1024;
      pl.smem = std::max(pl.smem, red + 1024);
    } else {
      pl.smem = (size_t)pl.mt * pl.kchunk * 4 + red;
    }
    pl.ws = kCounterBytes + (pl.ksplit > 1 ? (size_t)pl.ksplit * p.M * p.N * 4 : 0);
    return pl;
  }
  if ((forced == kPathAuto || forced == kPathF32) && dq_f32_eligible(p)) {
    pl.kind = 4;
    pl.ws = dq_f32_workspace(p);
    return pl;
  }
  pl.kind = 0;
  const int64_t tn = (p.N + SIMT_BN - 1) / SIMT_BN, tm = (p.M + SIMT_BM - 1) / SIMT_BM;
  int64_t want = (2 * sms + tn * tm - 1) / (tn * tm);
  if (want < 1) want = 1;
  int64_t kchunk = (p.K + want - 1) / want;
  kchunk = (kchunk + SIMT_BK - 1) / SIMT_BK * SIMT_BK;
  if (kchunk < SIMT_BK) kchunk = SIMT_BK;
  pl.kchunk = kchunk;
  pl.ksplit = (int)((p.K + kchunk - 1) / kchunk);
  if (pl.ksplit < 1 || tn * tm > (int64_t)kMaxCounters) {
    pl.kchunk = p.K;
    pl.ksplit = 1;
  }
  pl.grid = dim3((unsigned)tn, (unsigned)tm, (unsigned)pl.ksplit);
  if (pl.ksplit > 1) pl.ws = kCounterBytes + (size_t)pl.ksplit * p.M * p.N * 4;
  return pl;
}

template <typename T> static int launch_simt(const DqMmParams &p, const Plan &pl, cudaStream_t st) {
  dq_gemm_simt<T><<<pl.grid, 256, 0, st>>>(p);
  B2_LAUNCH_CHECK();
  return B2_OK;
}

template <typename K>
static int launch_smem(K kern, const Plan &pl, const DqMmParams &p, cudaStream_t st) {
  if (pl.smem > 48 * 1024)
    B2_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.smem));
  kern<<<pl.grid, GEMV_THREADS, pl.smem, st>>>(p);
  B2_LAUNCH_CHECK();
  return B2_OK;
}

template <int MT>
static int launch_gemv_i4h(const DqMmParams &p, const Plan &pl, cudaStream_t st) {
  CUtensorMap map_w;
  const uint64_t dims[2] = {(uint64_t)p.N / 2, (uint64_t)p.K};
  const uint64_t strides[1] = {(uint64_t)p.N / 2};
  const uint32_t box[2] = {128, GV_ROWS};
  int rc = make_tensor_map(&map_w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, p.w, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  auto kern = dq_gemv_i4h<MT>;
  B2_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.smem));
  kern<<<pl.grid, GV_THREADS, pl.smem, st>>>(map_w, p);
  B2_LAUNCH_CHECK();
  return B2_OK;
}

static int launch_gemv(DqMmParams p, const Plan &pl, cudaStream_t st) {
  p.gemv_nkb = pl.nkb;
  if (pl.fast16) {
    switch (pl.mt) {
    case 1: return launch_gemv_i4h<1>(p, pl, st);
    case 2: return launch_gemv_i4h<2>(p, pl, st);
    default: return launch_gemv_i4h<4>(p, pl, st);
    }
  }
  if (pl.bits == 4) {
    if (pl.mt == 1) return launch_smem(dq_gemv<1, 4>, pl, p, st);
    return launch_smem(dq_gemv<2, 4>, pl, p, st);
  }
  if (pl.mt == 1) return launch_smem(dq_gemv<1, 8>, pl, p, st);
  return launch_smem(dq_gemv<2, 8>, pl, p, st);
}

} // namespace b2

using namespace b2;

extern "C" int b2_dequantize_matmul(const b2_tensor *a, const b2_tensor *w,
                                    const b2_tensor *w_scale, const b2_tensor *w_zero_point,
                                    int64_t axis, int32_t cast_dtype, b2_tensor *y,
                                    void *workspace, size_t *workspace_bytes, void *stream) {
  DqMmParams p{};
  int rc = dq_mm_validate(a, w, w_scale, w_zero_point, axis, cast_dtype, y, p);
  if (rc) return rc;
  const Plan pl = make_plan(p);
  rc = workspace_check(workspace, workspace_bytes, pl.ws);
  if (rc < 0) return rc;
  if (rc == 1) return B2_OK; // size query
  if (p.M == 0 || p.N == 0) return B2_OK;
  p.a = a->data;
  p.w = static_cast<const uint8_t *>(w->data);
  p.scale = static_cast<const uint8_t *>(w_scale->data);
  p.zp = w_zero_point ? static_cast<const uint8_t *>(w_zero_point->data) : nullptr;
  p.y = y->data;
  p.kchunk = pl.kchunk;
  p.ksplit = pl.ksplit;
  if (workspace) {
    p.counters = static_cast<uint32_t *>(workspace);
    p.partials = reinterpret_cast<float *>(static_cast<uint8_t *>(workspace) + kCounterBytes);
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (p.K == 0) {
    // Empty reduction: y = 0.
    B2_CUDA(cudaMemsetAsync(y->data, 0, (size_t)p.M * p.N * (p.ydt == kFloat ? 4 : 2), st));
    return B2_OK;
  }
  if (pl.kind >= 3 && pl.kind <= 8) {
    if (pl.kind == 3 && dq_mma_aligned(p)) return dq_mma_launch(p, workspace, st);
    if (pl.kind == 5 && dq_mma_aligned(p)) return dq_x_launch(p, workspace, st);
    if (pl.kind == 6 && dq_mma_aligned(p)) return dq_n_launch(p, st);
    if ((pl.kind == 7 || pl.kind == 8) && dq_mma_aligned(p)) return dq_c_launch(p, st, pl.kind == 8);
    if (pl.kind == 4 && dq_f32_aligned(p)) return dq_f32_launch(p, workspace, st);
    // TMA / vector loads need aligned tensors: fall back to the unsplit
    // CUDA-core kernel, which needs no workspace.
    Plan one;
    one.kchunk = p.K;
    one.ksplit = 1;
    one.grid = dim3((unsigned)((p.N + SIMT_BN - 1) / SIMT_BN),
                    (unsigned)((p.M + SIMT_BM - 1) / SIMT_BM), 1);
    p.kchunk = p.K;
    p.ksplit = 1;
    if (pl.kind == 4) return launch_simt<float>(p, one, st);
    return launch_simt<__half>(p, one, st);
  }
  if (pl.kind == 2) return dq_tc_launch(p, workspace, st);
  if (pl.kind == 1) return launch_gemv(p, pl, st);
  if (p.ydt == kFloat) return launch_simt<float>(p, pl, st);
  if (p.ydt == kFloat16) return launch_simt<__half>(p, pl, st);
  return launch_simt<__nv_bfloat16>(p, pl, st);
}

// The sharded-output fields of p from one b2_peer_out (after p's validation).
static int peer_fill(const b2_peer_out *out, DqMmParams &p, const char *fn) {
  if (!out) B2_FAIL(B2_ERR_INVALID_ARGUMENT, "%s: null peer output", fn);
  B2_ENFORCE(out->world >= 2 && out->world <= 8, "%s: world must be 2..8", fn);
  B2_ENFORCE(out->rank >= 0 && out->rank < out->world, "%s: rank out of range", fn);
  B2_ENFORCE(out->n_full == p.N * out->world,
             "%s: n_full must be world x the local slice's columns", fn);
  B2_ENFORCE(out->counters != nullptr, "%s: null counters", fn);
  for (int r = 0; r < out->world; ++r)
    B2_ENFORCE(out->full[r] && out->flags[r] && reinterpret_cast<uintptr_t>(out->full[r]) % 16 == 0,
               "%s: peer buffers must be non-null and 16-byte aligned", fn);
  p.y = out->full[out->rank];
  p.world = out->world;
  p.rank = out->rank;
  p.n_full = out->n_full;
  p.col_off = (int64_t)out->rank * p.N;
  for (int r = 0; r < out->world; ++r) {
    p.peer_full[r] = out->full[r];
    p.peer_flags[r] = out->flags[r];
  }
  p.pctr = out->counters;
  p.wait_input = out->wait_input;
  if (!dq_mma_aligned(p) || (p.col_off * 2) % 4 != 0 || (p.n_full * 2) % 4 != 0)
    B2_FAIL(B2_ERR_UNSUPPORTED, "%s: tensors must be 16-byte aligned", fn);
  if (p.M == 0 || p.N == 0 || p.K == 0)
    B2_FAIL(B2_ERR_UNSUPPORTED, "%s: empty shapes are not sharded", fn);
  return B2_OK;
}

extern "C" int b2_dequantize_matmul_peer(const b2_tensor *a, const b2_tensor *w,
                                         const b2_tensor *w_scale, const b2_tensor *w_zero_point,
                                         int64_t axis, int32_t cast_dtype, const b2_tensor *y_local,
                                         const b2_peer_out *out, void *workspace,
                                         size_t *workspace_bytes, void *stream) {
  if (!out) B2_FAIL(B2_ERR_INVALID_ARGUMENT, "b2_dequantize_matmul_peer: null peer output");
  DqMmParams p{};
  int rc = dq_mm_validate(a, w, w_scale, w_zero_point, axis, cast_dtype, y_local, p);
  if (rc) return rc;
  // the fused peer stores live in the register-MMA decode kernel only
  if (forced_path() != kPathAuto || !dq_mma_eligible(p))
    B2_FAIL(B2_ERR_UNSUPPORTED,
            "b2_dequantize_matmul_peer: only the int4 / fp16 decode kernel (M <= 16) stores to peers");
  p.a = a->data;
  p.w = static_cast<const uint8_t *>(w->data);
  p.scale = static_cast<const uint8_t *>(w_scale->data);
  p.zp = nullptr;
  rc = peer_fill(out, p, "b2_dequantize_matmul_peer");
  if (rc) return rc;
  const size_t need = dq_mma_workspace(p);
  rc = workspace_check(workspace, workspace_bytes, need);
  if (rc < 0) return rc;
  if (rc == 1) return B2_OK; // size query
  return dq_mma_launch(p, workspace, static_cast<cudaStream_t>(stream));
}

// Validated parameters of the members of a group call (same a, axis, no
// zero point, no cast).
static int group_params(const char *fn, int32_t count, const b2_tensor *a, const b2_tensor *w,
                        const b2_tensor *w_scale, int64_t axis, const b2_tensor *y, DqMmParams *ps) {
  B2_ENFORCE(count >= 1 && count <= 4, "%s: count must be 1..4", fn);
  B2_ENFORCE(a && w && w_scale && y, "%s: null tensor array", fn);
  for (int i = 0; i < count; ++i) {
    ps[i] = DqMmParams{};
    int rc = dq_mm_validate(a, &w[i], &w_scale[i], nullptr, axis, 0, &y[i], ps[i]);
    if (rc) return rc;
    ps[i].a = a->data;
    ps[i].w = static_cast<const uint8_t *>(w[i].data);
    ps[i].scale = static_cast<const uint8_t *>(w_scale[i].data);
    ps[i].zp = nullptr;
    ps[i].y = y[i].data;
  }
  return B2_OK;
}

extern "C" int b2_dequantize_matmul_group(int32_t count, const b2_tensor *a, const b2_tensor *w,
                                          const b2_tensor *w_scale, int64_t axis, b2_tensor *y,
                                          void *workspace, size_t *workspace_bytes, void *stream) {
  DqMmParams ps[4];
  int rc = group_params("b2_dequantize_matmul_group", count, a, w, w_scale, axis, y, ps);
  if (rc) return rc;
  bool nonempty = true;
  for (int i = 0; i < count; ++i) nonempty = nonempty && ps[i].M > 0 && ps[i].N > 0 && ps[i].K > 0;
  if (forced_path() == kPathAuto && nonempty && dq_mma_group_eligible(ps, count)) {
    rc = workspace_check(workspace, workspace_bytes, dq_mma_group_workspace(ps, count));
    if (rc < 0) return rc;
    if (rc == 1) return B2_OK; // size query
    return dq_mma_launch_group(ps, count, workspace, static_cast<cudaStream_t>(stream));
  }
  // Not one launch: each member as its own call, in order, on one workspace
  // of the largest member's size.
  size_t need = 0;
  for (int i = 0; i < count; ++i) need = std::max(need, make_plan(ps[i]).ws);
  rc = workspace_check(workspace, workspace_bytes, need);
  if (rc < 0) return rc;
  if (rc == 1) return B2_OK; // size query
  for (int i = 0; i < count; ++i) {
    size_t wsb = workspace_bytes ? *workspace_bytes : 0;
    rc = b2_dequantize_matmul(a, &w[i], &w_scale[i], nullptr, axis, 0, &y[i], workspace,
                              workspace ? &wsb : nullptr, stream);
    if (rc) return rc;
  }
  return B2_OK;
}

extern "C" int b2_dequantize_matmul_group_peer(int32_t count, const b2_tensor *a, const b2_tensor *w,
                                               const b2_tensor *w_scale, int64_t axis,
                                               const b2_tensor *y_local, const b2_peer_out *out,
                                               void *workspace, size_t *workspace_bytes,
                                               void *stream) {
  const char *fn = "b2_dequantize_matmul_group_peer";
  if (!out) B2_FAIL(B2_ERR_INVALID_ARGUMENT, "%s: null peer outputs", fn);
  DqMmParams ps[4];
  int rc = group_params(fn, count, a, w, w_scale, axis, y_local, ps);
  if (rc) return rc;
  for (int i = 0; i < count; ++i) {
    rc = peer_fill(&out[i], ps[i], fn);
    if (rc) return rc;
    B2_ENFORCE(out[i].world == out[0].world && out[i].rank == out[0].rank,
               "%s: every member must have the same world and rank", fn);
  }
  // the call's completion is published once, through the first member's
  // flags and counters
  for (int i = 1; i < count; ++i) {
    for (int r = 0; r < out[0].world; ++r) ps[i].peer_flags[r] = ps[0].peer_flags[r];
    ps[i].pctr = ps[0].pctr;
    ps[i].wait_input = ps[0].wait_input;
  }
  if (forced_path() != kPathAuto || !dq_mma_group_eligible(ps, count))
    B2_FAIL(B2_ERR_UNSUPPORTED,
            "%s: the members must share K, the weight type and the scale layout and fit the int4 / "
            "fp16 decode kernel (M <= 16)", fn);
  rc = workspace_check(workspace, workspace_bytes, dq_mma_group_workspace(ps, count));
  if (rc < 0) return rc;
  if (rc == 1) return B2_OK; // size query
  return dq_mma_launch_group(ps, count, workspace, static_cast<cudaStream_t>(stream));
}

// Self-test of the tensor-core GEMM's time-out path (see the header): the
// planned dq_gemm_tc launch runs with no TMA issued, so its first data wait
// runs out after limit_ns; every CTA gives up, arrives on its split-K counter
// with the give-up mark and returns.  Returns the code the kernel recorded.
extern "C" int b2_selftest_gemm_timeout(const b2_tensor *a, const b2_tensor *w,
                                        const b2_tensor *w_scale, b2_tensor *y, void *workspace,
                                        size_t workspace_bytes, int64_t limit_ns, void *stream) {
  if (limit_ns <= 0 || limit_ns > 2000000000ll)
    B2_FAIL(B2_ERR_INVALID_ARGUMENT, "b2_selftest_gemm_timeout: limit must be in (0, 2 s]");
  DqMmParams p{};
  int rc = dq_mm_validate(a, w, w_scale, nullptr, 0, 0, y, p);
  if (rc) return rc;
  if (!dq_tc_eligible(p) || p.M == 0 || p.N == 0 || p.K == 0)
    B2_FAIL(B2_ERR_UNSUPPORTED, "b2_selftest_gemm_timeout: the tensor-core GEMM does not take this shape");
  const size_t need = dq_tc_workspace(p);
  if (workspace == nullptr || workspace_bytes < need)
    B2_FAIL(B2_ERR_WORKSPACE, "b2_selftest_gemm_timeout: workspace of %zu bytes required", need);
  p.a = a->data;
  p.w = static_cast<const uint8_t *>(w->data);
  p.scale = static_cast<const uint8_t *>(w_scale->data);
  p.y = y->data;
  if (status_read_dq_gemm_tc(1) < 0) B2_FAIL(B2_ERR_CUDA, "b2_selftest_gemm_timeout: status reset failed");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  rc = dq_tc_launch(p, workspace, st, (uint64_t)limit_ns, true);
  if (rc) return rc;
  B2_CUDA(cudaStreamSynchronize(st));
  const int v = status_read_dq_gemm_tc(0);
  if (v < 0) B2_FAIL(B2_ERR_CUDA, "b2_selftest_gemm_timeout: status read failed");
  return v;
}
