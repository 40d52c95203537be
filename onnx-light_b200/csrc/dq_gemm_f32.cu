// FLOAT-activation fused DequantizeLinear -> [Cast] -> MatMul for 4- and
// 8-bit integer weights (INT4 / UINT4 / INT8 / UINT8), FLOAT output: the fp32
// chain of the reference's own CPU case, e.g. A [1, 32, 4096] times an int4
// weight [4096, 4096] with int4 zero points and FLOAT scales blocked by 32.
//
// Reference semantics (onnx_light/onnx_extensions/kernels/kernels/quantization/
// kernel_dequantizelinear.cc:332-520, then kernels/math/kernel_matmul.cc:181-223):
//   w[k, n] = (q[k, n] - zp[k / block, n]) * s[k / block, n]   in fp32,
//   rounded to the DequantizeLinear output type (FLOAT, or FLOAT16 for FLOAT16
//   scales followed by a Cast to FLOAT),  y = A . W  with fp32 accumulation.
// Every weight is formed exactly that way here ((q - zp) exact as an integer,
// one RNE product with the scale, the same half rounding), so the result
// differs from the reference's only by the order of the fp32 sums (rel-L2
// about 1e-7 against the 1e-5 contract).
//
// Why CUDA cores.  The 1e-5 contract on fp32 accumulation rules out the 16-bit
// tensor-core path, and at M <= 64 rows the chain is bound by the FP32 pipe
// (config 1: 1.07 GFLOP against 11.8 MB of HBM traffic, 14.4 us of FMAs at the
// full pipe rate against 1.8 us of HBM).  The kernel is built to keep that pipe
// busy:
//  * each lane owns 4 adjacent columns and MR activation rows, so one weight
//    load (2 bytes of int4) and one dequantization of 4 weights feed 4 * MR
//    FMAs, issued as packed fp32x2 FMAs (MR * 2 instructions);
//  * the activations of the CTA's K range are staged once in shared memory,
//    transposed to [k][m], so the MR values of row k are MR / 4 broadcast
//    128-bit loads;
//  * (q - zp) becomes a float with one integer add and one float subtract
//    (the 1.5 * 2^23 magic number), not an int->float conversion;
//  * weight rows are loaded 8 ahead of use.
// Work split: a CTA covers 128 columns x MR rows x a K range; its eight warps
// take consecutive slices of that range and are summed through shared memory
// in warp order; CTAs that share a tile (split-K) are summed by the last one to
// arrive, in split order.  Both orders are fixed, so results are reproducible.
#include "dq_matmul.cuh"

namespace b2 {

namespace {

constexpr int F32_THREADS = 256;
constexpr int F32_WARPS = F32_THREADS / 32;
constexpr int F32_TN = 128;                  // columns per CTA (4 per lane)
constexpr int F32_KALIGN = 128;              // K range granularity (16 rows per warp)
constexpr size_t F32_SMEM = 128 * 1024;      // staged activations / warp partials
constexpr int32_t F32_MAGIC = 0x4B400000;    // bit pattern of 1.5 * 2^23
constexpr float F32_MAGIC_F = 12582912.0f;   // 1.5 * 2^23

struct F32Args {
  const float *a;     // [M, K]
  const uint8_t *w;   // [K, N] packed
  const uint8_t *scale;
  const uint8_t *zp;  // nullable, dtype of w, layout of the scale
  float *y;           // [M, N]
  float *partials;    // [ksplit][M][N]
  uint32_t *counters; // one per (column tile, row tile)
  int M, K, N;
  int kchunk;         // K rows per CTA (multiple of F32_KALIGN)
  int kstage;         // K rows staged in shared memory at a time (multiple of F32_KALIGN)
  int ksplit;
  int block;          // scale rows cover `block` weight rows (axis-0 blocked), else 0
  int slayout;
  int bits;           // 4 or 8
  int is_signed;
  int s_f16;
};

// Four codes of one weight row (columns n .. n + 3) as integers.
template <int BITS>
__device__ __forceinline__ void codes4(uint32_t raw, int is_signed, int (&q)[4]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (BITS == 4) {
      const uint32_t nib = (raw >> (4 * i)) & 0xfu;
      q[i] = is_signed ? (int)(nib ^ 8u) - 8 : (int)nib;
    } else {
      const uint32_t b = (raw >> (8 * i)) & 0xffu;
      q[i] = is_signed ? (int)(int8_t)b : (int)b;
    }
  }
}

template <int BITS>
__device__ __forceinline__ uint32_t load_row(const uint8_t *base, int64_t elem) {
  if (BITS == 4) return *reinterpret_cast<const uint16_t *>(base + (elem >> 1));
  return *reinterpret_cast<const uint32_t *>(base + elem);
}

// Scales and zero-point offsets of columns n .. n + 3 for scale row `srow`:
// mz[i] = magic - zp so that float(q - zp) = as_float(mz + q) - magic.
template <int BITS>
__device__ __forceinline__ void load_scale(const F32Args &g, int64_t srow, int n, float (&s)[4],
                                           int (&mz)[4]) {
  if (g.slayout == kScaleTensor) {
    const float v = g.s_f16 ? f16_bits_to_f32(*reinterpret_cast<const uint16_t *>(g.scale))
                            : *reinterpret_cast<const float *>(g.scale);
    int z = 0;
    if (g.zp) {
      int q[4];
      codes4<BITS>(BITS == 4 ? (uint32_t)(g.zp[0] & 0xfu) : (uint32_t)g.zp[0], g.is_signed, q);
      z = q[0];
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      s[i] = v;
      mz[i] = F32_MAGIC - z;
    }
    return;
  }
  const int64_t e = srow * g.N + n; // kScaleAxis0Block (srow = k / block) or kScaleAxis1 (srow = 0)
  if (g.s_f16) {
    const uint2 h = *reinterpret_cast<const uint2 *>(g.scale + e * 2);
    s[0] = f16_bits_to_f32((uint16_t)(h.x & 0xffffu));
    s[1] = f16_bits_to_f32((uint16_t)(h.x >> 16));
    s[2] = f16_bits_to_f32((uint16_t)(h.y & 0xffffu));
    s[3] = f16_bits_to_f32((uint16_t)(h.y >> 16));
  } else {
    const float4 f = *reinterpret_cast<const float4 *>(g.scale + e * 4);
    s[0] = f.x;
    s[1] = f.y;
    s[2] = f.z;
    s[3] = f.w;
  }
  int z[4] = {0, 0, 0, 0};
  if (g.zp) codes4<BITS>(load_row<BITS>(g.zp, e), g.is_signed, z);
#pragma unroll
  for (int i = 0; i < 4; ++i) mz[i] = F32_MAGIC - z[i];
}

// d = a * b + c on two fp32 lanes (one packed instruction on sm_100; the same
// IEEE fma per element).
__device__ __forceinline__ void ffma2(float &c0, float &c1, float a, float b0, float b1) {
  uint64_t c;
  asm("{\n\t.reg .b64 ra, rb, rc;\n\t"
      "mov.b64 ra, {%1, %1};\n\tmov.b64 rb, {%2, %3};\n\tmov.b64 rc, {%4, %5};\n\t"
      "fma.rn.f32x2 %0, ra, rb, rc;\n\t}"
      : "=l"(c)
      : "f"(a), "f"(b0), "f"(b1), "f"(c0), "f"(c1));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(c0), "=f"(c1) : "l"(c));
}

template <int BITS, int MR>
__global__ void __launch_bounds__(F32_THREADS, 1) dq_gemm_f32(const F32Args g) {
  extern __shared__ float4 sm4[];
  float *sm = reinterpret_cast<float *>(sm4);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * F32_TN;
  const int m0 = blockIdx.y * MR;
  const int split = blockIdx.z;
  const int kbeg = split * g.kchunk;
  const int kend = min(g.K, kbeg + g.kchunk);
  const int n = n0 + lane * 4;
  const bool col_ok = n < g.N; // N % 4 == 0: all four columns or none
  const int mrows = min(MR, g.M - m0);

  float acc[MR][4];
#pragma unroll
  for (int m = 0; m < MR; ++m)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[m][i] = 0.0f;

  float s[4];
  int mz[4];
  if (g.slayout != kScaleAxis0Block && col_ok) load_scale<BITS>(g, 0, n, s, mz);

  for (int k0 = kbeg; k0 < kend; k0 += g.kstage) {
    const int krows = min(g.kstage, kend - k0);
    __syncthreads(); // the previous stage's activations are consumed
    // Stage A[m0 .. m0 + MR, k0 .. k0 + kstage] as [k][m] (zeros past M / K):
    // thread -> (row m, 4 consecutive k), so a warp's shared stores hit
    // distinct banks.
    for (int e = threadIdx.x; e < MR * (g.kstage / 4); e += F32_THREADS) {
      const int m = e % MR, kq = e / MR;
      float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      if (m < mrows && 4 * kq < krows)
        v = *reinterpret_cast<const float4 *>(g.a + (int64_t)(m0 + m) * g.K + k0 + 4 * kq);
      sm[(4 * kq + 0) * MR + m] = v.x;
      sm[(4 * kq + 1) * MR + m] = v.y;
      sm[(4 * kq + 2) * MR + m] = v.z;
      sm[(4 * kq + 3) * MR + m] = v.w;
    }
    __syncthreads();
    if (!col_ok) continue;
    // this warp's slice of the staged rows
    const int per = g.kstage / F32_WARPS;
    const int kw0 = k0 + warp * per;
    const int kw1 = min(kw0 + per, k0 + krows);
    if (kw0 >= kw1) continue;
    int next_srow_k = kw0; // first row of the next scale block (axis-0 blocked)
    int64_t srow = g.block ? kw0 / g.block : 0;
    uint32_t buf[8];
#pragma unroll
    for (int j = 0; j < 8; ++j)
      buf[j] = kw0 + j < kw1 ? load_row<BITS>(g.w, (int64_t)(kw0 + j) * g.N + n) : 0u;
    for (int kb = kw0; kb < kw1; kb += 8) {
      uint32_t cur[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        cur[j] = buf[j];
        const int kn = kb + 8 + j;
        buf[j] = kn < kw1 ? load_row<BITS>(g.w, (int64_t)kn * g.N + n) : 0u;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int k = kb + j;
        if (k >= kw1) break;
        if (g.block && k == next_srow_k) {
          srow = k / g.block;
          load_scale<BITS>(g, srow, n, s, mz);
          next_srow_k = (int)((srow + 1) * g.block);
        }
        int q[4];
        codes4<BITS>(cur[j], g.is_signed, q);
        float wv[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          float v = __fmul_rn(__int_as_float(mz[i] + q[i]) - F32_MAGIC_F, s[i]);
          if (g.s_f16) v = f16_bits_to_f32(f32_to_f16_bits(v)); // FLOAT16 DequantizeLinear output
          wv[i] = v;
        }
        const float4 *arow = reinterpret_cast<const float4 *>(sm + (k - k0) * MR);
#pragma unroll
        for (int mq = 0; mq < MR / 4; ++mq) {
          const float4 av = arow[mq];
          ffma2(acc[4 * mq + 0][0], acc[4 * mq + 0][1], av.x, wv[0], wv[1]);
          ffma2(acc[4 * mq + 0][2], acc[4 * mq + 0][3], av.x, wv[2], wv[3]);
          ffma2(acc[4 * mq + 1][0], acc[4 * mq + 1][1], av.y, wv[0], wv[1]);
          ffma2(acc[4 * mq + 1][2], acc[4 * mq + 1][3], av.y, wv[2], wv[3]);
          ffma2(acc[4 * mq + 2][0], acc[4 * mq + 2][1], av.z, wv[0], wv[1]);
          ffma2(acc[4 * mq + 2][2], acc[4 * mq + 2][3], av.z, wv[2], wv[3]);
          ffma2(acc[4 * mq + 3][0], acc[4 * mq + 3][1], av.w, wv[0], wv[1]);
          ffma2(acc[4 * mq + 3][2], acc[4 * mq + 3][3], av.w, wv[2], wv[3]);
        }
      }
    }
  }

  // ---- sum the eight warps' partials in warp order ----
  __syncthreads();
  float4 *red = sm4; // [warp][m][128 columns] as float4 per lane
#pragma unroll
  for (int m = 0; m < MR; ++m)
    red[(warp * MR + m) * 32 + lane] = make_float4(acc[m][0], acc[m][1], acc[m][2], acc[m][3]);
  __syncthreads();
  const bool direct = g.ksplit == 1;
  float *part = g.partials + (int64_t)split * g.M * g.N;
  for (int e = threadIdx.x; e < MR * F32_TN; e += F32_THREADS) {
    const int m = e / F32_TN, c = e % F32_TN;
    if (m >= mrows || n0 + c >= g.N) continue;
    float v = 0.0f;
#pragma unroll
    for (int w = 0; w < F32_WARPS; ++w) v += sm[((w * MR + m) * 32) * 4 + c];
    const int64_t o = (int64_t)(m0 + m) * g.N + n0 + c;
    if (direct) g.y[o] = v;
    else part[o] = v;
  }
  if (direct) return;

  // ---- split-K: the last CTA of the tile sums the partials in split order ----
  __shared__ bool last;
  __syncthreads();
  const int tile = blockIdx.y * gridDim.x + blockIdx.x;
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t prev = atomicAdd(g.counters + tile, 1u);
    last = prev + 1 == (uint32_t)g.ksplit;
    if (last) {
      __threadfence();
      g.counters[tile] = 0u;
    }
  }
  __syncthreads();
  if (!last) return;
  for (int e = threadIdx.x; e < MR * F32_TN; e += F32_THREADS) {
    const int m = e / F32_TN, c = e % F32_TN;
    if (m >= mrows || n0 + c >= g.N) continue;
    const int64_t o = (int64_t)(m0 + m) * g.N + n0 + c;
    float v = 0.0f;
    for (int sp = 0; sp < g.ksplit; ++sp) v += __ldcg(g.partials + (int64_t)sp * g.M * g.N + o);
    g.y[o] = v;
  }
}

struct F32Plan {
  int mr = 32, ksplit = 1, kchunk = 0, kstage = 0;
  dim3 grid;
  size_t ws = 0;
};

F32Plan f32_plan(const DqMmParams &p) {
  F32Plan pl;
  pl.mr = p.M <= 8 ? 8 : p.M <= 16 ? 16 : 32;
  const int64_t tn = (p.N + F32_TN - 1) / F32_TN, tm = (p.M + pl.mr - 1) / pl.mr;
  const int64_t kblocks = (p.K + F32_KALIGN - 1) / F32_KALIGN;
  int64_t ksplit = std::max<int64_t>(1, sm_count() / (tn * tm));
  ksplit = std::min<int64_t>(ksplit, kblocks);
  if (tn * tm > (int64_t)kMaxCounters) ksplit = 1;
  const int64_t kchunk = (kblocks + ksplit - 1) / ksplit * F32_KALIGN;
  pl.ksplit = (int)((p.K + kchunk - 1) / kchunk);
  pl.kchunk = (int)kchunk;
  // staged rows: the CTA's whole range if it fits, else F32_SMEM / (MR * 4)
  const int64_t cap = (int64_t)(F32_SMEM / ((size_t)pl.mr * 4)) / F32_KALIGN * F32_KALIGN;
  pl.kstage = (int)std::min<int64_t>(kchunk, cap);
  pl.grid = dim3((unsigned)tn, (unsigned)tm, (unsigned)pl.ksplit);
  pl.ws = pl.ksplit > 1 ? kCounterBytes + (size_t)pl.ksplit * p.M * p.N * 4 : 0;
  return pl;
}

template <int BITS, int MR> int f32_launch_t(const F32Args &g, const F32Plan &pl, cudaStream_t st) {
  auto kern = dq_gemm_f32<BITS, MR>;
  const size_t smem = std::max((size_t)pl.kstage * MR * 4, (size_t)F32_WARPS * MR * F32_TN * 4);
  B2_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  kern<<<pl.grid, F32_THREADS, smem, st>>>(g);
  B2_LAUNCH_CHECK();
  return B2_OK;
}

} // namespace

bool dq_f32_eligible(const DqMmParams &p) {
  if (p.ydt != kFloat) return false;
  if (p.wdt != kInt4 && p.wdt != kUint4 && p.wdt != kInt8 && p.wdt != kUint8) return false;
  if (p.cast_dt != 0 && p.cast_dt != kFloat) return false;
  if (p.slayout != kScaleTensor && p.slayout != kScaleAxis0Block && p.slayout != kScaleAxis1)
    return false;
  // 4 columns per lane: whole 2- / 4-byte weight groups and 16-byte (fp32) or
  // 8-byte (fp16) scale groups; K % 4 for the 16-byte activation loads
  if (p.N % 4 != 0 || p.K % 4 != 0 || p.M < 1 || p.K < 1) return false;
  if (p.K > ((int64_t)1 << 30) || p.N > ((int64_t)1 << 30)) return false;
  return true;
}

bool dq_f32_aligned(const DqMmParams &p) {
  auto al = [](const void *q, uintptr_t n) { return (reinterpret_cast<uintptr_t>(q) % n) == 0; };
  const bool four = p.wdt == kInt4 || p.wdt == kUint4;
  return al(p.a, 16) && al(p.w, four ? 2 : 4) && (p.zp == nullptr || al(p.zp, four ? 2 : 4)) &&
         al(p.scale, p.s_f16 ? 8 : 16);
}

size_t dq_f32_workspace(const DqMmParams &p) { return f32_plan(p).ws; }

int dq_f32_launch(const DqMmParams &p, void *workspace, cudaStream_t st) {
  const F32Plan pl = f32_plan(p);
  if (pl.ws && workspace == nullptr) B2_FAIL(B2_ERR_WORKSPACE, "workspace of %zu bytes required", pl.ws);
  F32Args g{};
  g.a = static_cast<const float *>(p.a);
  g.w = p.w;
  g.scale = p.scale;
  g.zp = p.zp;
  g.y = static_cast<float *>(p.y);
  if (workspace) {
    g.counters = static_cast<uint32_t *>(workspace);
    g.partials = reinterpret_cast<float *>(static_cast<uint8_t *>(workspace) + kCounterBytes);
  }
  g.M = (int)p.M;
  g.K = (int)p.K;
  g.N = (int)p.N;
  g.kchunk = pl.kchunk;
  g.kstage = pl.kstage;
  g.ksplit = pl.ksplit;
  g.block = p.slayout == kScaleAxis0Block ? (int)p.block : 0;
  g.slayout = p.slayout;
  g.bits = (p.wdt == kInt4 || p.wdt == kUint4) ? 4 : 8;
  g.is_signed = p.wdt == kInt4 || p.wdt == kInt8;
  g.s_f16 = p.s_f16;
  if (g.bits == 4) {
    if (pl.mr == 8) return f32_launch_t<4, 8>(g, pl, st);
    if (pl.mr == 16) return f32_launch_t<4, 16>(g, pl, st);
    return f32_launch_t<4, 32>(g, pl, st);
  }
  if (pl.mr == 8) return f32_launch_t<8, 8>(g, pl, st);
  if (pl.mr == 16) return f32_launch_t<8, 16>(g, pl, st);
  return f32_launch_t<8, 32>(g, pl, st);
}

} // namespace b2
