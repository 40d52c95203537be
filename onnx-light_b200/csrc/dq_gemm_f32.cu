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
//  * lane 0 of warp 0 streams the CTA's operands into a ring of shared-memory
//    stages with TMA (it refills a slot once all eight warps are done with it;
//    a ninth, producer-only warp would cap the registers at 168 per thread) (128 K rows per stage: the activation box [MR rows, 128],
//    the packed weight box [128 rows, 128 columns], and the stage's scale and
//    zero-point rows), so the FMA loop never waits on a global load;
//  * each consumer lane owns 4 adjacent columns and MR activation rows: one
//    2-byte (int4) shared load and one dequantization of 4 weights feed 4 * MR
//    FMAs, issued as packed fp32x2 FMAs; the activations of 4 K rows are one
//    broadcast 128-bit shared load per activation row;
//  * (q - zp) becomes a float with one integer add and one float subtract
//    (the 1.5 * 2^23 magic number), not an int->float conversion.
// Work split: a CTA covers 128 columns x MR rows x a K range; its eight
// consumer warps take 16 rows of every stage and are summed through shared
// memory in warp order; CTAs that share a tile (split-K) are summed by the
// last one to arrive, in split order.  Both orders are fixed, so results are
// reproducible.
#include "dq_matmul.cuh"
#include "tc_common.cuh"

namespace b2 {

// Wait time-outs of dq_gemm_f32 (a TMA copy or a ring slot that never
// arrived); the kernel then skips its remaining work.
__device__ int g_dq_gemm_f32_status;

int status_read_dq_gemm_f32(int reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_dq_gemm_f32_status, sizeof(int)) != cudaSuccess) return -1;
  if (reset && v) {
    const int z = 0;
    if (cudaMemcpyToSymbol(g_dq_gemm_f32_status, &z, sizeof(int)) != cudaSuccess) return -1;
  }
  return v;
}

namespace {

constexpr int F32_KWARPS = 8;                            // warps splitting a stage's K rows (16 each)
constexpr int F32_TN = 128;                              // columns per CTA (4 per lane)
constexpr int F32_SK = 128;                              // K rows per stage (16 per warp)
constexpr int F32_MAXST = 8;                             // ring stages at most
constexpr size_t F32_RING_BUDGET = 200 * 1024;
constexpr int32_t F32_MAGIC = 0x4B400000;                // bit pattern of 1.5 * 2^23
constexpr float F32_MAGIC_F = 12582912.0f;               // 1.5 * 2^23

struct F32Args {
  const uint8_t *scale; // per-column / per-tensor scales (read directly)
  const uint8_t *zp;    // per-column / per-tensor zero points (read directly), nullable
  float *y;             // [M, N]
  float *partials;      // [ksplit][M][N]
  uint32_t *counters;   // one per (column tile, row tile)
  int M, K, N;
  int kchunk;           // K rows per CTA (multiple of F32_SK)
  int ksplit;
  int block;            // axis-0 blocked scales: rows per scale row, else 0
  int srows;            // scale rows per stage box (blocked)
  int slayout;
  int is_signed;
  int s_f16;
  int has_zp;
  int stages;           // ring depth
  uint32_t off_w, off_s, off_z, stage_bytes, tx_bytes; // stage layout
  uint64_t wait_ns;
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

template <int BITS> __device__ __forceinline__ uint32_t ld_codes(const uint8_t *p) {
  if (BITS == 4) return *reinterpret_cast<const uint16_t *>(p);
  return *reinterpret_cast<const uint32_t *>(p);
}

// Scales and zero-point offsets of 4 columns from one scale row at `srow_p`
// (FLOAT or FLOAT16) and `zrow_p` (codes, nullable): mz[i] = magic - zp so
// that float(q - zp) = as_float(mz + q) - magic.
template <int BITS>
__device__ __forceinline__ void scale4(const uint8_t *srow_p, const uint8_t *zrow_p, int s_f16,
                                       int is_signed, float (&s)[4], int (&mz)[4]) {
  if (s_f16) {
    const uint2 h = *reinterpret_cast<const uint2 *>(srow_p);
    s[0] = f16_bits_to_f32((uint16_t)(h.x & 0xffffu));
    s[1] = f16_bits_to_f32((uint16_t)(h.x >> 16));
    s[2] = f16_bits_to_f32((uint16_t)(h.y & 0xffffu));
    s[3] = f16_bits_to_f32((uint16_t)(h.y >> 16));
  } else {
    const float4 f = *reinterpret_cast<const float4 *>(srow_p);
    s[0] = f.x;
    s[1] = f.y;
    s[2] = f.z;
    s[3] = f.w;
  }
  int z[4] = {0, 0, 0, 0};
  if (zrow_p) codes4<BITS>(ld_codes<BITS>(zrow_p), is_signed, z);
#pragma unroll
  for (int i = 0; i < 4; ++i) mz[i] = F32_MAGIC - z[i];
}

// c = a * b + c on two fp32 lanes (one packed instruction on sm_100; the same
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

// GROUPS groups of eight warps; group gr owns activation rows
// [gr MRW, (gr + 1) MRW) of the CTA's MR = GROUPS * MRW, and its eight warps
// split every stage's 128 K rows (16 each).  Two groups of 16 rows (512
// threads, <= 128 registers each) rather than one group of 32 rows keep four
// warps per scheduler to hide the shared-memory latency.
// RG: K rows per activation load (a 128-bit load per activation row for 4,
// 64-bit for 2: 16 rows per warp keep 64 accumulators and two dequantized
// rows within 128 registers).
template <int BITS, int MRW, int GROUPS, int RG = (MRW >= 16 ? 2 : 4)>
__global__ void __launch_bounds__(GROUPS * F32_KWARPS * 32, 1)
    dq_gemm_f32(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_w,
                const __grid_constant__ CUtensorMap map_s, const __grid_constant__ CUtensorMap map_z,
                const F32Args g) {
  extern __shared__ uint8_t dsm[];
  uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(dsm) + 127) & ~uintptr_t(127));
  const size_t ring = (size_t)g.stages * g.stage_bytes;
  constexpr int MR = MRW * GROUPS;
  constexpr int NWARPS = GROUPS * F32_KWARPS;
  constexpr int NTHREADS = NWARPS * 32;
  const size_t red_bytes = (size_t)F32_KWARPS * MR * F32_TN * 4;
  uint64_t *full = reinterpret_cast<uint64_t *>(sm + (ring > red_bytes ? ring : red_bytes));
  uint64_t *empty = full + F32_MAXST;
  volatile int *flags = reinterpret_cast<volatile int *>(empty + F32_MAXST); // [0] abort, [1] last

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * F32_TN;
  const int m0 = blockIdx.y * MR;
  const int split = blockIdx.z;
  const int kbeg = split * g.kchunk;
  const int kend = min(g.K, kbeg + g.kchunk);
  const int nst = (kend - kbeg + F32_SK - 1) / F32_SK;

  if (threadIdx.x == 0) {
    for (int i = 0; i < g.stages; ++i) {
      tc::mbar_init(&full[i], 1);
      tc::mbar_init(&empty[i], NWARPS);
    }
    flags[0] = 0;
    flags[1] = 0;
    tc::fence_barrier_init();
  }
  __syncthreads();

  // Fill `i` of the ring (stage i of this CTA's K range) into slot i % stages.
  auto fill = [&](int i) {
    const int sl = i % g.stages;
    const int k0 = kbeg + i * F32_SK;
    uint8_t *st = sm + (size_t)sl * g.stage_bytes;
    tc::mbar_expect_tx(&full[sl], g.tx_bytes);
    tc::tma_load_2d(st, &map_a, &full[sl], k0, m0);
    tc::tma_load_2d(st + g.off_w, &map_w, &full[sl], n0 * BITS / 8, k0);
    if (g.block) {
      tc::tma_load_2d(st + g.off_s, &map_s, &full[sl], n0, k0 / g.block);
      if (g.has_zp) tc::tma_load_2d(st + g.off_z, &map_z, &full[sl], n0 * BITS / 8, k0 / g.block);
    }
  };
  const bool loader = threadIdx.x == 0;
  int issued = 0;
  if (loader) {
    tc::prefetch_tensormap(&map_a);
    tc::prefetch_tensormap(&map_w);
    if (g.block) {
      tc::prefetch_tensormap(&map_s);
      if (g.has_zp) tc::prefetch_tensormap(&map_z);
    }
    for (; issued < nst && issued < g.stages; ++issued) fill(issued);
  }

  // ------------------------------ consumers -------------------------------
  const int n = n0 + lane * 4;
  const bool col_ok = n < g.N; // N % 4 == 0: all four columns or none
  const int mrows = min(MR, g.M - m0);
  const int kw = warp % F32_KWARPS, grp = warp / F32_KWARPS;
  float acc[MRW][4];
#pragma unroll
  for (int m = 0; m < MRW; ++m)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[m][i] = 0.0f;
  float s[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  int mz[4] = {F32_MAGIC, F32_MAGIC, F32_MAGIC, F32_MAGIC};
  if (!g.block && col_ok) {
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
    } else { // per column
      scale4<BITS>(g.scale + (size_t)n * (g.s_f16 ? 2 : 4),
                   g.zp ? g.zp + (size_t)n * BITS / 8 : nullptr, g.s_f16, g.is_signed, s, mz);
    }
  }
  const int r0 = kw * (F32_SK / F32_KWARPS); // this warp's 16 rows of every stage
  bool ok = true;
  for (int i = 0; i < nst; ++i) {
    const int sl = i % g.stages;
    if (ok && flags[0]) ok = false;
    if (ok && !tc::mbar_wait(&full[sl], (i / g.stages) & 1, g.wait_ns)) {
      atomicExch(&g_dq_gemm_f32_status, tc::kTimeoutFull);
      flags[0] = 1;
      ok = false;
    }
    const int k0 = kbeg + i * F32_SK;
    if (ok && col_ok && k0 + r0 < kend) {
      const uint8_t *st = sm + (size_t)sl * g.stage_bytes;
      if (g.block) {
        // rows k0 + r0 .. + 15 share one scale row (block % 16 == 0)
        const int srow = (k0 + r0) / g.block - k0 / g.block;
        scale4<BITS>(st + g.off_s + (size_t)srow * F32_TN * (g.s_f16 ? 2 : 4) + lane * (g.s_f16 ? 8 : 16),
                     g.has_zp ? st + g.off_z + (size_t)srow * F32_TN * BITS / 8 + lane * BITS / 2 : nullptr,
                     g.s_f16, g.is_signed, s, mz);
      }
      const float *as = reinterpret_cast<const float *>(st) + grp * MRW * F32_SK; // this group's rows
      const uint8_t *ws = st + g.off_w + lane * (BITS / 2);
#pragma unroll
      for (int rq = 0; rq < 16; rq += RG) {
        // dequantize RG rows x 4 columns (rows past K are zero codes against
        // zero activations: their products vanish)
        float wv[RG][4];
#pragma unroll
        for (int j = 0; j < RG; ++j) {
          int q[4];
          codes4<BITS>(ld_codes<BITS>(ws + (size_t)(r0 + rq + j) * (F32_TN * BITS / 8)), g.is_signed, q);
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            float v = __fmul_rn(__int_as_float(mz[c] + q[c]) - F32_MAGIC_F, s[c]);
            if (g.s_f16) v = f16_bits_to_f32(f32_to_f16_bits(v)); // FLOAT16 DequantizeLinear output
            wv[j][c] = v;
          }
        }
#pragma unroll
        for (int m = 0; m < MRW; ++m) {
          float av[RG];
          if constexpr (RG == 4) {
            const float4 a4 = *reinterpret_cast<const float4 *>(as + m * F32_SK + r0 + rq);
            av[0] = a4.x, av[1] = a4.y, av[2] = a4.z, av[3] = a4.w;
          } else {
            const float2 a2 = *reinterpret_cast<const float2 *>(as + m * F32_SK + r0 + rq);
            av[0] = a2.x, av[1] = a2.y;
          }
#pragma unroll
          for (int j = 0; j < RG; ++j) {
            ffma2(acc[m][0], acc[m][1], av[j], wv[j][0], wv[j][1]);
            ffma2(acc[m][2], acc[m][3], av[j], wv[j][2], wv[j][3]);
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) tc::mbar_arrive(&empty[sl]);
    // refill this slot with fill i + stages once every warp is done with it
    if (loader && issued < nst && !flags[0]) {
      if (tc::mbar_wait(&empty[sl], (i / g.stages) & 1, g.wait_ns)) {
        fill(issued);
        ++issued;
      } else {
        atomicExch(&g_dq_gemm_f32_status, tc::kTimeoutEmpty);
        flags[0] = 1;
      }
    }
  }
  // the CTA must not end with copies in flight into its shared memory: wait
  // (bounded) for the last fill of every slot that was issued
  if (loader && flags[0])
    for (int i = issued > g.stages ? issued - g.stages : 0; i < issued; ++i)
      tc::mbar_wait(&full[i % g.stages], (i / g.stages) & 1, g.wait_ns);

  // ---- sum the eight warps' partials in warp order (the ring is free) ----
  __syncthreads();
  float4 *red = reinterpret_cast<float4 *>(sm); // [warp][m][32 lanes]
#pragma unroll
  for (int m = 0; m < MRW; ++m)
    red[(kw * MR + grp * MRW + m) * 32 + lane] = make_float4(acc[m][0], acc[m][1], acc[m][2], acc[m][3]);
  __syncthreads();
  const bool direct = g.ksplit == 1;
  const bool abort = flags[0] != 0;
  const float *redf = reinterpret_cast<const float *>(sm);
  float *part = g.partials + (int64_t)split * g.M * g.N;
  for (int e = threadIdx.x; e < MR * F32_TN; e += NTHREADS) {
    const int m = e / F32_TN, c = e % F32_TN;
    if (abort || m >= mrows || n0 + c >= g.N) continue;
    float v = 0.0f;
#pragma unroll
    for (int w = 0; w < F32_KWARPS; ++w) v += redf[((w * MR + m) * 32) * 4 + c];
    const int64_t o = (int64_t)(m0 + m) * g.N + n0 + c;
    if (direct) g.y[o] = v;
    else part[o] = v;
  }
  if (direct) return;

  // ---- split-K: the last CTA of the tile sums the partials in split order ----
  __syncthreads();
  const int tile = blockIdx.y * gridDim.x + blockIdx.x;
  if (threadIdx.x == 0) {
    __threadfence();
    bool any_gave_up = false;
    const bool last = arrive_marked(g.counters + tile, (uint32_t)g.ksplit, abort, &any_gave_up);
    if (last) __threadfence();
    flags[1] = last && !any_gave_up ? 1 : 0;
  }
  __syncthreads();
  if (!flags[1]) return;
  for (int e = threadIdx.x; e < MR * F32_TN; e += NTHREADS) {
    const int m = e / F32_TN, c = e % F32_TN;
    if (m >= mrows || n0 + c >= g.N) continue;
    const int64_t o = (int64_t)(m0 + m) * g.N + n0 + c;
    float v = 0.0f;
    for (int sp = 0; sp < g.ksplit; ++sp) v += __ldcg(g.partials + (int64_t)sp * g.M * g.N + o);
    g.y[o] = v;
  }
}

struct F32Plan {
  int mr = 32, ksplit = 1, kchunk = 0, srows = 0, stages = 0;
  uint32_t off_w = 0, off_s = 0, off_z = 0, stage_bytes = 0, tx = 0;
  dim3 grid;
  size_t ws = 0, smem = 0;
};

uint32_t up128(uint32_t v) { return (v + 127u) & ~127u; }

F32Plan f32_plan(const DqMmParams &p) {
  F32Plan pl;
  pl.mr = p.M <= 8 ? 8 : p.M <= 16 ? 16 : 32;
  const int bits = (p.wdt == kInt4 || p.wdt == kUint4) ? 4 : 8;
  const int64_t tn = (p.N + F32_TN - 1) / F32_TN, tm = (p.M + pl.mr - 1) / pl.mr;
  const int64_t kblocks = (p.K + F32_SK - 1) / F32_SK;
  int64_t ksplit = std::max<int64_t>(1, sm_count() / (tn * tm));
  ksplit = std::min<int64_t>(ksplit, kblocks);
  if (tn * tm > (int64_t)kMaxCounters) ksplit = 1;
  const int64_t kchunk = (kblocks + ksplit - 1) / ksplit * F32_SK;
  pl.ksplit = (int)((p.K + kchunk - 1) / kchunk);
  pl.kchunk = (int)kchunk;
  pl.grid = dim3((unsigned)tn, (unsigned)tm, (unsigned)pl.ksplit);
  pl.ws = pl.ksplit > 1 ? kCounterBytes + (size_t)pl.ksplit * p.M * p.N * 4 : 0;
  // stage layout: activations [MR][128] fp32, weights [128][128 columns],
  // then (blocked scales) the scale and zero-point rows the stage touches
  if (p.slayout == kScaleAxis0Block) {
    const int b = (int)p.block;
    pl.srows = (F32_SK % b == 0) ? F32_SK / b : (b % F32_SK == 0 ? 1 : F32_SK / b + 2);
  }
  const uint32_t a_bytes = (uint32_t)pl.mr * F32_SK * 4;
  const uint32_t w_bytes = F32_SK * F32_TN * bits / 8;
  const uint32_t s_bytes = (uint32_t)pl.srows * F32_TN * (p.s_f16 ? 2 : 4);
  const uint32_t z_bytes = p.zp && pl.srows ? (uint32_t)pl.srows * F32_TN * bits / 8 : 0;
  pl.off_w = up128(a_bytes);
  pl.off_s = up128(pl.off_w + w_bytes);
  pl.off_z = up128(pl.off_s + s_bytes);
  pl.stage_bytes = up128(pl.off_z + z_bytes);
  pl.tx = a_bytes + w_bytes + s_bytes + z_bytes;
  const int nst = (int)(kchunk / F32_SK);
  pl.stages = (int)std::min<size_t>(F32_RING_BUDGET / pl.stage_bytes, F32_MAXST);
  pl.stages = std::max(1, std::min(pl.stages, nst));
  const size_t red = (size_t)F32_KWARPS * pl.mr * F32_TN * 4;
  const size_t ring = (size_t)pl.stages * pl.stage_bytes;
  pl.smem = std::max(ring, red) + 2 * F32_MAXST * 8 + 16 + 128;
  return pl;
}

template <int BITS, int MRW, int GROUPS>
int f32_launch_t(const DqMmParams &p, const F32Plan &pl, F32Args &g, cudaStream_t st) {
  constexpr int MR = MRW * GROUPS;
  CUtensorMap map_a, map_w, map_s, map_z;
  {
    const uint64_t dims[2] = {(uint64_t)p.K, (uint64_t)p.M};
    const uint64_t strides[1] = {(uint64_t)p.K * 4};
    const uint32_t box[2] = {F32_SK, (uint32_t)MR};
    int rc = make_tensor_map(&map_a, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, p.a, dims, strides, box,
                             CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
  }
  {
    const uint64_t dims[2] = {(uint64_t)p.N * BITS / 8, (uint64_t)p.K};
    const uint64_t strides[1] = {(uint64_t)p.N * BITS / 8};
    const uint32_t box[2] = {F32_TN * BITS / 8, F32_SK};
    int rc = make_tensor_map(&map_w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, p.w, dims, strides, box,
                             CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
  }
  map_s = map_w;
  map_z = map_w;
  if (pl.srows) {
    const uint64_t rows = (uint64_t)p.s_alen;
    {
      const uint64_t dims[2] = {(uint64_t)p.N, rows};
      const uint64_t strides[1] = {(uint64_t)p.N * (p.s_f16 ? 2 : 4)};
      const uint32_t box[2] = {F32_TN, (uint32_t)pl.srows};
      int rc = make_tensor_map(&map_s, p.s_f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                               2, p.scale, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE);
      if (rc) return rc;
    }
    if (p.zp) {
      const uint64_t dims[2] = {(uint64_t)p.N * BITS / 8, rows};
      const uint64_t strides[1] = {(uint64_t)p.N * BITS / 8};
      const uint32_t box[2] = {F32_TN * BITS / 8, (uint32_t)pl.srows};
      int rc = make_tensor_map(&map_z, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, p.zp, dims, strides, box,
                               CU_TENSOR_MAP_SWIZZLE_NONE);
      if (rc) return rc;
    }
  }
  auto kern = dq_gemm_f32<BITS, MRW, GROUPS>;
  B2_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.smem));
  kern<<<pl.grid, GROUPS * F32_KWARPS * 32, pl.smem, st>>>(map_a, map_w, map_s, map_z, g);
  B2_LAUNCH_CHECK();
  return B2_OK;
}

} // namespace

bool dq_f32_eligible(const DqMmParams &p) {
  if (p.ydt != kFloat) return false;
  const bool four = p.wdt == kInt4 || p.wdt == kUint4;
  if (!four && p.wdt != kInt8 && p.wdt != kUint8) return false;
  if (p.cast_dt != 0 && p.cast_dt != kFloat) return false;
  if (p.slayout != kScaleTensor && p.slayout != kScaleAxis0Block && p.slayout != kScaleAxis1)
    return false;
  // a 16-row warp slice shares one scale row
  if (p.slayout == kScaleAxis0Block && (p.block < 16 || p.block % 16 != 0)) return false;
  // TMA row strides are 16-byte multiples: packed weight rows (N / 2 or N
  // bytes), scale rows (N * 4 or N * 2 bytes), activation rows (K * 4 bytes)
  if (p.N % (four ? 32 : 16) != 0 || (p.s_f16 && p.N % 8 != 0) || p.K % 4 != 0) return false;
  if (p.M < 1 || p.K < 1) return false;
  if (p.K > ((int64_t)1 << 30) || p.N > ((int64_t)1 << 30) || p.M > ((int64_t)1 << 30)) return false;
  return true;
}

bool dq_f32_aligned(const DqMmParams &p) {
  auto al = [](const void *q, uintptr_t n) { return (reinterpret_cast<uintptr_t>(q) % n) == 0; };
  // TMA bases (activations, weights, blocked scales / zero points) 16 bytes;
  // per-column scale groups of 4 read directly: 16 (FLOAT) / 8 (FLOAT16)
  return al(p.a, 16) && al(p.w, 16) && al(p.scale, 16) && (p.zp == nullptr || al(p.zp, 16));
}

size_t dq_f32_workspace(const DqMmParams &p) { return f32_plan(p).ws; }

int dq_f32_launch(const DqMmParams &p, void *workspace, cudaStream_t st) {
  const F32Plan pl = f32_plan(p);
  if (pl.ws && workspace == nullptr) B2_FAIL(B2_ERR_WORKSPACE, "workspace of %zu bytes required", pl.ws);
  F32Args g{};
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
  g.ksplit = pl.ksplit;
  g.block = p.slayout == kScaleAxis0Block ? (int)p.block : 0;
  g.srows = pl.srows;
  g.slayout = p.slayout;
  g.is_signed = p.wdt == kInt4 || p.wdt == kInt8;
  g.s_f16 = p.s_f16;
  g.has_zp = p.zp != nullptr;
  g.stages = pl.stages;
  g.off_w = pl.off_w;
  g.off_s = pl.off_s;
  g.off_z = pl.off_z;
  g.stage_bytes = pl.stage_bytes;
  g.tx_bytes = pl.tx;
  g.wait_ns = kWaitNs;
  const bool four = p.wdt == kInt4 || p.wdt == kUint4;
  if (four) {
    if (pl.mr == 8) return f32_launch_t<4, 8, 1>(p, pl, g, st);
    if (pl.mr == 16) return f32_launch_t<4, 8, 2>(p, pl, g, st);
    return f32_launch_t<4, 16, 2>(p, pl, g, st);
  }
  if (pl.mr == 8) return f32_launch_t<8, 8, 1>(p, pl, g, st);
  if (pl.mr == 16) return f32_launch_t<8, 8, 2>(p, pl, g, st);
  return f32_launch_t<8, 16, 2>(p, pl, g, st);
}

} // namespace b2
