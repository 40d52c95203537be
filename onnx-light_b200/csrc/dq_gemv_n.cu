// Decode-shaped fused DequantizeLinear -> [Cast] -> MatMul on narrow column
// tiles: INT4 / UINT4 weights, FLOAT16 scales (no zero point), FLOAT16
// activations and output, M <= 64 rows.  The weight is dequantized exactly as
// the reference does (fp16(q * s), see dq_gemv_x.cu for the argument) and
// multiplied on mma.sync with fp32 accumulation.
//
// Reference semantics (onnx_light/onnx_extensions/kernels/kernels/quantization/
// kernel_dequantizelinear.cc:332-520 then kernels/math/kernel_matmul.cc:181-223).
//
// Why narrow tiles.  A decode projection moves a few MB and its launch is
// latency-bound: in the stream-K kernels (dq_gemv_mma, dq_gemv_x) the
// critical path of a 4096 x 4096 launch is dominated not by streaming but by
// the cross-CTA split-K merge (partial stores, an acquire/release arrival, the
// last arriver's reads of every partial) that follows it.  Here a CTA owns 32
// whole columns (16 packed bytes per weight row) over the full K range, so no
// tile is ever shared between CTAs: the eight warps split K among themselves
// and are summed once through shared memory.  Each 16-byte row piece is half
// a DRAM sector; the neighbouring CTA reads the other half at the same time,
// so L2 serves it and HBM traffic stays the packed weight once.
//
// Pipeline: the K range is cut into chunks of 256 / NT rows (64 at least);
// chunk c belongs to warp c % 8, which owns its own ring slots and loads its
// own chunks by TMA (weights, the chunk's scale rows, the activation slice in
// 128-byte swizzled 64-column boxes), so warps never wait for one another
// before the final reduction.  The activation fragments of a k16 step come
// from one non-transposing ldmatrix per pair of 8-row tiles.  The first
// ring fill's weights and scales of every warp are requested before the
// programmatic-launch wait (they do not depend on the kernel ahead), their
// activations after it.  Up to four activation tiles every mma.sync
// accumulator chain alternates between two register sets, so consecutive k16
// steps do not wait on each other's results (eight tiles give the same
// independence within a step).
#include "dq_matmul.cuh"
#include "tc_common.cuh"

namespace b2 {

// Wait time-outs of the narrow-tile decode kernel (a TMA copy that never
// arrived); the kernel then skips its remaining work.
__device__ int g_gemv_n_status;

int status_read_gemv_n(int reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_gemv_n_status, sizeof(int)) != cudaSuccess) return -1;
  if (reset && v) {
    const int z = 0;
    if (cudaMemcpyToSymbol(g_gemv_n_status, &z, sizeof(int)) != cudaSuccess) return -1;
  }
  return v;
}

namespace {

constexpr int GN_TN = 32;                  // columns per tile (16 packed bytes per row)
constexpr int GN_WARPS = 8;
constexpr int GN_THREADS = GN_WARPS * 32;
constexpr int GN_CH_MIN = 64;              // smallest chunk (one 64-column activation box)
constexpr int GN_MAX_ROWS = 64;            // activation rows (eight 8-row tiles)

// Ring slots per warp for each activation-tile count (shared memory bound).
#ifndef GN_SPW1
#define GN_SPW1 2
#endif
#ifndef GN_SPW2
#define GN_SPW2 3
#endif
#ifndef GN_SPW4
#define GN_SPW4 4
#endif
#ifndef GN_SPW8
#define GN_SPW8 2
#endif

struct GnArgs {
  __half *y;
  int M, N, K;
  int ntiles, nchunks, grid;
  int block;     // scale block along K (0: one scale row for all K)
  int srows;     // scale rows loaded per chunk (0: per-tensor scale)
  int arows;     // activation rows loaded per box (min(M, 8 NT))
  const uint16_t *scalar_scale;
  int is_signed;
  uint64_t wait_ns;
};

// Chunk rows per activation-tile count: the activation slice of a chunk
// (rows x 8 NT x 2 bytes) stays 4 KB up to four tiles (8 KB for eight), and
// every warp owns kSpw ring slots.
template <int NT> struct GnCfg {
  static constexpr int kCh = 256 / NT < GN_CH_MIN ? GN_CH_MIN : 256 / NT; // weight rows per chunk
  static constexpr int kSpw = NT == 1 ? GN_SPW1 : NT == 2 ? GN_SPW2 : NT == 4 ? GN_SPW4 : GN_SPW8;
  static constexpr int kSlots = GN_WARPS * kSpw;
  static constexpr int kSets = NT >= 8 ? 1 : 2;               // accumulator sets (k16 parity)
  static constexpr uint32_t kW = kCh * GN_TN / 2;             // packed weights of a chunk
  static constexpr int kScRows = kCh / 16;                    // scale rows per chunk at most (block 16)
  static constexpr uint32_t kSc = kScRows * GN_TN * 2;
  static constexpr uint32_t kABox = 8u * NT * 128;            // one 64-column box, 8 NT rows
  static constexpr uint32_t kA = (kCh / 64) * kABox;          // a chunk's activations
  static constexpr uint32_t kOffA = kSlots * kW;              // 1024-aligned (swizzled boxes)
  static constexpr uint32_t kOffS = kOffA + kSlots * kA;
  static constexpr uint32_t kOffRed = kOffS + kSlots * kSc;
  static constexpr uint32_t kRedBytes = GN_WARPS * 2 * NT * 4 * 32 * 4;
  static constexpr uint32_t kOffBar = kOffRed + kRedBytes;
  static constexpr uint32_t kBytes = kOffBar + kSlots * 8 + 16;
  static constexpr size_t kDynamic = kBytes + 1024; // alignment slack
  static_assert(kOffA % 1024 == 0 && kABox % 1024 == 0, "swizzled activation boxes");
  static_assert(kDynamic <= 232448, "shared memory per CTA");
};

__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, "
      "{%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm_t4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm2(uint32_t addr, uint32_t (&r)[2]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];"
               : "=r"(r[0]), "=r"(r[1])
               : "r"(addr));
}
// Two fp16 weights from two packed codes at bits 0..3 and 16..19 of `v`:
// (1024 + code') - magic = q exactly, then q * s rounded to nearest even.
__device__ __forceinline__ uint32_t dq2(uint32_t v, uint32_t magic, uint32_t s2) {
  uint32_t h = (v & 0x000f000fu) ^ magic, q, w;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(q) : "r"(h), "r"(magic));
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(w) : "r"(q), "r"(s2));
  return w;
}

template <int NT>
__global__ void __launch_bounds__(GN_THREADS, 1)
    dq_gemv_n(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_a,
              const __grid_constant__ CUtensorMap map_s, const GnArgs g) {
  using C = GnCfg<NT>;
  constexpr int SPW = C::kSpw;
  constexpr int NS = C::kSets;
  static_assert(C::kCh % 64 == 0 && C::kCh >= GN_CH_MIN, "whole 64-column activation boxes");
  extern __shared__ uint8_t dsm[];
  uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(dsm) + 1023) & ~uintptr_t(1023));
  uint64_t *full = reinterpret_cast<uint64_t *>(sm + C::kOffBar);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(full + C::kSlots);
  float *red = reinterpret_cast<float *>(sm + C::kOffRed);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gq = lane >> 2;
  if (threadIdx.x == 0) {
    for (int i = 0; i < C::kSlots; ++i) tc::mbar_init(&full[i], 1);
    *abort_flag = 0;
    tc::fence_barrier_init();
    tc::prefetch_tensormap(&map_w);
    tc::prefetch_tensormap(&map_a);
    if (g.srows) tc::prefetch_tensormap(&map_s);
  }
  __syncthreads();

  // This warp's chunks over every tile of the CTA: tile t = blockIdx.x +
  // grid * it, chunk c = warp + 8 j.  `seq` numbers them in order; fill seq
  // goes to slot 2 warp + (seq & 1) with phase (seq >> 1) & 1.
  const int nmy = (g.nchunks - warp + GN_WARPS - 1) / GN_WARPS; // chunks per tile of this warp
  const int ntile_mine = (g.ntiles - (int)blockIdx.x + g.grid - 1) / g.grid;
  const int total = nmy * ntile_mine;
  const uint32_t tx = C::kW + (uint32_t)(C::kCh / 64) * g.arows * 128 + (uint32_t)g.srows * GN_TN * 2;
  auto coords = [&](int seq, int &tile, int &k0) {
    const int it = seq / nmy, j = seq % nmy;
    tile = (int)blockIdx.x + g.grid * it;
    k0 = (warp + GN_WARPS * j) * C::kCh;
  };
  auto fill_w = [&](int seq) {
    int tile, k0;
    coords(seq, tile, k0);
    const int sl = warp * SPW + seq % SPW;
    tc::mbar_expect_tx(&full[sl], tx);
    tc::tma_load_2d(sm + sl * C::kW, &map_w, &full[sl], tile * (GN_TN / 2), k0);
    if (g.srows) {
      const int srow = g.block ? k0 / g.block : 0;
      tc::tma_load_2d(sm + C::kOffS + sl * C::kSc, &map_s, &full[sl], tile * GN_TN, srow);
    }
  };
  auto fill_a = [&](int seq) {
    int tile, k0;
    coords(seq, tile, k0);
    const int sl = warp * SPW + seq % SPW;
    uint8_t *sa = sm + C::kOffA + sl * C::kA;
#pragma unroll
    for (int q = 0; q < C::kCh / 64; ++q) tc::tma_load_2d(sa + q * C::kABox, &map_a, &full[sl], k0 + 64 * q, 0);
  };
  const int pre = total < SPW ? total : SPW;
  int nissued = pre; // fills this warp has requested (lane 0's count)
  if (lane == 0)
    for (int s = 0; s < pre; ++s) fill_w(s);
  // Everything below may read what the previous kernel on the stream wrote
  // (activations) or write what it reads (the output).
  griddep_wait();
  griddep_launch();
  if (lane == 0)
    for (int s = 0; s < pre; ++s) fill_a(s);

  const uint32_t magic = g.is_signed ? 0x64086408u : 0x64006400u; // fp16 (1032, 1032) / (1024, 1024)
  uint32_t scalar2 = 0;
  if (!g.srows) {
    const uint32_t h = __ldg(g.scalar_scale);
    scalar2 = h | (h << 16);
  }
  const int mi = lane >> 3;
  bool ok = true;
  int seq = 0;
  for (int it = 0; it < ntile_mine; ++it) {
    const int tile = (int)blockIdx.x + g.grid * it;
    float acc[NS][2][NT][4]; // [set][m-tile][activation tile][fragment]
#pragma unroll
    for (int st = 0; st < NS; ++st)
#pragma unroll
      for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[st][mt][nt][e] = 0.0f;
    for (int j = 0; j < nmy; ++j, ++seq) {
      const int sl = warp * SPW + seq % SPW;
      if (ok && *abort_flag) ok = false;
      if (ok && !tc::mbar_wait(&full[sl], (seq / SPW) & 1, g.wait_ns)) {
        atomicExch(&g_gemv_n_status, tc::kTimeoutFull);
        *abort_flag = 1;
        ok = false;
      }
      const int k0 = (warp + GN_WARPS * j) * C::kCh;
      if (ok) {
        const uint8_t *wst = sm + sl * C::kW;
        const uint8_t *ast = sm + C::kOffA + sl * C::kA;
        const uint8_t *sst = sm + C::kOffS + sl * C::kSc;
        uint32_t slo[2] = {scalar2, scalar2}, shi[2] = {scalar2, scalar2};
        int cur_srow = -1;
#pragma unroll 2
        for (int kk = 0; kk < C::kCh; kk += 32) {
          // rows kk .. kk + 31 of the chunk: matrices (rows kk + 8 i + (lane & 7))
          uint32_t r[4];
          ldsm_t4(tc::smem_u32(wst + (kk + 8 * mi + (lane & 7)) * 16), r);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int r0 = kk + 16 * h; // k16 step rows r0 .. r0 + 15
            if (g.srows) {
              const int srow = (g.block && g.block < C::kCh) ? r0 / g.block : 0;
              if (srow != cur_srow) {
                cur_srow = srow;
                const uint2 w4 = *reinterpret_cast<const uint2 *>(sst + srow * GN_TN * 2 + gq * 8);
                slo[0] = __byte_perm(w4.x, w4.x, 0x1010);
                shi[0] = __byte_perm(w4.x, w4.x, 0x3232);
                slo[1] = __byte_perm(w4.y, w4.y, 0x1010);
                shi[1] = __byte_perm(w4.y, w4.y, 0x3232);
              }
            }
            // activation fragments of the k16 step: non-transposing ldmatrix
            // of the swizzled box, matrix i of lane group i = (tile 2p + (i >> 1),
            // k half i & 1); lane (g, t) receives row g, k 2t and 2t + 1
            uint32_t B0[NT], B1[NT];
            {
              const uint8_t *box = ast + (r0 >> 6) * C::kABox;
              const int ch0 = (r0 & 63) >> 3; // first 16-byte chunk of the step
#pragma unroll
              for (int pr = 0; pr < (NT + 1) / 2; ++pr) {
                const int row = (2 * pr + ((mi >> 1) & (NT > 1 ? 1 : 0))) * 8 + (lane & 7);
                const uint32_t addr = tc::smem_u32(box + row * 128 + (((ch0 + (mi & 1)) ^ (row & 7)) << 4));
                if constexpr (NT == 1) {
                  uint32_t r2[2];
                  ldsm2(addr, r2);
                  B0[0] = r2[0];
                  B1[0] = r2[1];
                } else {
                  uint32_t r4[4];
                  ldsm4(addr, r4);
                  B0[2 * pr] = r4[0];
                  B1[2 * pr] = r4[1];
                  B0[2 * pr + 1] = r4[2];
                  B1[2 * pr + 1] = r4[3];
                }
              }
            }
            const uint32_t x = r[2 * h], y = r[2 * h + 1]; // rows r0 + 2t.. and r0 + 8 + 2t..
            {
              const uint32_t a0 = dq2(x, magic, slo[0]), a1 = dq2(x >> 4, magic, shi[0]);
              const uint32_t a2 = dq2(y, magic, slo[0]), a3 = dq2(y >> 4, magic, shi[0]);
#pragma unroll
              for (int nt = 0; nt < NT; ++nt) mma16816(acc[h % NS][0][nt], a0, a1, a2, a3, B0[nt], B1[nt]);
            }
            {
              const uint32_t a0 = dq2(x >> 8, magic, slo[1]), a1 = dq2(x >> 12, magic, shi[1]);
              const uint32_t a2 = dq2(y >> 8, magic, slo[1]), a3 = dq2(y >> 12, magic, shi[1]);
#pragma unroll
              for (int nt = 0; nt < NT; ++nt) mma16816(acc[h % NS][1][nt], a0, a1, a2, a3, B0[nt], B1[nt]);
            }
          }
        }
      }
      (void)k0;
      // this warp alone reads the slot: once every lane is past it, refill it
      // with the warp's chunk two ahead
      __syncwarp();
      if (lane == 0 && seq + SPW < total && !*abort_flag) {
        tc::fence_proxy_async();
        fill_w(seq + SPW);
        fill_a(seq + SPW);
        nissued = seq + SPW + 1;
      }
    }
    // ---- the eight warps' K slices summed in warp order ----
    float *rw = red + (size_t)warp * (2 * NT * 4 * 32);
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) rw[((mt * NT + nt) * 4 + e) * 32 + lane] = NS == 2 ? acc[0][mt][nt][e] + acc[NS - 1][mt][nt][e] : acc[0][mt][nt][e];
    __syncthreads();
    const bool abort_now = *abort_flag != 0;
    for (int idx = threadIdx.x; idx < 2 * NT * 4 * 32; idx += GN_THREADS) {
      float v = 0.0f;
#pragma unroll
      for (int w = 0; w < GN_WARPS; ++w) v += red[(size_t)w * (2 * NT * 4 * 32) + idx];
      // idx = ((mt * NT + nt) * 4 + e) * 32 + lane'
      const int ln = idx & 31, e = (idx >> 5) & 3, mnt = idx >> 7;
      const int mt = mnt / NT, nt = mnt % NT;
      const int g2 = ln >> 2, t2 = ln & 3;
      const int col = tile * GN_TN + 4 * g2 + 2 * mt + (e >> 1); // e 0,1: row g; 2,3: row g + 8 (next column)
      const int m = nt * 8 + 2 * t2 + (e & 1);
      if (!abort_now && m < g.M && col < g.N) g.y[(int64_t)m * g.N + col] = __float2half_rn(v);
    }
    __syncthreads(); // red is reused by the next tile
  }
  // The CTA must not end with copies in flight into its shared memory: after
  // a give-up, wait (bounded) for the fills this warp issued.
  if (lane == 0 && *abort_flag)
    for (int s = nissued > SPW ? nissued - SPW : 0; s < nissued; ++s)
      tc::mbar_wait(&full[warp * SPW + s % SPW], (s / SPW) & 1, g.wait_ns);
}

struct GnPlan {
  int nt = 1, grid = 0, ntiles = 0, nchunks = 0, srows = 0, block = 0, arows = 0;
};

GnPlan gn_plan(const DqMmParams &p) {
  GnPlan m;
  m.nt = p.M <= 8 ? 1 : p.M <= 16 ? 2 : p.M <= 32 ? 4 : 8;
  m.ntiles = (int)((p.N + GN_TN - 1) / GN_TN);
  const int ch = m.nt == 1 ? GnCfg<1>::kCh : m.nt == 2 ? GnCfg<2>::kCh : m.nt == 4 ? GnCfg<4>::kCh : GnCfg<8>::kCh;
  m.nchunks = (int)((p.K + ch - 1) / ch);
  m.grid = std::min(m.ntiles, sm_count());
  m.arows = (int)std::min<int64_t>(p.M, 8 * m.nt);
  if (p.slayout == kScaleTensor) {
    m.srows = 0;
  } else if (p.slayout == kScaleAxis1) {
    m.srows = 1;
  } else {
    m.block = (int)p.block;
    m.srows = p.block < ch ? (int)(ch / p.block) : 1;
  }
  return m;
}

template <int NT> int launch_n(const DqMmParams &p, const GnPlan &m, cudaStream_t st) {
  CUtensorMap map_w, map_a, map_s;
  {
    const uint64_t dims[2] = {(uint64_t)p.N / 2, (uint64_t)p.K};
    const uint64_t strides[1] = {(uint64_t)p.N / 2};
    const uint32_t box[2] = {GN_TN / 2, (uint32_t)GnCfg<NT>::kCh};
    int rc = make_tensor_map(&map_w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, p.w, dims, strides, box,
                             CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
  }
  {
    const uint64_t dims[2] = {(uint64_t)p.K, (uint64_t)p.M};
    const uint64_t strides[1] = {(uint64_t)p.K * 2};
    const uint32_t box[2] = {64, (uint32_t)m.arows};
    int rc = make_tensor_map(&map_a, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, p.a, dims, strides, box,
                             CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  map_s = map_w;
  if (m.srows) {
    const uint64_t rows = p.slayout == kScaleAxis1 ? 1 : (uint64_t)p.s_alen;
    const uint64_t dims[2] = {(uint64_t)p.N, rows};
    const uint64_t strides[1] = {(uint64_t)p.N * 2};
    const uint32_t box[2] = {GN_TN, (uint32_t)m.srows};
    int rc = make_tensor_map(&map_s, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, p.scale, dims, strides,
                             box, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
  }
  GnArgs a{};
  a.y = static_cast<__half *>(p.y);
  a.M = (int)p.M;
  a.N = (int)p.N;
  a.K = (int)p.K;
  a.ntiles = m.ntiles;
  a.nchunks = m.nchunks;
  a.grid = m.grid;
  a.block = m.block;
  a.srows = m.srows;
  a.arows = m.arows;
  a.is_signed = p.wdt == kInt4;
  a.scalar_scale = reinterpret_cast<const uint16_t *>(p.scale);
  a.wait_ns = kWaitNs;
  auto kern = dq_gemv_n<NT>;
  const size_t smem = GnCfg<NT>::kDynamic;
  B2_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)m.grid);
  cfg.blockDim = dim3(GN_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  B2_CUDA(cudaLaunchKernelEx(&cfg, kern, map_w, map_a, map_s, a));
  return B2_OK;
}

} // namespace

bool dq_n_eligible(const DqMmParams &p) {
  if (p.wdt != kInt4 && p.wdt != kUint4) return false;
  if (!p.s_f16 || p.zp != nullptr || p.ydt != kFloat16) return false;
  if (p.cast_dt != 0 && p.cast_dt != kFloat16) return false;
  // N % 32: whole 16-byte packed row pieces per tile (TMA box and strides)
  if (p.M < 1 || p.M > GN_MAX_ROWS || p.N < 32 || p.N % 32 != 0 || p.K < 16 || p.K % 8 != 0) return false;
  if (p.N > (int64_t)1 << 30 || p.K > (int64_t)1 << 30) return false;
  switch (p.slayout) {
  case kScaleTensor:
  case kScaleAxis1: return true;
  case kScaleAxis0Block:
    // every k16 step inside one scale block; a chunk's scale rows are whole
    // (chunks of 256, 128 or 64 rows)
    if (p.block % 16 != 0) return false;
    return p.block <= GN_CH_MIN ? GN_CH_MIN % p.block == 0 : p.block % 256 == 0 || 256 % p.block == 0;
  default: return false;
  }
}

int dq_n_launch(const DqMmParams &p, cudaStream_t st) {
  const GnPlan m = gn_plan(p);
  if (m.nt == 1) return launch_n<1>(p, m, st);
  if (m.nt == 2) return launch_n<2>(p, m, st);
  if (m.nt == 4) return launch_n<4>(p, m, st);
  return launch_n<8>(p, m, st);
}

} // namespace b2
