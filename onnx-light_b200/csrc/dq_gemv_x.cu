// Decode-shaped fused DequantizeLinear -> [Cast] -> MatMul with the weight
// dequantized exactly as the reference does, for INT4 / UINT4 weights with
// FLOAT16 scales (no zero point) and FLOAT16 activations, M <= 64 rows: the
// int4 weight-only projection of LLM decoding at batch 1 to 64.
//
// Reference semantics (onnx_light/onnx_extensions/kernels/kernels/quantization/
// kernel_dequantizelinear.cc:332-520 then kernels/math/kernel_matmul.cc:181-223):
// w[k, n] = fp16(q[k, n] * s[k / block, n]) and y[m, n] = sum_k a[m, k] w[k, n]
// accumulated in fp32.  Here every weight is that same fp16 value: the packed
// code becomes the exact fp16 integer q (one logic operation and one fp16
// subtraction of the magic offset), and one fp16 multiplication by the scale
// rounds q * s to nearest even exactly as the reference's fp32 product
// followed by its fp16 conversion does (q * s is exact in fp32 and the two
// roundings coincide, subnormals included).  The products with the fp16
// activations are exact in the fp32 accumulators of mma.sync, so the result
// differs from the reference's only in the order of the fp32 sums.
//
// Why register MMA: the weight tile is dequantized once in registers and feeds
// the A operand of mma.sync m16n8k16 for every 8-row activation tile (NT of
// them) -- the dequantization cost is paid once per weight whatever the batch,
// and nothing of the expanded weight touches shared memory.  Each warp's
// k16 step: two transposing ldmatrix of the packed stage give every lane the
// 4 columns 32c + 4g .. +3 of rows 2t, 2t + 1 (and + 8) packed in one register;
// nibble j of each half is isolated (shift + logic), offset into the fp16
// integer 1024 + code, turned into q by one fp16 subtraction and into the
// weight by one fp16 multiplication with (s_col, s_col).
//
// Work split: as in dq_gemv_mma -- units of 128 weight rows x 256 columns
// (16 KB packed), numbered tile-major, equal contiguous unit ranges per CTA
// (stream-K), a tile shared by several CTAs merged by the last to arrive in
// CTA order.  Activation rows beyond 8 * NT take grid.y passes, CTA (b, p)
// covering rows 32p .. 32p + 31 of the same units as (b, 0), so the weights
// cross HBM once and L2 serves the other passes.
//
// Pipeline: eight warps, all consumers (warp w: column half w & 1, rows
// 32 (w >> 1) .. + 31 of every stage); thread 0 also loads: a ring of TMA
// stages (packed weights with the 128-byte swizzle, the activation slice, the
// scale rows), refilled once all eight warps are done with a slot.  The first
// fills' weights and scales are requested before the programmatic-launch wait
// (they do not depend on the kernel ahead), their activations after it.  With
// one activation tile (M <= 8) a CTA takes at most half an SM (96 KB of shared
// memory, <= 128 registers), so the next projection's CTAs can be resident and
// load their weights while this one finishes.
#include "dq_matmul.cuh"
#include "tc_common.cuh"

namespace b2 {

// Wait time-outs of the exact decode kernel (a TMA copy or a ring slot that
// never arrived); the kernel then skips its remaining work.
__device__ int g_gemv_x_status;

int status_read_gemv_x(int reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_gemv_x_status, sizeof(int)) != cudaSuccess) return -1;
  if (reset && v) {
    const int z = 0;
    if (cudaMemcpyToSymbol(g_gemv_x_status, &z, sizeof(int)) != cudaSuccess) return -1;
  }
  return v;
}

namespace {

constexpr int GX_TN = 256;                         // columns per tile (128 packed bytes / row)
constexpr int GX_TK = 128;                         // weight rows per stage
constexpr int GX_WARPS = 8;
constexpr int GX_THREADS = GX_WARPS * 32;
constexpr int GX_QUADS = 4;                        // warps per column half
constexpr uint32_t GX_W_BYTES = GX_TK * GX_TN / 2; // 16 KB
constexpr int GX_SC_ROWS = 4;                      // scale rows per stage at most (block 32)
constexpr uint32_t GX_SC_BYTES = GX_SC_ROWS * GX_TN * 2;

struct GxArgs {
  __half *y;
  float *partials;
  uint32_t *counters;
  int M, N, K;
  int ntiles, kunits, units, grid;
  int block;     // scale block along K (0: one scale row for all K)
  int srows;     // scale rows loaded per stage (0: per-tensor scale)
  const uint16_t *scalar_scale;
  int is_signed;
  uint64_t wait_ns;
};

// Ring depth and shared-memory layout per activation-tile count.
template <int NT> struct GxCfg {
  static constexpr int kStages = NT == 1 ? 4 : NT == 2 ? 8 : 6;
  static constexpr int kCtasPerSm = NT == 1 ? 2 : 1;
  static constexpr uint32_t kA = 2u * 8 * NT * 128; // two 64-column boxes, 8*NT rows each
  static constexpr uint32_t kOffA = kStages * GX_W_BYTES;
  static constexpr uint32_t kOffS = kOffA + kStages * kA;
  static constexpr uint32_t kOffRed = kOffS + kStages * GX_SC_BYTES;
  // GX_QUADS / 2 slots per column half for the tree reduction over its warps
  static constexpr uint32_t kRedBytes = (GX_QUADS / 2) * 2u * 32 * NT * 32 * 4;
  static constexpr uint32_t kOffBar = kOffRed + kRedBytes;
  static constexpr uint32_t kBytes = kOffBar + 2 * kStages * 8 + 16;
  static constexpr size_t kDynamic = kBytes + 1024; // alignment slack
};

__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void prefetch_l2_2d(const CUtensorMap *map, int32_t x, int32_t y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ uint32_t atom_add_acq_rel(uint32_t *p, uint32_t v) {
  uint32_t old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
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
// Two fp16 weights from two packed codes at bits 0..3 and 16..19 of `v`:
// (1024 + code') - magic = q exactly, then q * s rounded to nearest even.
__device__ __forceinline__ uint32_t dq2(uint32_t v, uint32_t magic, uint32_t s2) {
  uint32_t h = (v & 0x000f000fu) ^ magic, q, w;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(q) : "r"(h), "r"(magic));
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(w) : "r"(q), "r"(s2));
  return w;
}
__device__ __forceinline__ int unit_begin(int c, int U, int G) {
  return (int)((uint32_t)c * (uint32_t)U / (uint32_t)G); // units * grid < 2^31 (host check)
}
__device__ __forceinline__ int cta_of(int u, int U, int G) {
  return (int)(((uint32_t)(u + 1) * (uint32_t)G - 1u) / (uint32_t)U);
}
// Column (within the warp's 128-column half) of lane row g of m-tile mt;
// lane row g + 8 holds the next column.
__device__ __forceinline__ int mt_col(int mt, int g) { return (mt >> 1) * 32 + 4 * g + 2 * (mt & 1); }

template <int NT>
__global__ void __launch_bounds__(GX_THREADS, GxCfg<NT>::kCtasPerSm)
    dq_gemv_x(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_a,
              const __grid_constant__ CUtensorMap map_s, const GxArgs g) {
  using C = GxCfg<NT>;
  constexpr int S = C::kStages;
  extern __shared__ uint8_t dsm[];
  uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(dsm) + 1023) & ~uintptr_t(1023));
  uint64_t *full = reinterpret_cast<uint64_t *>(sm + C::kOffBar);
  uint64_t *empty = full + S;
  volatile int *flags = reinterpret_cast<volatile int *>(empty + S); // [0] abort, [1] last
  float *red = reinterpret_cast<float *>(sm + C::kOffRed);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.x, pass = blockIdx.y;
  const int u0 = unit_begin(b, g.units, g.grid);
  const int u1 = unit_begin(b + 1, g.units, g.grid);
  const int nun = u1 - u0;
  const int arow = pass * 8 * NT; // first activation row of this pass
  const bool loader = threadIdx.x == 0;

  if (loader) {
    for (int i = 0; i < S; ++i) {
      tc::mbar_init(&full[i], 1);
      tc::mbar_init(&empty[i], GX_WARPS);
    }
    flags[0] = 0;
    flags[1] = 0;
    tc::fence_barrier_init();
    tc::prefetch_tensormap(&map_w);
    tc::prefetch_tensormap(&map_a);
    if (g.srows) tc::prefetch_tensormap(&map_s);
    for (int u = u0; u < u1; ++u)
      prefetch_l2_2d(&map_w, (u / g.kunits) * (GX_TN / 2), (u % g.kunits) * GX_TK);
  }
  __syncthreads();
  const uint32_t tx = GX_W_BYTES + C::kA + (uint32_t)g.srows * GX_TN * 2;
  auto fill_w = [&](int i) { // weights + scales of fill i (constants of the call)
    const int s = i % S;
    const int u = u0 + i, tile = u / g.kunits, kb = u % g.kunits;
    tc::mbar_expect_tx(&full[s], tx);
    tc::tma_load_2d(sm + s * GX_W_BYTES, &map_w, &full[s], tile * (GX_TN / 2), kb * GX_TK);
    if (g.srows) {
      const int srow = g.block ? (kb * GX_TK) / g.block : 0;
      tc::tma_load_2d(sm + C::kOffS + s * GX_SC_BYTES, &map_s, &full[s], tile * GX_TN, srow);
    }
  };
  auto fill_a = [&](int i) { // activations of fill i (written by the kernel ahead)
    const int s = i % S;
    const int kb = (u0 + i) % g.kunits;
    uint8_t *sa = sm + C::kOffA + s * C::kA;
    tc::tma_load_2d(sa, &map_a, &full[s], kb * GX_TK, arow);
    tc::tma_load_2d(sa + C::kA / 2, &map_a, &full[s], kb * GX_TK + 64, arow);
  };
  const int pre = nun < S ? nun : S;
  if (loader)
    for (int i = 0; i < pre; ++i) fill_w(i);
  // Everything below may read what the previous kernel on the stream wrote
  // (activations) or write what it reads (output, workspace).
  griddep_wait();
  griddep_launch();
  if (loader)
    for (int i = 0; i < pre; ++i) fill_a(i);
  int issued = pre;

  const int wn = warp & 1, quad = warp >> 1;
  const int gq = lane >> 2, t = lane & 3;
  const uint32_t magic = g.is_signed ? 0x64086408u : 0x64006400u; // fp16 (1032, 1032) / (1024, 1024)
  uint32_t scalar2 = 0;
  if (!g.srows) {
    const uint32_t h = __ldg(g.scalar_scale);
    scalar2 = h | (h << 16);
  }
  float acc[8][NT][4];
#pragma unroll
  for (int mt = 0; mt < 8; ++mt)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[mt][nt][e] = 0.0f;
  bool ok = true;
  const int first_tile = u0 / g.kunits;
  const int slab_row0 = quad * 32;
  const int mi = lane >> 3;
  const int lrow = (mi & 1) * 8 + (lane & 7); // ldmatrix source row within a k16 step

  int seg0 = 0; // first stage of the current tile segment
  while (seg0 < nun) {
    const int tile = (u0 + seg0) / g.kunits;
    const int seg1 = min(nun, (tile + 1) * g.kunits - u0);
    for (int i = seg0; i < seg1; ++i) {
      const int s = i % S;
      const int kb = (u0 + i) % g.kunits;
      if (ok && flags[0]) ok = false;
      if (ok && !tc::mbar_wait(&full[s], (i / S) & 1, g.wait_ns)) {
        atomicExch(&g_gemv_x_status, tc::kTimeoutFull);
        flags[0] = 1;
        ok = false;
      }
      if (ok) {
        const uint8_t *wst = sm + s * GX_W_BYTES;
        const uint8_t *ast = sm + C::kOffA + s * C::kA;
        // (s_col, s_col) and (s_col+1, s_col+1) of this lane's 8 column pairs
        // for the slab's scale row (scale blocks are >= 32 rows: one per slab)
        uint32_t slo[8], shi[8];
        if (g.srows) {
          const int srow = (g.block && g.block < GX_TK) ? slab_row0 / g.block : 0;
          const uint8_t *sp = sm + C::kOffS + s * GX_SC_BYTES + srow * GX_TN * 2 + wn * 256;
#pragma unroll
          for (int mt = 0; mt < 8; ++mt) {
            const uint32_t w2 = *reinterpret_cast<const uint32_t *>(sp + mt_col(mt, gq) * 2);
            slo[mt] = __byte_perm(w2, w2, 0x1010);
            shi[mt] = __byte_perm(w2, w2, 0x3232);
          }
        } else {
#pragma unroll
          for (int mt = 0; mt < 8; ++mt) slo[mt] = shi[mt] = scalar2;
        }
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int r0 = slab_row0 + 16 * j;
          // activation fragments of the k16 step for every 8-row tile; rows
          // past K read as zeros in every operand (TMA fill)
          uint32_t B0[NT], B1[NT];
          {
            const int kb2 = ((r0 & 63) + 2 * t) * 2; // byte within the 64-column activation box
            const uint8_t *box = ast + (r0 >= 64 ? 8 * NT * 128 : 0);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              const int row = nt * 8 + gq;
              const uint8_t *rb = box + row * 128;
              B0[nt] = *reinterpret_cast<const uint32_t *>(rb + ((((kb2 >> 4) ^ (row & 7)) << 4) | (kb2 & 15)));
              const int kb3 = kb2 + 16;
              B1[nt] = *reinterpret_cast<const uint32_t *>(rb + ((((kb3 >> 4) ^ (row & 7)) << 4) | (kb3 & 15)));
            }
          }
          const int row = r0 + lrow;
          const uint32_t rbase = tc::smem_u32(wst + row * 128);
#pragma unroll
          for (int pair = 0; pair < 2; ++pair) {
            const int lch = wn * 4 + pair * 2 + (mi >> 1);
            uint32_t r[4];
            ldsm_t4(rbase + ((lch ^ (row & 7)) << 4), r);
#pragma unroll
            for (int c = 0; c < 2; ++c) {
              const uint32_t x = r[2 * c], y = r[2 * c + 1]; // k rows 2t.. and 2t+8..
              const int mt = (pair * 2 + c) * 2;
              {
                const uint32_t a0 = dq2(x, magic, slo[mt]), a1 = dq2(x >> 4, magic, shi[mt]);
                const uint32_t a2 = dq2(y, magic, slo[mt]), a3 = dq2(y >> 4, magic, shi[mt]);
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) mma16816(acc[mt][nt], a0, a1, a2, a3, B0[nt], B1[nt]);
              }
              {
                const uint32_t a0 = dq2(x >> 8, magic, slo[mt + 1]), a1 = dq2(x >> 12, magic, shi[mt + 1]);
                const uint32_t a2 = dq2(y >> 8, magic, slo[mt + 1]), a3 = dq2(y >> 12, magic, shi[mt + 1]);
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
                  mma16816(acc[mt + 1][nt], a0, a1, a2, a3, B0[nt], B1[nt]);
              }
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&empty[s]);
      // refill this slot with fill `issued` once every warp is done with it
      if (loader && issued < nun && issued == i + S && !flags[0]) {
        if (tc::mbar_wait(&empty[s], (i / S) & 1, g.wait_ns)) {
          fill_w(issued);
          fill_a(issued);
          ++issued;
        } else {
          atomicExch(&g_gemv_x_status, tc::kTimeoutEmpty);
          flags[0] = 1;
        }
      }
    }

    // ------------------------ end of a tile segment ------------------------
    // Sum the four warps of each column half (fixed-order tree); the warps of
    // quad 0 end with the column half's sums.
#pragma unroll
    for (int half = GX_QUADS / 2; half >= 1; half >>= 1) {
      __syncthreads();
      if (quad >= half && quad < 2 * half) {
        float *r = red + (size_t)((quad - half) * 2 + wn) * 32 * NT * 32;
#pragma unroll
        for (int mt = 0; mt < 8; ++mt)
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) r[((mt * NT + nt) * 4 + e) * 32 + lane] = acc[mt][nt][e];
      }
      __syncthreads();
      if (quad < half) {
        const float *r = red + (size_t)(quad * 2 + wn) * 32 * NT * 32;
#pragma unroll
        for (int mt = 0; mt < 8; ++mt)
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[mt][nt][e] += r[((mt * NT + nt) * 4 + e) * 32 + lane];
      }
    }
    const int uf = tile * g.kunits, ul = uf + g.kunits - 1;
    const int cf = cta_of(uf, g.units, g.grid), cl = cta_of(ul, g.units, g.grid);
    const int n0 = tile * GX_TN;
    if (cf == cl) {
      // The whole tile is this CTA's: write the output.
      if (quad == 0 && ok) {
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
          const int col = n0 + wn * 128 + mt_col(mt, gq);
          if (col >= g.N) continue; // ragged last tile (N % 256 != 0); N is even
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            const int m = arow + nt * 8 + 2 * t;
            if (m < g.M)
              *reinterpret_cast<__half2 *>(g.y + (int64_t)m * g.N + col) =
                  __floats2half2_rn(acc[mt][nt][0], acc[mt][nt][2]);
            if (m + 1 < g.M)
              *reinterpret_cast<__half2 *>(g.y + (int64_t)(m + 1) * g.N + col) =
                  __floats2half2_rn(acc[mt][nt][1], acc[mt][nt][3]);
          }
        }
      }
    } else {
      // partials [pass][cta][slot][8 NT rows][256 columns]
      const int slot = tile == first_tile ? 0 : 1;
      const size_t pstride = (size_t)8 * NT * GX_TN;
      float *pbase = g.partials + (size_t)pass * g.grid * 2 * pstride;
      float *part = pbase + (size_t)(b * 2 + slot) * pstride;
      if (quad == 0) {
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
          const int col = wn * 128 + mt_col(mt, gq);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            const int m = nt * 8 + 2 * t;
            *reinterpret_cast<float2 *>(part + m * GX_TN + col) = make_float2(acc[mt][nt][0], acc[mt][nt][2]);
            *reinterpret_cast<float2 *>(part + (m + 1) * GX_TN + col) =
                make_float2(acc[mt][nt][1], acc[mt][nt][3]);
          }
        }
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        // Release this CTA's partial (the barrier above orders the other
        // threads' stores before it), acquire the others' if last.  A CTA
        // whose wait gave up arrives with kAbortMark, and then the last one
        // does not merge (the partials are not all valid).
        uint32_t *ctr = g.counters + pass * g.ntiles + tile;
        const uint32_t inc = flags[0] ? kAbortMark + 1u : 1u;
        const uint32_t now = atom_add_acq_rel(ctr, inc) + inc;
        const bool last = (now & (kAbortMark - 1u)) == (uint32_t)(cl - cf + 1);
        if (last) *ctr = 0u;
        flags[1] = last && (now >> 16) == 0u ? 1 : 0;
      }
      __syncthreads();
      if (flags[1] && ok) {
        // Last to arrive: sum the contributors' partials in CTA order, with the
        // loads of up to 16 contributors in flight before the first add.
        const int nc = cl - cf + 1;
        const int rows = min(8 * NT, g.M - arow);
        for (int e = threadIdx.x; e < rows * (GX_TN / 4); e += GX_THREADS) {
          float4 sum = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
          for (int c0 = 0; c0 < nc; c0 += 16) {
            float4 v[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              v[j] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
              const int c = cf + c0 + j;
              if (c0 + j < nc) {
                const int cslot = unit_begin(c, g.units, g.grid) / g.kunits == tile ? 0 : 1;
                v[j] = __ldcg(reinterpret_cast<const float4 *>(pbase + (size_t)(c * 2 + cslot) * pstride) + e);
              }
            }
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              sum.x += v[j].x;
              sum.y += v[j].y;
              sum.z += v[j].z;
              sum.w += v[j].w;
            }
          }
          const int m = e / (GX_TN / 4), col = (e % (GX_TN / 4)) * 4;
          if (n0 + col >= g.N) continue; // ragged last tile; N % 4 == 0
          __half2 *dst = reinterpret_cast<__half2 *>(g.y + (int64_t)(arow + m) * g.N + n0 + col);
          dst[0] = __floats2half2_rn(sum.x, sum.y);
          dst[1] = __floats2half2_rn(sum.z, sum.w);
        }
      }
    }
#pragma unroll
    for (int mt = 0; mt < 8; ++mt)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[mt][nt][e] = 0.0f;
    seg0 = seg1;
  }
  // The CTA must not end with copies in flight into its shared memory: after
  // a give-up, wait (bounded) for the last fill of every slot issued.
  if (loader && flags[0])
    for (int i = issued > S ? issued - S : 0; i < issued; ++i)
      tc::mbar_wait(&full[i % S], (i / S) & 1, g.wait_ns);
}

struct GxPlan {
  int nt = 1, passes = 1, grid = 0, units = 0, kunits = 0, ntiles = 0, srows = 0, block = 0;
  size_t ws = 0;
};

GxPlan gx_plan(const DqMmParams &p) {
  GxPlan m;
  m.nt = p.M <= 8 ? 1 : p.M <= 16 ? 2 : 4;
  m.passes = (int)((p.M + 8 * m.nt - 1) / (8 * m.nt));
  m.ntiles = (int)((p.N + GX_TN - 1) / GX_TN); // the last tile may be ragged (TMA zero-fills)
  m.kunits = (int)((p.K + GX_TK - 1) / GX_TK);
  m.units = m.ntiles * m.kunits;
  m.grid = std::min(m.units, std::max(1, sm_count() / m.passes));
  if (p.slayout == kScaleTensor) {
    m.srows = 0;
  } else if (p.slayout == kScaleAxis1) {
    m.srows = 1;
  } else {
    m.block = (int)p.block;
    m.srows = p.block < GX_TK ? (int)(GX_TK / p.block) : 1;
  }
  bool split = false;
  for (int tile = 0; tile < m.ntiles && !split; ++tile) {
    const int uf = tile * m.kunits, ul = uf + m.kunits - 1;
    const int cf = (int)(((int64_t)(uf + 1) * m.grid - 1) / m.units);
    const int cl = (int)(((int64_t)(ul + 1) * m.grid - 1) / m.units);
    split = cf != cl;
  }
  // Arrival counters always (they start the workspace); partials when a tile is shared.
  m.ws = kCounterBytes + (split ? (size_t)m.passes * m.grid * 2 * 8 * m.nt * GX_TN * 4 : 0);
  return m;
}

template <int NT>
int launch_x(const DqMmParams &p, const GxPlan &m, void *workspace, cudaStream_t st) {
  CUtensorMap map_w, map_a, map_s;
  {
    const uint64_t dims[2] = {(uint64_t)p.N / 2, (uint64_t)p.K};
    const uint64_t strides[1] = {(uint64_t)p.N / 2};
    const uint32_t box[2] = {GX_TN / 2, GX_TK};
    int rc = make_tensor_map(&map_w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, p.w, dims, strides, box,
                             CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  {
    const uint64_t dims[2] = {(uint64_t)p.K, (uint64_t)p.M};
    const uint64_t strides[1] = {(uint64_t)p.K * 2};
    const uint32_t box[2] = {64, (uint32_t)(8 * NT)};
    int rc = make_tensor_map(&map_a, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, p.a, dims, strides, box,
                             CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  map_s = map_w;
  if (m.srows) {
    const uint64_t rows = p.slayout == kScaleAxis1 ? 1 : (uint64_t)p.s_alen;
    const uint64_t dims[2] = {(uint64_t)p.N, rows};
    const uint64_t strides[1] = {(uint64_t)p.N * 2};
    const uint32_t box[2] = {GX_TN, (uint32_t)m.srows};
    int rc = make_tensor_map(&map_s, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, p.scale, dims, strides,
                             box, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
  }
  GxArgs a{};
  a.y = static_cast<__half *>(p.y);
  a.counters = static_cast<uint32_t *>(workspace);
  a.partials = reinterpret_cast<float *>(static_cast<uint8_t *>(workspace) + kCounterBytes);
  a.M = (int)p.M;
  a.N = (int)p.N;
  a.K = (int)p.K;
  a.ntiles = m.ntiles;
  a.kunits = m.kunits;
  a.units = m.units;
  a.grid = m.grid;
  a.block = m.block;
  a.srows = m.srows;
  a.is_signed = p.wdt == kInt4;
  a.scalar_scale = reinterpret_cast<const uint16_t *>(p.scale);
  a.wait_ns = kWaitNs;
  auto kern = dq_gemv_x<NT>;
  const size_t smem = GxCfg<NT>::kDynamic;
  B2_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)m.grid, (unsigned)m.passes);
  cfg.blockDim = dim3(GX_THREADS);
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

bool dq_x_eligible(const DqMmParams &p) {
  if (p.wdt != kInt4 && p.wdt != kUint4) return false;
  if (!p.s_f16 || p.zp != nullptr || p.ydt != kFloat16) return false;
  if (p.cast_dt != 0 && p.cast_dt != kFloat16) return false;
  // N % 32: packed rows are whole 16-byte units (TMA strides); the last
  // 256-column tile may be partial.
  if (p.M < 1 || p.M > 64 || p.N < 32 || p.N % 32 != 0 || p.K < 16 || p.K % 8 != 0) return false;
  if (p.N > (int64_t)1 << 30 || p.K > (int64_t)1 << 30) return false;
  const int64_t ntiles = (p.N + GX_TN - 1) / GX_TN;
  const int64_t passes = (p.M + 31) / 32 > 1 ? (p.M + 31) / 32 : 1;
  if (ntiles * passes > (int64_t)kMaxCounters) return false;
  // unit numbers times the grid size stay below 2^31 (32-bit index arithmetic)
  const int64_t units = ntiles * ((p.K + GX_TK - 1) / GX_TK);
  if (units * (int64_t)(sm_count() + 1) >= ((int64_t)1 << 31)) return false;
  switch (p.slayout) {
  case kScaleTensor:
  case kScaleAxis1: return true;
  case kScaleAxis0Block:
    if (p.block % 32 != 0) return false;
    return p.block <= GX_TK ? GX_TK % p.block == 0 : p.block % GX_TK == 0;
  default: return false;
  }
}

size_t dq_x_workspace(const DqMmParams &p) { return gx_plan(p).ws; }

int dq_x_launch(const DqMmParams &p, void *workspace, cudaStream_t st) {
  const GxPlan m = gx_plan(p);
  if (m.ws && workspace == nullptr) B2_FAIL(B2_ERR_WORKSPACE, "workspace of %zu bytes required", m.ws);
  if (m.nt == 1) return launch_x<1>(p, m, workspace, st);
  if (m.nt == 2) return launch_x<2>(p, m, workspace, st);
  return launch_x<4>(p, m, workspace, st);
}

} // namespace b2
