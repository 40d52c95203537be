// Decode-shaped fused DequantizeLinear -> [Cast] -> MatMul with the weight
// dequantized exactly as the reference does (fp16(q * s), see dq_gemv_x.cu),
// INT4 / UINT4 weights with FLOAT16 scales (no zero point), FLOAT16
// activations and output, M <= 32 rows, split along K inside thread-block
// clusters.
//
// Reference semantics (onnx_light/onnx_extensions/kernels/kernels/quantization/
// kernel_dequantizelinear.cc:332-520 then kernels/math/kernel_matmul.cc:181-223).
//
// Why clusters.  A decode projection is latency-bound, and in a stream-K split
// (dq_gemv_mma, dq_gemv_x) most of a 4096 x 4096 launch's critical path is
// the cross-CTA merge: each CTA's partial goes to global memory, an
// acquire/release atomic counts arrivals, and the last arriver reads every
// partial back -- and a CTA whose unit range straddles two tiles pays that
// twice.  Here a tile (256 columns x all of K) belongs to one cluster of C
// CTAs (C <= 8, one K slice each, every CTA exactly one segment per tile), and
// the slices are summed through distributed shared memory: each CTA leaves its
// partial in its own shared memory, the cluster barrier publishes it, and CTA
// rank r sums columns [r 256/C, (r+1) 256/C) of all C partials in rank order
// (deterministic) and writes them.  No workspace, no global atomics.  Clusters
// take tiles round-robin when there are more tiles than clusters.
//
// Pipeline (as dq_gemv_x): eight warps, all consumers (warp w: column half
// w & 1, rows 32 (w >> 1) .. + 31 of every stage; the four warps of a half
// are summed by a fixed-order tree); thread 0 also streams the CTA's units
// (128 weight rows x 256 columns, 16 KB packed) through a TMA ring, weights
// and scales of the first fills before the programmatic-launch wait.  Every
// thread of the cluster passes the same cluster barriers in the same order
// (two per tile), also after a wait gave up, so no CTA is left waiting.
#include "dq_matmul.cuh"
#include "tc_common.cuh"

namespace b2 {

// Wait time-outs of the cluster decode kernel (a TMA copy or a ring slot that
// never arrived); the kernel then skips its remaining work.
__device__ int g_gemv_c_status;

int status_read_gemv_c(int reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_gemv_c_status, sizeof(int)) != cudaSuccess) return -1;
  if (reset && v) {
    const int z = 0;
    if (cudaMemcpyToSymbol(g_gemv_c_status, &z, sizeof(int)) != cudaSuccess) return -1;
  }
  return v;
}

namespace {

constexpr int GC_TN = 256;                         // columns per tile (128 packed bytes / row)
constexpr int GC_TK = 128;                         // weight rows per stage
constexpr int GC_WARPS = 8;
constexpr int GC_THREADS = GC_WARPS * 32;
constexpr int GC_QUADS = 4;                        // warps per column half
constexpr uint32_t GC_W_BYTES = GC_TK * GC_TN / 2; // 16 KB
constexpr int GC_SC_ROWS = 4;                      // scale rows per stage at most (block 32)
constexpr uint32_t GC_SC_BYTES = GC_SC_ROWS * GC_TN * 2;

struct GcArgs {
  __half *y;
  int M, N, K;
  int ntiles, kunits;
  int kper;      // units per cluster rank (K slice)
  int block;     // scale block along K (0: one scale row for all K)
  int srows;     // scale rows loaded per stage (0: per-tensor scale)
  const uint16_t *scalar_scale;
  int is_signed;
  uint64_t wait_ns;
};

// Ring depth and shared-memory layout per activation-tile count.
template <int NT> struct GcCfg {
  static constexpr int kStages = NT == 1 ? 4 : NT == 2 ? 7 : 4;
  static constexpr int kCtasPerSm = NT == 1 ? 2 : 1;
  static constexpr uint32_t kA = 2u * 8 * NT * 128; // two 64-column boxes, 8*NT rows each
  static constexpr uint32_t kOffA = kStages * GC_W_BYTES;
  static constexpr uint32_t kOffS = kOffA + kStages * kA;
  static constexpr uint32_t kOffRed = kOffS + kStages * GC_SC_BYTES;
  // GC_QUADS / 2 slots per column half for the tree reduction over its warps
  static constexpr uint32_t kRedBytes = (GC_QUADS / 2) * 2u * 32 * NT * 32 * 4;
  static constexpr uint32_t kOffX = kOffRed + kRedBytes;          // this CTA's partial [8 NT][256]
  static constexpr uint32_t kXBytes = 8u * NT * GC_TN * 4;
  static constexpr uint32_t kOffBar = kOffX + kXBytes;
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
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_id() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_count() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
// All threads of every CTA of the cluster; release / acquire orders the
// shared-memory partials written before it with the remote reads after it.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ float ld_cluster_f32(uint32_t local_addr, uint32_t rank) {
  uint32_t remote;
  float v;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local_addr), "r"(rank));
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
  return v;
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
// Column (within the warp's 128-column half) of lane row g of m-tile mt;
// lane row g + 8 holds the next column.
__device__ __forceinline__ int mt_col(int mt, int g) { return (mt >> 1) * 32 + 4 * g + 2 * (mt & 1); }

// One k16 step of the magic-number form (as dq_gemv_mma's k16_step): rows r0
// .. r0 + 15 of the stage, the 128 columns of column half `wn`, activation
// tile nt.  Nibbles 0 and 1 of each 16-bit half become the exact fp16
// integers 1024 + code and 1024 + 16 code with one logic operation, nibbles 2
// and 3 after a shift by 8; D accumulates sum a * magic, O sum a (ones row).
template <int NT>
__device__ __forceinline__ void k16_magic(const uint8_t *wst, const uint8_t *ast, int r0, int wn,
                                          int lane, int g, int t, int nt, uint32_t mlo, uint32_t mhi,
                                          float (&D)[8][4], float (&O)[4]) {
  uint32_t B0, B1;
  {
    const int kb = ((r0 & 63) + 2 * t) * 2;
    const uint8_t *box = ast + (r0 >= 64 ? 8 * NT * 128 : 0);
    const int row = nt * 8 + g;
    const uint8_t *rb = box + row * 128;
    B0 = *reinterpret_cast<const uint32_t *>(rb + ((((kb >> 4) ^ (row & 7)) << 4) | (kb & 15)));
    const int kb2 = kb + 16;
    B1 = *reinterpret_cast<const uint32_t *>(rb + ((((kb2 >> 4) ^ (row & 7)) << 4) | (kb2 & 15)));
  }
  const int mi = lane >> 3;
  const int row = r0 + (mi & 1) * 8 + (lane & 7);
  const uint32_t rbase = tc::smem_u32(wst + row * 128);
#pragma unroll
  for (int pair = 0; pair < 2; ++pair) {
    const int lch = wn * 4 + pair * 2 + (mi >> 1);
    uint32_t r[4];
    ldsm_t4(rbase + ((lch ^ (row & 7)) << 4), r);
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      const uint32_t x = r[2 * c], y = r[2 * c + 1];
      const int mt = (pair * 2 + c) * 2;
      mma16816(D[mt], (x & 0x000f000fu) ^ mlo, (x & 0x00f000f0u) ^ mhi, (y & 0x000f000fu) ^ mlo,
               (y & 0x00f000f0u) ^ mhi, B0, B1);
      const uint32_t xs = x >> 8, ys = y >> 8;
      mma16816(D[mt + 1], (xs & 0x000f000fu) ^ mlo, (xs & 0x00f000f0u) ^ mhi,
               (ys & 0x000f000fu) ^ mlo, (ys & 0x00f000f0u) ^ mhi, B0, B1);
    }
  }
  constexpr uint32_t kOnes = 0x3c003c00u; // (1.0, 1.0) in fp16
  mma16816(O, kOnes, kOnes, kOnes, kOnes, B0, B1);
}

// EXACT: weights formed as the reference's fp16 values (two fp16 operations
// per pair of weights); otherwise the cheaper magic-number form of
// dq_gemv_mma (one logic operation per pair, the scale applied to each
// 32-row block sum in fp32, within 2^-11 relative of the reference's weights).
template <int NT, int CL, bool EXACT>
__global__ void __launch_bounds__(GC_THREADS, GcCfg<NT>::kCtasPerSm)
    dq_gemv_c(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_a,
              const __grid_constant__ CUtensorMap map_s, const GcArgs g) {
  using C = GcCfg<NT>;
  constexpr int S = C::kStages;
  extern __shared__ uint8_t dsm[];
  uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(dsm) + 1023) & ~uintptr_t(1023));
  uint64_t *full = reinterpret_cast<uint64_t *>(sm + C::kOffBar);
  uint64_t *empty = full + S;
  volatile int *flags = reinterpret_cast<volatile int *>(empty + S); // [0] abort, [1] last
  float *red = reinterpret_cast<float *>(sm + C::kOffRed);
  float *xbuf = reinterpret_cast<float *>(sm + C::kOffX);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rank = (int)cluster_rank();
  const int cid = (int)cluster_id(), ncl = (int)cluster_count();
  // this CTA's K slice of every tile, and the tiles of its cluster
  const int kb0 = min(g.kunits, rank * g.kper), kb1 = min(g.kunits, kb0 + g.kper);
  const int nk = kb1 - kb0;
  const int ntile_mine = cid < g.ntiles ? (g.ntiles - cid + ncl - 1) / ncl : 0;
  const int nun = nk * ntile_mine;
  const bool loader = threadIdx.x == 0;

  if (loader) {
    for (int i = 0; i < S; ++i) {
      tc::mbar_init(&full[i], 1);
      tc::mbar_init(&empty[i], GC_WARPS);
    }
    flags[0] = 0;
    flags[1] = 0;
    tc::fence_barrier_init();
    tc::prefetch_tensormap(&map_w);
    tc::prefetch_tensormap(&map_a);
    if (g.srows) tc::prefetch_tensormap(&map_s);
    for (int i = 0; i < nun; ++i)
      prefetch_l2_2d(&map_w, (cid + ncl * (i / nk)) * (GC_TN / 2), (kb0 + i % nk) * GC_TK);
  }
  __syncthreads();
  const uint32_t tx = GC_W_BYTES + C::kA + (uint32_t)g.srows * GC_TN * 2;
  auto fill_w = [&](int i) { // weights + scales of fill i (constants of the call)
    const int s = i % S;
    const int tile = cid + ncl * (i / nk), kb = kb0 + i % nk;
    tc::mbar_expect_tx(&full[s], tx);
    tc::tma_load_2d(sm + s * GC_W_BYTES, &map_w, &full[s], tile * (GC_TN / 2), kb * GC_TK);
    if (g.srows) {
      const int srow = g.block ? (kb * GC_TK) / g.block : 0;
      tc::tma_load_2d(sm + C::kOffS + s * GC_SC_BYTES, &map_s, &full[s], tile * GC_TN, srow);
    }
  };
  auto fill_a = [&](int i) { // activations of fill i (written by the kernel ahead)
    const int s = i % S;
    const int kb = kb0 + i % nk;
    uint8_t *sa = sm + C::kOffA + s * C::kA;
    tc::tma_load_2d(sa, &map_a, &full[s], kb * GC_TK, 0);
    tc::tma_load_2d(sa + C::kA / 2, &map_a, &full[s], kb * GC_TK + 64, 0);
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
  const uint32_t mlo = magic;
  const uint32_t mhi = g.is_signed ? 0x64806480u : 0x64006400u;
  const float blo = g.is_signed ? 1032.0f : 1024.0f;
  const float bhi = g.is_signed ? 1152.0f : 1024.0f;
  uint32_t scalar2 = 0;
  float scalar = 0.0f;
  if (!g.srows) {
    const uint32_t h = __ldg(g.scalar_scale);
    scalar2 = h | (h << 16);
    scalar = __half2float(__ushort_as_half((uint16_t)h));
  }
  float acc[8][NT][4];
#pragma unroll
  for (int mt = 0; mt < 8; ++mt)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[mt][nt][e] = 0.0f;
  bool ok = true;
  const int slab_row0 = quad * 32;
  const int mi = lane >> 3;
  const int lrow = (mi & 1) * 8 + (lane & 7); // ldmatrix source row within a k16 step

  for (int it = 0; it < ntile_mine; ++it) {
    const int tile = cid + ncl * it;
    const int seg0 = it * nk, seg1 = seg0 + nk;
    for (int i = seg0; i < seg1; ++i) {
      const int s = i % S;
      if (ok && flags[0]) ok = false;
      if (ok && !tc::mbar_wait(&full[s], (i / S) & 1, g.wait_ns)) {
        atomicExch(&g_gemv_c_status, tc::kTimeoutFull);
        flags[0] = 1;
        ok = false;
      }
      if (ok && !EXACT) {
        const uint8_t *wst = sm + s * GC_W_BYTES;
        const uint8_t *ast = sm + C::kOffA + s * C::kA;
        const uint8_t *sst = sm + C::kOffS + s * GC_SC_BYTES;
        const int srow = (g.block && g.block < GC_TK) ? slab_row0 / g.block : 0;
        const uint8_t *srow_p = sst + srow * GC_TN * 2 + wn * 256;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          float D[8][4], O[4];
#pragma unroll
          for (int mt = 0; mt < 8; ++mt)
#pragma unroll
            for (int e = 0; e < 4; ++e) D[mt][e] = 0.0f;
#pragma unroll
          for (int e = 0; e < 4; ++e) O[e] = 0.0f;
#pragma unroll
          for (int j = 0; j < 2; ++j)
            k16_magic<NT>(wst, ast, slab_row0 + 16 * j, wn, lane, gq, t, nt, mlo, mhi, D, O);
          // block done: acc += s_eff * (D - bias * sum a), the high nibbles'
          // scale divided by 16
#pragma unroll
          for (int mt = 0; mt < 8; ++mt) {
            float se0 = scalar, se1 = scalar * 0.0625f;
            if (g.srows) {
              const uint32_t w2 = *reinterpret_cast<const uint32_t *>(srow_p + mt_col(mt, gq) * 2);
              se0 = __half2float(__ushort_as_half((uint16_t)(w2 & 0xffffu)));
              se1 = __half2float(__ushort_as_half((uint16_t)(w2 >> 16))) * 0.0625f;
            }
            const float c0 = fmaf(-blo, O[0], D[mt][0]), c1 = fmaf(-blo, O[1], D[mt][1]);
            const float c2 = fmaf(-bhi, O[0], D[mt][2]), c3 = fmaf(-bhi, O[1], D[mt][3]);
            acc[mt][nt][0] = fmaf(se0, c0, acc[mt][nt][0]);
            acc[mt][nt][1] = fmaf(se0, c1, acc[mt][nt][1]);
            acc[mt][nt][2] = fmaf(se1, c2, acc[mt][nt][2]);
            acc[mt][nt][3] = fmaf(se1, c3, acc[mt][nt][3]);
          }
        }
      }
      if (ok && EXACT) {
        const uint8_t *wst = sm + s * GC_W_BYTES;
        const uint8_t *ast = sm + C::kOffA + s * C::kA;
        // (s_col, s_col) and (s_col+1, s_col+1) of this lane's 8 column pairs
        // for the slab's scale row (scale blocks are >= 32 rows: one per slab)
        uint32_t slo[8], shi[8];
        if (g.srows) {
          const int srow = (g.block && g.block < GC_TK) ? slab_row0 / g.block : 0;
          const uint8_t *sp = sm + C::kOffS + s * GC_SC_BYTES + srow * GC_TN * 2 + wn * 256;
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
          atomicExch(&g_gemv_c_status, tc::kTimeoutEmpty);
          flags[0] = 1;
        }
      }
    }

    // ------------------------ end of a tile segment ------------------------
    // Sum the four warps of each column half (fixed-order tree); the warps of
    // quad 0 end with the column half's sums.
#pragma unroll
    for (int half = GC_QUADS / 2; half >= 1; half >>= 1) {
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
    // This CTA's partial of the tile into its own shared memory, [row][256].
    if (quad == 0) {
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        const int col = wn * 128 + mt_col(mt, gq);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const int m = nt * 8 + 2 * t;
          *reinterpret_cast<float2 *>(xbuf + m * GC_TN + col) = make_float2(acc[mt][nt][0], acc[mt][nt][2]);
          *reinterpret_cast<float2 *>(xbuf + (m + 1) * GC_TN + col) = make_float2(acc[mt][nt][1], acc[mt][nt][3]);
        }
      }
    }
    cluster_sync(); // every rank's partial is visible cluster-wide
    {
      // rank r sums columns [r W, (r + 1) W) over the cluster, in rank order
      constexpr int W = GC_TN / CL;
      const bool abort_now = flags[0] != 0;
      const int rows = min(8 * NT, g.M);
      const int n0 = tile * GC_TN + rank * W;
      const uint32_t xl = tc::smem_u32(xbuf);
      for (int e = threadIdx.x; e < rows * W; e += GC_THREADS) {
        const int m = e / W, c = e % W;
        const uint32_t a = xl + (uint32_t)(m * GC_TN + rank * W + c) * 4u;
        float v = 0.0f;
#pragma unroll
        for (int r = 0; r < CL; ++r) v += ld_cluster_f32(a, (uint32_t)r);
        if (!abort_now && n0 + c < g.N) g.y[(int64_t)m * g.N + n0 + c] = __float2half_rn(v);
      }
    }
    cluster_sync(); // the partials may be overwritten (next tile) or freed (exit)
#pragma unroll
    for (int mt = 0; mt < 8; ++mt)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[mt][nt][e] = 0.0f;
  }
  // The CTA must not end with copies in flight into its shared memory: after
  // a give-up, wait (bounded) for the last fill of every slot issued.
  if (loader && flags[0])
    for (int i = issued > S ? issued - S : 0; i < issued; ++i)
      tc::mbar_wait(&full[i % S], (i / S) & 1, g.wait_ns);
}

struct GcPlan {
  int nt = 1, cl = 8, nclusters = 0, kunits = 0, ntiles = 0, kper = 0, srows = 0, block = 0;
};


// Clusters of CL CTAs that can be resident at once for this kernel (host
// query, cached per instance).
template <int NT, int CL, bool EXACT> int max_clusters() {
  static int cached = -1;
  if (cached >= 0) return cached;
  auto kern = dq_gemv_c<NT, CL, EXACT>;
  const size_t smem = GcCfg<NT>::kDynamic;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess ||
      cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 0) != cudaSuccess)
    return 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(CL * 64);
  cfg.blockDim = dim3(GC_THREADS);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = CL;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) n = 0;
  cached = n;
  return n;
}

template <int NT> int max_clusters_of(int cl) {
  // both forms have the same shared memory and launch bounds
  switch (cl) {
  case 1: return max_clusters<NT, 1, false>();
  case 2: return max_clusters<NT, 2, false>();
  case 4: return max_clusters<NT, 4, false>();
  default: return max_clusters<NT, 8, false>();
  }
}

GcPlan gc_plan(const DqMmParams &p) {
  GcPlan m;
  m.nt = p.M <= 8 ? 1 : p.M <= 16 ? 2 : 4;
  m.ntiles = (int)((p.N + GC_TN - 1) / GC_TN); // the last tile may be ragged (TMA zero-fills)
  m.kunits = (int)((p.K + GC_TK - 1) / GC_TK);
  // K slices per tile: 8, fewer when K has fewer 128-row units
  m.cl = m.kunits >= 8 ? 8 : m.kunits >= 4 ? 4 : m.kunits >= 2 ? 2 : 1;
  m.kper = (m.kunits + m.cl - 1) / m.cl;
  const int resident = m.nt == 1 ? max_clusters_of<1>(m.cl) : m.nt == 2 ? max_clusters_of<2>(m.cl)
                                                                        : max_clusters_of<4>(m.cl);
  m.nclusters = std::max(1, std::min(m.ntiles, resident));
  if (p.slayout == kScaleTensor) {
    m.srows = 0;
  } else if (p.slayout == kScaleAxis1) {
    m.srows = 1;
  } else {
    m.block = (int)p.block;
    m.srows = p.block < GC_TK ? (int)(GC_TK / p.block) : 1;
  }
  return m;
}

template <int NT, int CL, bool EXACT> int launch_c_t(const DqMmParams &p, const GcPlan &m, cudaStream_t st) {
  CUtensorMap map_w, map_a, map_s;
  {
    const uint64_t dims[2] = {(uint64_t)p.N / 2, (uint64_t)p.K};
    const uint64_t strides[1] = {(uint64_t)p.N / 2};
    const uint32_t box[2] = {GC_TN / 2, GC_TK};
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
    const uint32_t box[2] = {GC_TN, (uint32_t)m.srows};
    int rc = make_tensor_map(&map_s, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, p.scale, dims, strides,
                             box, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
  }
  GcArgs a{};
  a.y = static_cast<__half *>(p.y);
  a.M = (int)p.M;
  a.N = (int)p.N;
  a.K = (int)p.K;
  a.ntiles = m.ntiles;
  a.kunits = m.kunits;
  a.kper = m.kper;
  a.block = m.block;
  a.srows = m.srows;
  a.is_signed = p.wdt == kInt4;
  a.scalar_scale = reinterpret_cast<const uint16_t *>(p.scale);
  a.wait_ns = kWaitNs;
  auto kern = dq_gemv_c<NT, CL, EXACT>;
  const size_t smem = GcCfg<NT>::kDynamic;
  B2_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(m.nclusters * CL));
  cfg.blockDim = dim3(GC_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = CL;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  B2_CUDA(cudaLaunchKernelEx(&cfg, kern, map_w, map_a, map_s, a));
  return B2_OK;
}

template <int NT, bool EXACT> int launch_c(const DqMmParams &p, const GcPlan &m, cudaStream_t st) {
  switch (m.cl) {
  case 1: return launch_c_t<NT, 1, EXACT>(p, m, st);
  case 2: return launch_c_t<NT, 2, EXACT>(p, m, st);
  case 4: return launch_c_t<NT, 4, EXACT>(p, m, st);
  default: return launch_c_t<NT, 8, EXACT>(p, m, st);
  }
}

} // namespace

bool dq_c_eligible(const DqMmParams &p) {
  if (p.wdt != kInt4 && p.wdt != kUint4) return false;
  if (!p.s_f16 || p.zp != nullptr || p.ydt != kFloat16) return false;
  if (p.cast_dt != 0 && p.cast_dt != kFloat16) return false;
  // N % 32: packed rows are whole 16-byte units (TMA strides); the last
  // 256-column tile may be partial.
  if (p.M < 1 || p.M > 32 || p.N < 32 || p.N % 32 != 0 || p.K < 16 || p.K % 8 != 0) return false;
  if (p.N > (int64_t)1 << 30 || p.K > (int64_t)1 << 30) return false;
  switch (p.slayout) {
  case kScaleTensor:
  case kScaleAxis1: return true;
  case kScaleAxis0Block:
    if (p.block % 32 != 0) return false;
    return p.block <= GC_TK ? GC_TK % p.block == 0 : p.block % GC_TK == 0;
  default: return false;
  }
}

int dq_c_launch(const DqMmParams &p, cudaStream_t st, bool exact) {
  const GcPlan m = gc_plan(p);
  if (exact) {
    if (m.nt == 1) return launch_c<1, true>(p, m, st);
    if (m.nt == 2) return launch_c<2, true>(p, m, st);
    return launch_c<4, true>(p, m, st);
  }
  if (m.nt == 1) return launch_c<1, false>(p, m, st);
  if (m.nt == 2) return launch_c<2, false>(p, m, st);
  return launch_c<4, false>(p, m, st);
}

} // namespace b2
