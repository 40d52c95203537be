// Decode-shaped fused DequantizeLinear -> [Cast] -> MatMul (M <= 16 rows of
// activations), INT4/UINT4 weights with FLOAT16 scales and FLOAT16
// activations: the int4 weight-only projection of LLM decoding.
//
// Reference semantics (onnx_light/onnx_extensions/kernels/kernels/quantization/
// kernel_dequantizelinear.cc:332-520 then kernels/math/kernel_matmul.cc:181-223):
// y[m, n] = sum_k a[m, k] * w[k, n] with w[k, n] = (q[k, n] - 0) * s[k / block, n]
// and fp32 accumulation.
//
// Arithmetic.  Each packed nibble is turned into an fp16 "magic number" with one
// logic operation per pair of weights: 1024 + (q + 8) for the low nibble of a
// byte and 1024 + 16 (q + 8) for the high one (signed; unsigned codes drop the
// + 8).  These exact fp16 integers go straight into mma.sync m16n8k16 (fp16
// inputs, fp32 accumulators) against the activations, together with one
// all-ones row that yields sum_k a[m, k] of the same k range.  At the end of
// every scale block the offset is removed and the scale applied in fp32:
//   sum_k a q s = s * (D - bias * sum_k a)            (low nibbles, bias 1032)
//   sum_k a q s = (s / 16) * (D - bias * sum_k a)     (high nibbles, bias 1152)
// so the weight is never rounded to fp16: the result differs from the
// reference's only by the reference's own fp16 rounding of each dequantized
// weight (at most 2^-11 relative per weight), and by the order of the fp32
// sums.  The fp32 cancellation of the offset costs about 2^-24 * 1152 / |q|
// relative per block sum (about 1e-5), far inside the rel-L2 1e-3 contract.
//
// Why register-level MMA and not tcgen05 here: the kernel is bound by HBM
// (half a byte per weight) and by the instructions spent per weight.  tcgen05
// takes its operands from shared memory or tensor memory, so every expanded
// weight would cost 2 bytes of shared-memory writes and reads per 0.5 byte
// fetched; built in registers, the fragment feeds the MMA directly and shared
// memory carries the packed weights once.  Large M goes to the tcgen05 kernel
// (dq_gemm_tc.cu).
//
// Work split ("stream-K"): the weight is cut into units of 128 rows x 256
// columns (16 KB packed, one pipeline stage), numbered tile-major (tile = 256
// columns); the grid's CTAs take equal contiguous ranges of units,
// so every SM streams the same number of bytes whatever the shape.  A tile
// covered by one CTA is written directly; a tile shared by several CTAs is
// finished by the last one to arrive, which sums the fp32 partials in CTA
// order (deterministic).
//
// Pipeline: one producer warp fills a 4-stage ring with TMA (packed weights
// 128 x 128 bytes with the 128-byte swizzle, the activation slice 128 x M in
// two swizzled boxes, the stage's scale rows).  Four consumer warps, two per
// 128-column half, take every stage together (64 rows each) or, with more
// stages per CTA, form two groups of two that take alternate whole stages.
// A CTA holds about 90 KB of shared memory and 160 threads, so two fit on an
// SM, and a launch of two or more units per SM runs two per SM: their rings
// keep 8 stages per SM in flight, and as CTAs finish, the CTAs of the next
// launch on the stream take their slots (programmatic dependent launch) and
// load their first weights while this launch ends.  Before
// waiting on the kernel launched ahead of it (programmatic dependent launch),
// each CTA asks the TMA unit to prefetch its whole weight range into L2: the
// prefetch changes no value (L2 is the point of coherence), so it is safe
// whatever the earlier kernel writes, and it lets consecutive projections
// stream HBM back to back.
#include "dq_matmul.cuh"
#include "tc_common.cuh"

#include <cstdlib>
#include <cstring>

namespace b2 {

// Wait time-outs of the decode kernel (a TMA copy or a consumer that never
// arrived) are recorded here; the kernel then skips its remaining work.
__device__ int g_gemv_mma_status;

namespace {

constexpr int kPeerMax = 8;
// Projections of one launch that share the activations.  The kernel is
// instantiated per count NP so that its parameters (NP weight and scale
// tensor maps, NP output descriptions) stay as small as the call needs: the
// launch of a 4096 x 4096 decode projection measured 6.9 us with one slot
// and 7.4 us with four (about 0.15 us per 400 bytes of parameters).
constexpr int kGroupMax = 4;
constexpr int GM_TN = 256;                         // columns per tile (128 packed bytes / row)
constexpr int GM_TK = 128;                         // weight rows per stage
#ifndef GM_RING
#define GM_RING 4
#endif
#ifndef GM_CTAS_PER_SM
#define GM_CTAS_PER_SM 2
#endif
constexpr int GM_STAGES = GM_RING;                 // ring depth
#ifndef GM_QUADS_N
#define GM_QUADS_N 2
#endif
constexpr int GM_QUADS = GM_QUADS_N;               // consumer warps per column half
constexpr int GM_CONSUMERS = 2 * GM_QUADS;         // consumer warps
constexpr int GM_THREADS = (GM_CONSUMERS + 1) * 32;
constexpr uint32_t GM_W_BYTES = GM_TK * GM_TN / 2; // 16 KB
constexpr int GM_SC_ROWS = 4;                      // scale rows per stage at most (block 32)
constexpr uint32_t GM_SC_BYTES = GM_SC_ROWS * GM_TN * 2;
constexpr uint32_t GM_ONES = 0x3c003c00u;          // (1.0, 1.0) in fp16
#ifndef GM_GROUPS_THRESHOLD
#define GM_GROUPS_THRESHOLD 2
#endif
constexpr int kGroupsThreshold = GM_GROUPS_THRESHOLD; // stages per CTA up to which G = 1

// The weight and scale tensor maps of each projection of the launch.
template <int NP> struct GmMaps {
  CUtensorMap w[NP];
  CUtensorMap s[NP];
};

template <int NP> struct GmArgs {
  float *partials;
  uint32_t *counters;
  int M, K;
  // Projections of the launch (NP >= 1; all read the same activations, K,
  // weight type and scale layout): projection p owns the 256-column tiles
  // tile_end[p - 1] .. tile_end[p] - 1 of the launch's tile numbering, has
  // Np[p] columns and writes y[p] (row stride ldy[p]).
  int tile_end[NP];
  int Np[NP];
  __half *y[NP];
  int ntiles, kunits, units, grid;
  int block;     // scale block along K (0: one scale row for all K)
  int srows;     // scale rows loaded per stage (0: per-tensor scale)
  const uint16_t *scalar_scale; // the per-tensor scale (srows == 0)
  int is_signed;
  // Tile-aligned split (aligned != 0): tiles 0 .. cr-1 get cq + 1 CTAs, the
  // others cq; each CTA one contiguous K slice of one tile.
  int aligned, cq, cr;
  uint64_t wait_ns;
  // Column-sharded output over a multi-GPU group (world > 1): every output
  // value goes to each rank's full [M, ldy] buffer at column col_off + n, and
  // the call first waits until every rank has finished the group's previous
  // call, then publishes its own completion (a generation number) in every
  // rank's flag array.
  int world, rank;
  int64_t ldy[NP], col_off[NP];
  __half *peer_y[NP][kPeerMax];
  uint32_t *peer_flags[kPeerMax];
  uint32_t *pctr; // this rank's [0] CTA arrivals, [1] generation
  int wait_input; // wait for every rank's previous call before reading a
};

template <int NT> struct GmSmem {
  static constexpr uint32_t kA = 2u * 8 * NT * 128; // two 64-column boxes, 8*NT rows each
  static constexpr uint32_t kOffA = GM_STAGES * GM_W_BYTES;
  static constexpr uint32_t kOffS = kOffA + GM_STAGES * kA;
  static constexpr uint32_t kOffRed = kOffS + GM_STAGES * GM_SC_BYTES;
  // GM_QUADS - 1 slots per column half for the sum over its warp groups
  static constexpr uint32_t kRedBytes = (GM_QUADS - 1) * 2u * 32 * NT * 32 * 4;
  static constexpr uint32_t kOffBar = kOffRed + kRedBytes;
  static constexpr uint32_t kBytes = kOffBar + 2 * GM_STAGES * 8 + 16;
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
__device__ __forceinline__ void consumers_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(GM_CONSUMERS * 32) : "memory");
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
// d = a * b + c on two fp32 lanes (one packed instruction on sm_100).
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  uint64_t d;
  asm("{\n\t.reg .b64 ra, rb, rc;\n\t"
      "mov.b64 ra, {%1, %2};\n\tmov.b64 rb, {%3, %4};\n\tmov.b64 rc, {%5, %6};\n\t"
      "fma.rn.f32x2 %0, ra, rb, rc;\n\t}"
      : "=l"(d)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(d));
  return r;
}
__device__ __forceinline__ int unit_begin(int c, int U, int G) {
  return (int)((uint32_t)c * (uint32_t)U / (uint32_t)G); // units * grid < 2^31 (host check)
}
__device__ __forceinline__ int cta_of(int u, int U, int G) {
  return (int)(((uint32_t)(u + 1) * (uint32_t)G - 1u) / (uint32_t)U);
}
// Tile-aligned split: CTA b -> (tile, K slice, slices of the tile, the tile's
// first CTA).  Tiles 0 .. cr-1 have cq + 1 consecutive CTAs, the rest cq.
__device__ __forceinline__ void tile_slice(int b, int cq, int cr, int &tile, int &slice, int &nsl,
                                           int &first) {
  const int big = cr * (cq + 1);
  if (b < big) {
    tile = b / (cq + 1);
    slice = b % (cq + 1);
    nsl = cq + 1;
    first = tile * (cq + 1);
  } else {
    const int bb = b - big;
    tile = cr + bb / cq;
    slice = bb % cq;
    nsl = cq;
    first = big + (tile - cr) * cq;
  }
}
__device__ __forceinline__ void red_release_add(uint32_t *p, uint32_t v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Projection of a launch tile, and its first tile.
template <int NP> __device__ __forceinline__ int prob_of(const GmArgs<NP> &g, int tile) {
  int p = 0;
#pragma unroll
  for (int i = 0; i < NP - 1; ++i) p += tile >= g.tile_end[i] ? 1 : 0;
  return p;
}
template <int NP> __device__ __forceinline__ int prob_first_tile(const GmArgs<NP> &g, int p) {
  return p ? g.tile_end[p - 1] : 0;
}
// Two output values (columns col, col + 1 of row m of projection p) to its y,
// or to every rank's full buffer when the output is column-sharded.
template <int NP>
__device__ __forceinline__ void store_h2(const GmArgs<NP> &g, int p, int64_t m, int64_t col, __half2 v) {
  if (g.world <= 1) {
    *reinterpret_cast<__half2 *>(g.y[p] + m * g.ldy[p] + col) = v;
    return;
  }
#pragma unroll
  for (int r = 0; r < kPeerMax; ++r)
    if (r < g.world)
      *reinterpret_cast<__half2 *>(g.peer_y[p][r] + m * g.ldy[p] + g.col_off[p] + col) = v;
}
__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Column (within the warp's 128-column half) of lane row g of m-tile mt;
// lane row g + 8 holds the next column.  m-tile mt = 2 * chunk + h covers
// columns 32 * chunk + 4 g + 2 h and + 1 for g = 0..7.
__device__ __forceinline__ int mt_col(int mt, int g) { return (mt >> 1) * 32 + 4 * g + 2 * (mt & 1); }

__device__ __forceinline__ void ldsm_t4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// One k16 step of one consumer warp: rows r0 .. r0+15 of the stage, the 128
// columns (four 16-byte chunks) of column half `wn`.  A transposing ldmatrix
// of 16-bit elements hands lane (g, t) the 4 columns 32c + 4g .. +3 of rows
// r0 + 2t and r0 + 2t + 1 (row block 0) or + 8 (row block 1) packed in one
// register, low half the first row -- the row pair an MMA A register holds.
// Nibbles 0 and 1 of each half become exact fp16 magic numbers with one logic
// operation each (1024 + code, 1024 + 16 code); nibbles 2 and 3 after a shift
// by 8.  D accumulates sum a * magic and O sum a (ones row) for activation
// rows nt*8 .. nt*8+7.
template <int NT>
__device__ __forceinline__ void k16_step(const uint8_t *wst, const uint8_t *ast, int r0, int wn,
                                         int lane, int g, int t, int nt, uint32_t mlo,
                                         uint32_t mhi, float (&D)[8][4], float (&O)[4]) {
  uint32_t B0, B1;
  {
    const int kb = ((r0 & 63) + 2 * t) * 2; // byte within the 64-column activation box
    const uint8_t *box = ast + (r0 >= 64 ? 8 * NT * 128 : 0);
    const int row = nt * 8 + g;
    const uint8_t *rb = box + row * 128;
    B0 = *reinterpret_cast<const uint32_t *>(rb + ((((kb >> 4) ^ (row & 7)) << 4) | (kb & 15)));
    const int kb2 = kb + 16;
    B1 = *reinterpret_cast<const uint32_t *>(rb + ((((kb2 >> 4) ^ (row & 7)) << 4) | (kb2 & 15)));
  }
  // ldmatrix source rows: lanes 8i .. 8i+7 address matrix i = (row block
  // i & 1, chunk i >> 1 of the pair); 128-byte swizzle of the TMA box.
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
      const uint32_t x = r[2 * c], y = r[2 * c + 1]; // row blocks 0 and 1
      const int mt = (pair * 2 + c) * 2;
      mma16816(D[mt], (x & 0x000f000fu) ^ mlo, (x & 0x00f000f0u) ^ mhi, (y & 0x000f000fu) ^ mlo,
               (y & 0x00f000f0u) ^ mhi, B0, B1);
      const uint32_t xs = x >> 8, ys = y >> 8;
      mma16816(D[mt + 1], (xs & 0x000f000fu) ^ mlo, (xs & 0x00f000f0u) ^ mhi,
               (ys & 0x000f000fu) ^ mlo, (ys & 0x00f000f0u) ^ mhi, B0, B1);
    }
  }
  mma16816(O, GM_ONES, GM_ONES, GM_ONES, GM_ONES, B0, B1);
}

// G = stage groups: the four warps of a column half split into G groups that
// take stages i with i % G == group, each stage's 128 rows cut into 4 / G slabs
// (G = 1: all eight warps on every stage, 32 rows each -- lowest latency per
// stage; G = 4: one warp pair per stage, 128 rows -- fewest epilogues).
// KS = k16 steps per scale block inside a slab (the slab's rows / 16 when the
// block is at least a slab), fixed at compile time so the steps unroll.
template <int NT, int G, int KS, int NP>
__global__ void __launch_bounds__(GM_THREADS, GM_CTAS_PER_SM)
    dq_gemv_mma(const __grid_constant__ GmMaps<NP> maps, const __grid_constant__ CUtensorMap map_a,
                const __grid_constant__ GmArgs<NP> g) {
  using L = GmSmem<NT>;
  extern __shared__ uint8_t dsm[];
  uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(dsm) + 1023) & ~uintptr_t(1023));
  uint64_t *full = reinterpret_cast<uint64_t *>(sm + L::kOffBar);
  uint64_t *empty = full + GM_STAGES;
  // [0] abort, [1] last
  volatile int *flags = reinterpret_cast<volatile int *>(empty + GM_STAGES);
  float *red = reinterpret_cast<float *>(sm + L::kOffRed);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.x;
  int u0, u1;
  int a_tile = 0, a_slice = 0, a_nsl = 1, a_first = 0; // tile-aligned split
  if (g.aligned) {
    tile_slice(b, g.cq, g.cr, a_tile, a_slice, a_nsl, a_first);
    u0 = a_tile * g.kunits + a_slice * g.kunits / a_nsl;
    u1 = a_tile * g.kunits + (a_slice + 1) * g.kunits / a_nsl;
  } else {
    u0 = unit_begin(b, g.units, g.grid);
    u1 = unit_begin(b + 1, g.units, g.grid);
  }
  const int nun = u1 - u0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < GM_STAGES; ++i) {
      tc::mbar_init(&full[i], 1);
      tc::mbar_init(&empty[i], 2 * (GM_QUADS / G)); // the warps that consume a stage
    }
    flags[0] = 0;
    flags[1] = 0;
    tc::fence_barrier_init();
  }
  if (warp == GM_CONSUMERS && lane == 0) {
    for (int q = 0; q < NP; ++q) {
      tc::prefetch_tensormap(&maps.w[q]);
      if (g.srows) tc::prefetch_tensormap(&maps.s[q]);
    }
    tc::prefetch_tensormap(&map_a);
    for (int u = u0; u < u1; ++u) {
      const int tile = u / g.kunits, q = prob_of(g, tile);
      prefetch_l2_2d(&maps.w[q], (tile - prob_first_tile(g, q)) * (GM_TN / 2), (u % g.kunits) * GM_TK);
    }
  }
  __syncthreads();
  // The weights and scales are constants of the call, independent of the
  // kernel launched ahead of this one: the first ring fill of each stage
  // (weights + scales) is issued before waiting for that kernel, and only the
  // activation boxes of those stages wait.  The stage's full barrier expects
  // all three, so consumers see a stage only when its activations are in.
  const uint32_t tx = GM_W_BYTES + L::kA + (uint32_t)g.srows * GM_TN * 2;
  const int pre = nun < GM_STAGES ? nun : GM_STAGES;
  auto load_weights = [&](int i) {
    const int s = i % GM_STAGES;
    const int u = u0 + i, tile = u / g.kunits, kb = u % g.kunits;
    const int q = prob_of(g, tile), lt = tile - prob_first_tile(g, q);
    tc::mbar_expect_tx(&full[s], tx);
    tc::tma_load_2d(sm + s * GM_W_BYTES, &maps.w[q], &full[s], lt * (GM_TN / 2), kb * GM_TK);
    if (g.srows) {
      const int srow = g.block ? (kb * GM_TK) / g.block : 0;
      tc::tma_load_2d(sm + L::kOffS + s * GM_SC_BYTES, &maps.s[q], &full[s], lt * GM_TN, srow);
    }
  };
  if (warp == GM_CONSUMERS && lane == 0)
    for (int i = 0; i < pre; ++i) load_weights(i);
  // Everything below may read what the previous kernel on the stream wrote
  // (activations) or write what it reads (output, workspace).
  griddep_wait();
  griddep_launch();
  if (g.world > 1 && g.wait_input) {
    // Column-sharded: the activations are a previous sharded call's output,
    // which other ranks store into this rank's buffer.  Wait (bounded) until
    // every rank has published this rank's current generation.
    if (threadIdx.x == 0) {
      const uint32_t gen = *(volatile uint32_t *)(g.pctr + 1); // calls this rank completed
      const uint32_t *mine = g.peer_flags[g.rank];
      const uint64_t t0 = tc::globaltimer();
      for (int r = 0; r < g.world && !flags[0]; ++r)
        while ((int32_t)(ld_acquire_sys(mine + r) - gen) < 0) {
          if (tc::globaltimer() - t0 > 5000000000ull) {
            atomicExch(&g_gemv_mma_status, tc::kTimeoutFull);
            flags[0] = 1;
            break;
          }
          __nanosleep(32);
        }
      asm volatile("fence.proxy.async.global;" ::: "memory"); // before the TMA reads of them
    }
    __syncthreads();
  }

  if (warp == GM_CONSUMERS) {
    // ------------------------------ producer ------------------------------
    if (lane == 0) {
      for (int i = 0; i < nun; ++i) {
        const int s = i % GM_STAGES;
        if (i >= GM_STAGES && !tc::mbar_wait(&empty[s], ((i / GM_STAGES) - 1) & 1)) {
          atomicExch(&g_gemv_mma_status, tc::kTimeoutEmpty);
          flags[0] = 1;
          break;
        }
        if (i >= pre) load_weights(i);
        const int kb = (u0 + i) % g.kunits;
        uint8_t *sa = sm + L::kOffA + s * L::kA;
        tc::tma_load_2d(sa, &map_a, &full[s], kb * GM_TK, 0);
        tc::tma_load_2d(sa + L::kA / 2, &map_a, &full[s], kb * GM_TK + 64, 0);
      }
    }
    return;
  }

  // ------------------------------ consumers -------------------------------
  const int wn = warp & 1, quad = warp >> 1;
  // Stage i goes to group i % G; every fill of a ring slot goes to the same
  // group, which has consumed the previous fill before waiting on the next.
  static_assert(GM_STAGES % G == 0, "each ring stage must belong to one stage group");
  constexpr int kSlabs = GM_QUADS / G;        // slabs per stage
  constexpr int kSlabRows = GM_TK / kSlabs;   // rows per slab
  const int grp = quad % G, slab = quad / G;
  const int gq = lane >> 2, t = lane & 3;
  const uint32_t mlo = g.is_signed ? 0x64086408u : 0x64006400u;
  const uint32_t mhi = g.is_signed ? 0x64806480u : 0x64006400u;
  const float blo = g.is_signed ? 1032.0f : 1024.0f;
  const float bhi = g.is_signed ? 1152.0f : 1024.0f;
  // scale blocks per slab and k16 steps per scale block
  constexpr int kSubs = (kSlabRows / 16) / KS;  // scale blocks per slab
  static_assert(kSubs * KS * 16 == kSlabRows, "slab rows");
  const int slab_row0 = slab * kSlabRows;
  const float scalar = g.srows ? 0.0f : __half2float(__ushort_as_half(__ldg(g.scalar_scale)));
  float acc[8][NT][4];
#pragma unroll
  for (int mt = 0; mt < 8; ++mt)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[mt][nt][e] = 0.0f;
  bool ok = true;
  const int first_tile = u0 / g.kunits;

  int seg0 = 0; // first stage of the current tile segment
  while (seg0 < nun) {
    const int tile = (u0 + seg0) / g.kunits;
    const int seg1 = min(nun, (tile + 1) * g.kunits - u0);
    // this group's stages of the segment: i = seg0 .. seg1-1 with i % G == grp
    for (int i = seg0 + ((grp - seg0 % G + G) % G); i < seg1; i += G) {
      const int s = i % GM_STAGES;
      if (ok && flags[0]) ok = false;
      if (ok && !tc::mbar_wait(&full[s], (i / GM_STAGES) & 1)) {
        atomicExch(&g_gemv_mma_status, tc::kTimeoutFull);
        flags[0] = 1;
        ok = false;
      }
      if (ok) {
        const uint8_t *wst = sm + s * GM_W_BYTES;
        const uint8_t *ast = sm + L::kOffA + s * L::kA;
        const uint8_t *sst = sm + L::kOffS + s * GM_SC_BYTES;
        // Rows past K read as zeros in every operand (TMA fill), so a
        // ragged last stage needs no bounds.
#pragma unroll
        for (int sub = 0; sub < kSubs; ++sub) {
          const int r0 = slab_row0 + sub * KS * 16;
          const int srow = (g.block && g.block < GM_TK) ? r0 / g.block : 0;
          // this scale row's factors are read after the k16 steps, so they
          // hold no registers during them
          const uint8_t *srow_p = sst + srow * GM_TN * 2 + wn * 256;
          // Rows 8..15 of the activations (M > 8) take a second pass over the
          // stage, so the registers stay those of one 8-row tile.
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
            for (int j = 0; j < KS; ++j)
              k16_step<NT>(wst, ast, r0 + 16 * j, wn, lane, gq, t, nt, mlo, mhi, D, O);
            // scale block done: acc += s_eff * (D - bias * sum a), the high
            // nibbles' scale divided by 16
#pragma unroll
            for (int mt = 0; mt < 8; ++mt) {
              float se0 = scalar, se1 = scalar * 0.0625f;
              if (g.srows) {
                const uint32_t w2 = *reinterpret_cast<const uint32_t *>(srow_p + mt_col(mt, gq) * 2);
                se0 = __half2float(__ushort_as_half((uint16_t)(w2 & 0xffffu)));
                se1 = __half2float(__ushort_as_half((uint16_t)(w2 >> 16))) * 0.0625f;
              }
              // pairs (e = 0, 1) and (2, 3) share the bias and the scale: one
              // packed fp32x2 FMA per pair (the same IEEE fma per element)
              const float2 o01 = make_float2(O[0], O[1]);
              const float2 c01 = ffma2(make_float2(-blo, -blo), o01, make_float2(D[mt][0], D[mt][1]));
              const float2 c23 = ffma2(make_float2(-bhi, -bhi), o01, make_float2(D[mt][2], D[mt][3]));
              const float2 a01 = ffma2(make_float2(se0, se0), c01,
                                       make_float2(acc[mt][nt][0], acc[mt][nt][1]));
              const float2 a23 = ffma2(make_float2(se1, se1), c23,
                                       make_float2(acc[mt][nt][2], acc[mt][nt][3]));
              acc[mt][nt][0] = a01.x;
              acc[mt][nt][1] = a01.y;
              acc[mt][nt][2] = a23.x;
              acc[mt][nt][3] = a23.y;
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&empty[s]);
    }

    // ------------------------ end of a tile segment ------------------------
    // Sum the warp groups of each column half in group order, in one round:
    // groups 1.. leave their sums in shared memory, group 0 adds them.
    consumers_sync();
    if (quad > 0) {
      float *r = red + (size_t)((quad - 1) * 2 + wn) * 32 * NT * 32;
#pragma unroll
      for (int mt = 0; mt < 8; ++mt)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) r[((mt * NT + nt) * 4 + e) * 32 + lane] = acc[mt][nt][e];
    }
    consumers_sync();
    if (quad == 0) {
#pragma unroll
      for (int q = 0; q < GM_QUADS - 1; ++q) {
        const float *r = red + (size_t)(q * 2 + wn) * 32 * NT * 32;
#pragma unroll
        for (int mt = 0; mt < 8; ++mt)
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[mt][nt][e] += r[((mt * NT + nt) * 4 + e) * 32 + lane];
      }
    }
    const int uf = tile * g.kunits, ul = uf + g.kunits - 1;
    const int cf = g.aligned ? a_first : cta_of(uf, g.units, g.grid);
    const int cl = g.aligned ? a_first + a_nsl - 1 : cta_of(ul, g.units, g.grid);
    const int pj = prob_of(g, tile);               // this tile's projection
    const int n0 = (tile - prob_first_tile(g, pj)) * GM_TN, Nj = g.Np[pj];
    if (g.aligned && cf != cl) {
      // ---- tile-aligned split: the tile's first CTA (slice 0) merges ----
      float *part = g.partials + (size_t)(b * 2) * g.M * GM_TN;
      uint32_t *ctr = g.counters + tile;
      if (a_slice != 0) {
        // Contributor: the partial to global memory, then a release add on
        // the tile's counter (with kAbortMark when a wait gave up).
        if (quad == 0) {
#pragma unroll
          for (int mt = 0; mt < 8; ++mt) {
            const int col = wn * 128 + mt_col(mt, gq);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              const int m = nt * 8 + 2 * t;
              if (m < g.M)
                *reinterpret_cast<float2 *>(part + m * GM_TN + col) =
                    make_float2(acc[mt][nt][0], acc[mt][nt][2]);
              if (m + 1 < g.M)
                *reinterpret_cast<float2 *>(part + (m + 1) * GM_TN + col) =
                    make_float2(acc[mt][nt][1], acc[mt][nt][3]);
            }
          }
        }
        consumers_sync(); // every consumer's partial stores before the release below
        if (threadIdx.x == 0) red_release_add(ctr, flags[0] ? kAbortMark + 1u : 1u);
      } else {
        // Merger: its own partial stays in shared memory; wait (bounded) for
        // the other slices, reset the counter, sum the slices in order.
        consumers_sync(); // the group sum's reads of `red` are done
        if (quad == 0) {
#pragma unroll
          for (int mt = 0; mt < 8; ++mt) {
            const int col = wn * 128 + mt_col(mt, gq);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              const int m = nt * 8 + 2 * t;
              *reinterpret_cast<float2 *>(red + m * GM_TN + col) = make_float2(acc[mt][nt][0], acc[mt][nt][2]);
              *reinterpret_cast<float2 *>(red + (m + 1) * GM_TN + col) =
                  make_float2(acc[mt][nt][1], acc[mt][nt][3]);
            }
          }
        }
        if (threadIdx.x == 0) {
          // Every contributor arrives exactly once, also after a give-up
          // (each of its waits is bounded), so waiting for all of them and
          // resetting leaves the counter at zero for the next call.
          const uint64_t t0 = tc::globaltimer();
          uint32_t v = ld_acquire_gpu(ctr);
          bool arrived = true;
          while ((v & (kAbortMark - 1u)) < (uint32_t)(a_nsl - 1)) {
            if (tc::globaltimer() - t0 > 3 * g.wait_ns) {
              atomicExch(&g_gemv_mma_status, tc::kTimeoutFull);
              arrived = false;
              break;
            }
            __nanosleep(32);
            v = ld_acquire_gpu(ctr);
          }
          if (arrived) *ctr = 0u;
          flags[1] = arrived && (v >> 16) == 0u && !flags[0] ? 1 : 0;
        }
        consumers_sync();
        if (flags[1]) {
          const int nc = a_nsl;
          for (int e = threadIdx.x; e < g.M * (GM_TN / 4); e += GM_CONSUMERS * 32) {
            float4 sum = reinterpret_cast<const float4 *>(red)[e];
            for (int c0 = 1; c0 < nc; c0 += 16) {
              float4 v[16];
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                v[j] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                if (c0 + j < nc)
                  v[j] = __ldcg(reinterpret_cast<const float4 *>(
                                    g.partials + (size_t)((b + c0 + j) * 2) * g.M * GM_TN) + e);
              }
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                sum.x += v[j].x;
                sum.y += v[j].y;
                sum.z += v[j].z;
                sum.w += v[j].w;
              }
            }
            const int m = e / (GM_TN / 4), col = (e % (GM_TN / 4)) * 4;
            if (n0 + col >= Nj) continue; // ragged last tile; N % 4 == 0
            store_h2(g, pj, m, n0 + col, __floats2half2_rn(sum.x, sum.y));
            store_h2(g, pj, m, n0 + col + 2, __floats2half2_rn(sum.z, sum.w));
          }
        }
      }
    } else if (cf == cl) {
      // The whole tile is this CTA's: write the output.
      if (quad == 0 && ok) {
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
          const int col = n0 + wn * 128 + mt_col(mt, gq);
          if (col >= Nj) continue; // ragged last tile (N % 256 != 0); N is even
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            const int m = nt * 8 + 2 * t;
            if (m < g.M) store_h2(g, pj, m, col, __floats2half2_rn(acc[mt][nt][0], acc[mt][nt][2]));
            if (m + 1 < g.M)
              store_h2(g, pj, m + 1, col, __floats2half2_rn(acc[mt][nt][1], acc[mt][nt][3]));
          }
        }
      }
    } else {
      const int slot = tile == first_tile ? 0 : 1;
      float *part = g.partials + (size_t)(b * 2 + slot) * g.M * GM_TN;
      if (quad == 0) {
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
          const int col = wn * 128 + mt_col(mt, gq);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            const int m = nt * 8 + 2 * t;
            if (m < g.M)
              *reinterpret_cast<float2 *>(part + m * GM_TN + col) =
                  make_float2(acc[mt][nt][0], acc[mt][nt][2]);
            if (m + 1 < g.M)
              *reinterpret_cast<float2 *>(part + (m + 1) * GM_TN + col) =
                  make_float2(acc[mt][nt][1], acc[mt][nt][3]);
          }
        }
      }
      consumers_sync();
      if (threadIdx.x == 0) {
        // Release this CTA's partial (the barrier above orders the other
        // threads' stores before it), acquire the others' if last.
        // A CTA whose wait gave up arrives with kAbortMark, and then the last
        // one does not merge (the partials are not all valid).
        const uint32_t inc = flags[0] ? kAbortMark + 1u : 1u;
        const uint32_t now = atom_add_acq_rel(g.counters + tile, inc) + inc;
        const bool last = (now & (kAbortMark - 1u)) == (uint32_t)(cl - cf + 1);
        if (last) g.counters[tile] = 0u;
        flags[1] = last && (now >> 16) == 0u ? 1 : 0;
      }
      consumers_sync();
      if (flags[1] && ok) {
        // Last to arrive: sum the contributors' partials in CTA order, with the
        // loads of up to 16 contributors in flight before the first add.
        const int nc = cl - cf + 1;
        for (int e = threadIdx.x; e < g.M * (GM_TN / 4); e += GM_CONSUMERS * 32) {
          float4 sum = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
          for (int c0 = 0; c0 < nc; c0 += 16) {
            float4 v[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              v[j] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
              const int c = cf + c0 + j;
              if (c0 + j < nc) {
                const int cslot = unit_begin(c, g.units, g.grid) / g.kunits == tile ? 0 : 1;
                v[j] = __ldcg(reinterpret_cast<const float4 *>(
                                  g.partials + (size_t)(c * 2 + cslot) * g.M * GM_TN) + e);
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
          const int m = e / (GM_TN / 4), col = (e % (GM_TN / 4)) * 4;
          if (n0 + col >= Nj) continue; // ragged last tile; N % 4 == 0
          store_h2(g, pj, m, n0 + col, __floats2half2_rn(sum.x, sum.y));
          store_h2(g, pj, m, n0 + col + 2, __floats2half2_rn(sum.z, sum.w));
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
  if (g.world > 1) {
    // Publish completion: every CTA counts itself done with a gpu-scope
    // acquire/release add (the barrier orders its threads' peer stores before
    // it); the last one, having acquired them all, issues one system-scope
    // fence -- cumulative over every store it has observed -- and then stores
    // the call's generation in every rank's flag array (a release pattern).
    // One system-scope fence per call: it sits on the path to the next
    // launch, so per-CTA fences would each add their NVLink round trip.
    consumers_sync();
    if (threadIdx.x == 0) {
      const uint32_t prev = atom_add_acq_rel(g.pctr, 1u);
      if (prev + 1 == gridDim.x) {
        g.pctr[0] = 0u;
        const uint32_t gen = g.pctr[1] + 1u;
        g.pctr[1] = gen;
        asm volatile("fence.acq_rel.sys;" ::: "memory");
#pragma unroll
        for (int r = 0; r < kPeerMax; ++r)
          if (r < g.world)
            asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(g.peer_flags[r] + g.rank), "r"(gen)
                         : "memory");
      }
    }
  }
}

struct MmaPlan {
  int nt = 1, groups = 4, grid = 0, units = 0, kunits = 0, ntiles = 0, srows = 0, block = 0;
  int aligned = 0, cq = 0, cr = 0;
  int tile_end[kGroupMax] = {};
  size_t ws = 0;
};

// One plan for the projections ps[0 .. count-1] (same activations, M, K,
// weight type and scale layout): their 256-column tiles numbered one after
// the other.
MmaPlan mma_plan(const DqMmParams *ps, int count) {
  const DqMmParams &p = ps[0];
  MmaPlan m;
  m.nt = p.M <= 8 ? 1 : 2;
  m.ntiles = 0;
  for (int i = 0; i < count; ++i) {
    m.ntiles += (int)((ps[i].N + GM_TN - 1) / GM_TN); // a last tile may be ragged (TMA zero-fills)
    m.tile_end[i] = m.ntiles;
  }
  m.kunits = (int)((p.K + GM_TK - 1) / GM_TK);
  m.units = m.ntiles * m.kunits;
  // Two CTAs per SM once there are two units per CTA: in a chain of decode
  // launches the CTAs of the next launch take the slots that this launch's
  // CTAs free as they finish (config 3, grouped step: 45.7 us at B = 1 and
  // 55.7 us at B = 8 against 48.6 / 56.6 us with two CTAs per SM only for
  // launches of 8 units per SM or more) -- unless that would split a tile
  // among more than 20 CTAs, whose merge reads every slice's partial (the
  // narrow column shards of a multi-GPU layer).
  const int sms = sm_count();
  const bool two = m.units >= 2 * sms && 2 * sms <= 20 * m.ntiles;
  m.grid = std::min(m.units, sms * (two ? GM_CTAS_PER_SM : 1));
  // Up to one tile per CTA: split each tile's K range among whole CTAs (a
  // CTA never straddles two tiles, and each tile's first CTA merges), which
  // takes one merge per tile off the critical path of stream-K.  Kept only
  // while it balances the work: whole CTAs per tile leave some CTAs with
  // ceil(kunits / cq) units against ceil(units / grid) for stream-K
  // (4096 x 22016 in one launch: 32 against 19 units).
  m.aligned = m.ntiles <= m.grid && getenv("ONNXL_B200_GEMV_STREAMK") == nullptr;
  if (m.aligned) {
    m.cq = m.grid / m.ntiles;
    m.cr = m.grid % m.ntiles;
    const int amax = (m.kunits + m.cq - 1) / m.cq, smax = (m.units + m.grid - 1) / m.grid;
    if (4 * amax > 5 * smax) m.aligned = 0;
  }
  // Stages per CTA below about 2 per stage group leave groups idle: put all
  // warps on every stage instead.
  const int per_cta = m.aligned ? (m.kunits + m.cq - 1) / m.cq : (m.units + m.grid - 1) / m.grid;
  m.groups = per_cta <= kGroupsThreshold ? 1 : GM_QUADS;
  if (p.slayout == kScaleTensor) {
    m.srows = 0;
  } else if (p.slayout == kScaleAxis1) {
    m.srows = 1;
  } else {
    m.block = (int)p.block;
    m.srows = p.block < GM_TK ? (int)(GM_TK / p.block) : 1;
  }
  bool split = m.aligned && m.grid > m.ntiles;
  for (int tile = 0; tile < m.ntiles && !split && !m.aligned; ++tile) {
    const int uf = tile * m.kunits, ul = uf + m.kunits - 1;
    const int cf = (int)(((int64_t)(uf + 1) * m.grid - 1) / m.units);
    const int cl = (int)(((int64_t)(ul + 1) * m.grid - 1) / m.units);
    split = cf != cl;
  }
  // Arrival counters always (they start the workspace); partials when a tile is shared.
  m.ws = kCounterBytes + (split ? (size_t)m.grid * 2 * p.M * GM_TN * 4 : 0);
  return m;
}

template <int NT, int G, int KS, int NP>
int launch_mma(const DqMmParams *ps, const MmaPlan &m, void *workspace, cudaStream_t st) {
  constexpr int count = NP;
  const DqMmParams &p = ps[0];
  GmMaps<NP> maps;
  memset(&maps, 0, sizeof(maps));
  CUtensorMap map_a;
  for (int i = 0; i < count; ++i) {
    const DqMmParams &q = ps[i];
    {
      const uint64_t dims[2] = {(uint64_t)q.N / 2, (uint64_t)q.K};
      const uint64_t strides[1] = {(uint64_t)q.N / 2};
      const uint32_t box[2] = {GM_TN / 2, GM_TK};
      int rc = make_tensor_map(&maps.w[i], CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, q.w, dims, strides, box,
                               CU_TENSOR_MAP_SWIZZLE_128B);
      if (rc) return rc;
    }
    maps.s[i] = maps.w[i];
    if (m.srows) {
      const uint64_t rows = q.slayout == kScaleAxis1 ? 1 : (uint64_t)q.s_alen;
      const uint64_t dims[2] = {(uint64_t)q.N, rows};
      const uint64_t strides[1] = {(uint64_t)q.N * 2};
      const uint32_t box[2] = {GM_TN, (uint32_t)m.srows};
      int rc = make_tensor_map(&maps.s[i], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, q.scale, dims, strides,
                               box, CU_TENSOR_MAP_SWIZZLE_NONE);
      if (rc) return rc;
    }
  }
  {
    const uint64_t dims[2] = {(uint64_t)p.K, (uint64_t)p.M};
    const uint64_t strides[1] = {(uint64_t)p.K * 2};
    const uint32_t box[2] = {64, (uint32_t)(8 * NT)};
    int rc = make_tensor_map(&map_a, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, p.a, dims, strides, box,
                             CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  GmArgs<NP> a{};
  a.counters = static_cast<uint32_t *>(workspace);
  a.partials = reinterpret_cast<float *>(static_cast<uint8_t *>(workspace) + kCounterBytes);
  a.M = (int)p.M;
  a.K = (int)p.K;
  a.world = p.world > 1 ? p.world : 1;
  a.rank = p.rank;
  for (int i = 0; i < count; ++i) {
    const DqMmParams &q = ps[i];
    a.tile_end[i] = m.tile_end[i];
    a.Np[i] = (int)q.N;
    a.y[i] = static_cast<__half *>(q.y);
    a.ldy[i] = p.world > 1 ? q.n_full : q.N;
    a.col_off[i] = p.world > 1 ? q.col_off : 0;
    for (int r = 0; r < kPeerMax; ++r)
      a.peer_y[i][r] = r < a.world ? static_cast<__half *>(q.peer_full[r]) : nullptr;
  }
  a.ntiles = m.ntiles;
  a.kunits = m.kunits;
  a.units = m.units;
  a.grid = m.grid;
  a.block = m.block;
  a.srows = m.srows;
  a.is_signed = p.wdt == kInt4;
  a.scalar_scale = reinterpret_cast<const uint16_t *>(p.scale);
  for (int r = 0; r < kPeerMax; ++r) a.peer_flags[r] = r < a.world ? p.peer_flags[r] : nullptr;
  a.pctr = p.pctr;
  a.wait_input = p.wait_input;
  a.aligned = m.aligned;
  a.cq = m.cq;
  a.cr = m.cr;
  a.wait_ns = kWaitNs;
  auto kern = dq_gemv_mma<NT, G, KS, NP>;
  const size_t smem = GmSmem<NT>::kDynamic;
  B2_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)m.grid);
  cfg.blockDim = dim3(GM_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  B2_CUDA(cudaLaunchKernelEx(&cfg, kern, maps, map_a, a));
  return B2_OK;
}

} // namespace

bool dq_mma_eligible(const DqMmParams &p) {
  if (p.wdt != kInt4 && p.wdt != kUint4) return false;
  if (!p.s_f16 || p.zp != nullptr || p.ydt != kFloat16) return false;
  if (p.cast_dt != 0 && p.cast_dt != kFloat16) return false;
  // N % 32: packed rows are whole 16-byte units (TMA strides); the last
  // 256-column tile may be partial.
  if (p.M < 1 || p.M > 16 || p.N < 32 || p.N % 32 != 0 || p.K < 16 || p.K % 8 != 0)
    return false;
  if (p.N > (int64_t)1 << 30 || p.K > (int64_t)1 << 30) return false;
  const int64_t ntiles = (p.N + GM_TN - 1) / GM_TN;
  if (ntiles > (int64_t)kMaxCounters) return false;
  // unit numbers times the grid size stay below 2^31 (32-bit index arithmetic)
  const int64_t units = ntiles * ((p.K + GM_TK - 1) / GM_TK);
  if (units * (int64_t)(sm_count() + 1) >= ((int64_t)1 << 31)) return false;
  switch (p.slayout) {
  case kScaleTensor:
  case kScaleAxis1: return true;
  case kScaleAxis0Block:
    if (p.block % 32 != 0) return false;
    return p.block <= GM_TK ? GM_TK % p.block == 0 : p.block % GM_TK == 0;
  default: return false;
  }
}

bool dq_mma_aligned(const DqMmParams &p) {
  auto al = [](const void *q, uintptr_t n) { return (reinterpret_cast<uintptr_t>(q) % n) == 0; };
  return al(p.a, 16) && al(p.w, 16) && al(p.y, 4) &&
         (p.slayout == kScaleTensor || al(p.scale, 16));
}

size_t dq_mma_workspace(const DqMmParams &p) { return mma_plan(&p, 1).ws; }

bool dq_mma_group_eligible(const DqMmParams *ps, int count) {
  if (count < 1 || count > kGroupMax) return false;
  int64_t ntiles = 0;
  for (int i = 0; i < count; ++i) {
    const DqMmParams &q = ps[i];
    if (!dq_mma_eligible(q) || !dq_mma_aligned(q)) return false;
    if (q.a != ps[0].a || q.M != ps[0].M || q.K != ps[0].K || q.wdt != ps[0].wdt ||
        q.slayout != ps[0].slayout || q.block != ps[0].block || q.s_alen != ps[0].s_alen)
      return false;
    ntiles += (q.N + GM_TN - 1) / GM_TN;
  }
  if (ntiles > (int64_t)kMaxCounters) return false;
  const int64_t units = ntiles * ((ps[0].K + GM_TK - 1) / GM_TK);
  return units * (int64_t)(sm_count() + 1) < ((int64_t)1 << 31);
}

size_t dq_mma_group_workspace(const DqMmParams *ps, int count) { return mma_plan(ps, count).ws; }

// One instance per (activation tiles, stage groups, k16 steps per scale
// block) of the plan and member count.
template <int NT, int G, int KS>
int launch_np(const DqMmParams *ps, int count, const MmaPlan &m, void *workspace, cudaStream_t st) {
  switch (count) {
  case 1: return launch_mma<NT, G, KS, 1>(ps, m, workspace, st);
  case 2: return launch_mma<NT, G, KS, 2>(ps, m, workspace, st);
  case 3: return launch_mma<NT, G, KS, 3>(ps, m, workspace, st);
  default: return launch_mma<NT, G, KS, 4>(ps, m, workspace, st);
  }
}

int dq_mma_launch_group(const DqMmParams *ps, int count, void *workspace, cudaStream_t st) {
  const MmaPlan m = mma_plan(ps, count);
  if (m.ws && workspace == nullptr) B2_FAIL(B2_ERR_WORKSPACE, "workspace of %zu bytes required", m.ws);
  if (m.groups == 1) // 32-row slabs: scale blocks are 32 rows or more
    return m.nt == 1 ? launch_np<1, 1, 2>(ps, count, m, workspace, st)
                     : launch_np<2, 1, 2>(ps, count, m, workspace, st);
  // 128-row slabs: k16 steps per scale block
  const int ks = (m.block == 0 || m.block >= GM_TK) ? 8 : m.block / 16;
  if (m.nt == 1) {
    if (ks == 2) return launch_np<1, GM_QUADS, 2>(ps, count, m, workspace, st);
    if (ks == 4) return launch_np<1, GM_QUADS, 4>(ps, count, m, workspace, st);
    return launch_np<1, GM_QUADS, 8>(ps, count, m, workspace, st);
  }
  if (ks == 2) return launch_np<2, GM_QUADS, 2>(ps, count, m, workspace, st);
  if (ks == 4) return launch_np<2, GM_QUADS, 4>(ps, count, m, workspace, st);
  return launch_np<2, GM_QUADS, 8>(ps, count, m, workspace, st);
}

int dq_mma_launch(const DqMmParams &p, void *workspace, cudaStream_t st) {
  return dq_mma_launch_group(&p, 1, workspace, st);
}

} // namespace b2

namespace b2 {
// Host: the time-out code this file's kernels recorded (0: none); reset != 0
// clears it.  Synchronous (the copy waits for the device).
int status_read_gemv_mma(int reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_gemv_mma_status, sizeof(int)) != cudaSuccess) return -1;
  if (reset && v) {
    const int z = 0;
    if (cudaMemcpyToSymbol(g_gemv_mma_status, &z, sizeof(int)) != cudaSuccess) return -1;
  }
  return v;
}
} // namespace b2
