// Prefill Attention on the 5th-generation tensor cores (tcgen05 + TMEM):
// FLOAT16 / BFLOAT16, head size 128, GQA, optional causal mask and softcap.
//
// Reference: kernel::Attention::operator() / ComputeAttentionRank4
// (onnx_light/onnx_extensions/kernels/kernels/nn/kernel_attention.cc:427-691,
// 767-852): per query row i (absolute position past_len + i) and key j,
// score = q . k * scale, softcap, causal mask j <= past_len + i, softmax with
// max subtraction, y = softmax . V -- in fp32 after promoting the inputs.
//
// One CTA owns 128 query rows -- pk query heads of one GQA group (pk the
// largest power of two up to 8 dividing the group) x 128 / pk positions, so a
// K / V tile read from L2 serves pk heads -- and walks 128-key tiles (up to
// the diagonal when causal):
//   warp 8 (TMA)   loads the Q tile once, then K and V tiles through 2-stage
//                  rings of their own ([128 keys][64 dims] boxes, 128-byte
//                  swizzle): a K stage frees when S is done, a V stage when
//                  P.V is done, so K runs a tile ahead;
//   warp 9 (MMA)   issues S_j = Q . K_j^T into one of two TMEM S buffers
//                  (M = 128 query rows, N = 128 keys, fp32), and, once the
//                  softmax warps have written P_{j-1}, O += P_{j-1} . V_{j-1}
//                  into the TMEM O accumulator with P read from TMEM (V read
//                  MN-major from shared memory);
//   warps 0-7      two threads per query row (its TMEM lane), one per 64-
//                  column half: read S, online softmax in base 2 (row maximum
//                  and sum combined through shared memory), write P over the
//                  S buffer it came from (tcgen05.st), and read, scale and
//                  store O at the end.
// P in the input type: FLOAT16 P carries 11 significant bits, enough for the
// rel-L2 1e-3 contract.  BFLOAT16 P would carry only 8 (about 1e-3 relative
// error in O on its own), so it is split into P_hi = bf16(p) and
// P_lo = bf16(p - P_hi) (16 bits together) and P.V runs as two MMAs per k
// step, P_hi.V + P_lo.V, the FP32 accumulation of the reference
// (kernel_attention.cc:670-678) to about 2^-17.
// The running maximum is re-based lazily: only when a row's maximum grows by
// more than 8 (log2 units) are l and the TMEM O row rescaled, so P stays
// within 2^8 and most tiles touch O only through the MMA.
//
// Every mbarrier is waited phase by phase by the threads that depend on it,
// and no barrier can run two phases ahead of a waiter (each producer of a
// phase needs the waiter's previous step first), so the parity waits are
// exact.  All waits are bounded; a time-out sets the status word and the CTA
// skips the rest, frees its TMEM and exits.
#include <type_traits>

#include "b2_common.cuh"
#include "tc_common.cuh"

namespace b2 {

__device__ int g_attn_prefill_tc_status;

namespace {

constexpr int PT_D = 128;
constexpr int PT_M = 128;            // query rows per CTA
constexpr int PT_N = 128;            // keys per tile
constexpr int PT_SOFT_WARPS = 8;                  // two per query row: column halves
constexpr int PT_TMA_WARP = PT_SOFT_WARPS, PT_MMA_WARP = PT_SOFT_WARPS + 1;
constexpr int PT_THREADS = (PT_SOFT_WARPS + 2) * 32;
constexpr uint32_t PT_HALF = 128 * 128;          // [128 rows][64 elements] bf16: 16 KB
constexpr uint32_t PT_OFF_Q = 0;                  // 2 halves
constexpr uint32_t PT_OFF_KV = 2 * PT_HALF;       // 2 stages x (K 2 halves, V 2 halves)
constexpr uint32_t PT_KV_STAGE = 4 * PT_HALF;
constexpr uint32_t PT_OFF_RED = PT_OFF_KV + 2 * PT_KV_STAGE; // [tile parity][half][row] partial maxima
constexpr uint32_t PT_OFF_BAR = PT_OFF_RED + 2 * 2 * PT_M * 4;
constexpr int PT_NBAR = 16;
// No alignment slack: the dynamic shared memory base is 1024-byte aligned
// (checked at run time; a CTA that finds it otherwise reports and skips).
constexpr size_t PT_SMEM = PT_OFF_BAR + PT_NBAR * 8 + 16;
// TMEM: S0 [0,128), S1 [128,256), O [256,384).  P_j is written over its S
// buffer: P_hi in columns [0, 64) of it, P_lo (BFLOAT16) in [64, 128).
constexpr uint32_t PT_TMEM_COLS = 512;
constexpr uint32_t PT_COL_O = 256;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRebase = 8.0f;                   // lazy re-basing threshold (log2 units)

struct PtArgs {
  void *y;
  int64_t y_sb, y_sh, y_ss; // strides (elements) of Y
  int Hq, group, Sq, L, past;
  int qtiles;
  int pk, np_, hpacks; // query heads per CTA (of one GQA group), positions per head, packs
  float scale_log2;
  float softcap;
  int causal;
};

template <typename T> __device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if constexpr (std::is_same<T, __half>::value) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t *>(&h);
  } else {
    const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t *>(&h);
  }
}

// 32 consecutive scores of one row into v[off .. off + 31]: raw when the
// scale is positive and there is no softcap (the scale is applied in the
// exponent), else already in base-2 units (scale or softcap); -inf for keys
// past the valid length or after the row's position.
__device__ __forceinline__ void load_scores(const uint32_t (&r)[32], float (&v)[64], int off,
                                            const PtArgs &g, bool need_mask, int key0, int pos) {
  if (g.softcap > 0.0f) {
#pragma unroll
    for (int e = 0; e < 32; ++e)
      v[off + e] = g.softcap * tanhf(__uint_as_float(r[e]) * g.scale_log2 / kLog2e / g.softcap) * kLog2e;
  } else if (g.scale_log2 > 0.0f) {
#pragma unroll
    for (int e = 0; e < 32; ++e) v[off + e] = __uint_as_float(r[e]);
  } else {
#pragma unroll
    for (int e = 0; e < 32; ++e) v[off + e] = __uint_as_float(r[e]) * g.scale_log2;
  }
  if (need_mask) {
#pragma unroll
    for (int e = 0; e < 32; ++e) {
      const int key = key0 + e;
      if (key >= g.L || (g.causal && key > pos)) v[off + e] = -INFINITY;
    }
  }
}

// 2^x with the hardware approximation (relative error about 2^-22; inputs are
// <= 8 here, and -inf gives 0).
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Three-way maximum (one instruction on sm_100).
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
// Element-wise a * b + c, a + b and a - b on two fp32 lanes (one packed
// instruction each on sm_100; the same IEEE operation per element).
__device__ __forceinline__ uint64_t f2pack(float x, float y) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(x), "f"(y));
  return r;
}
__device__ __forceinline__ float2 f2unpack(uint64_t r) {
  float2 v;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(v.x), "=f"(v.y) : "l"(r));
  return v;
}
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t fsub2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

template <typename T>
__global__ void __launch_bounds__(PT_THREADS, 1)
    attn_prefill_tc(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                    const __grid_constant__ CUtensorMap map_v, const PtArgs g) {
  extern __shared__ __align__(1024) uint8_t dsm[];
  if (tc::smem_u32(dsm) & 1023u) { // the layout below needs a 1024-byte aligned base
    if (threadIdx.x == 0) atomicExch(&g_attn_prefill_tc_status, tc::kTimeoutFull);
    return;
  }
  uint8_t *sm = dsm;
  uint64_t *bars = reinterpret_cast<uint64_t *>(sm + PT_OFF_BAR);
  float *red = reinterpret_cast<float *>(sm + PT_OFF_RED);
  uint64_t *q_full = bars;           // 1
  uint64_t *k_full = bars + 1;       // 2: K of a stage landed
  uint64_t *k_empty = bars + 3;      // 2: S of the stage's tile done (K free)
  uint64_t *v_full = bars + 5;       // 2
  uint64_t *v_empty = bars + 7;      // 2: P.V of the stage's tile done (V free)
  uint64_t *s_full = bars + 9;       // 2
  uint64_t *p_full = bars + 11;      // 2
  uint64_t *o_done = bars + 13;      // 2
  uint64_t *mma_done = bars + 15;    // 1: every MMA of the CTA finished
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + PT_NBAR);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // The 128 rows are pk query heads of one GQA group x np_ positions (row r:
  // head h0 + r / np_, position q0 + r % np_), so every K / V tile serves pk
  // heads.
  const int qt = g.qtiles - 1 - (int)(blockIdx.x % g.qtiles); // heavy (late) tiles first
  const int bhp = (int)(blockIdx.x / g.qtiles);
  const int b = bhp / g.hpacks, h0 = (bhp % g.hpacks) * g.pk, kvh = h0 / g.group;
  const int q0 = qt * g.np_;
  const int kend = g.causal ? min(g.L, g.past + q0 + g.np_) : g.L;
  const int ntiles = (kend + PT_N - 1) / PT_N;

  if (threadIdx.x == 0) {
    tc::mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(&k_full[i], 1);
      tc::mbar_init(&k_empty[i], 1);
      tc::mbar_init(&v_full[i], 1);
      tc::mbar_init(&v_empty[i], 1);
      tc::mbar_init(&s_full[i], 1);
      tc::mbar_init(&p_full[i], PT_SOFT_WARPS);
      tc::mbar_init(&o_done[i], 1);
    }
    tc::mbar_init(mma_done, 1);
    *abort_flag = 0;
    tc::fence_barrier_init();
  }
  if (warp == PT_MMA_WARP) {
    tc::tmem_alloc(tmem_slot, PT_TMEM_COLS);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == PT_TMA_WARP) {
    // ------------------------------ TMA producer ------------------------------
    // Lane 0 fills the K ring (a stage is free once S of its tile is done),
    // lane 1 the V ring (free once P.V is done), so the next K tile is on its
    // way while the softmax and P.V of the current one still run.
    if (lane < 2) {
      const bool is_k = lane == 0;
      const CUtensorMap *map = is_k ? &map_k : &map_v;
      uint64_t *full = is_k ? k_full : v_full;
      uint64_t *empty = is_k ? k_empty : v_empty;
      if (is_k) {
        tc::prefetch_tensormap(&map_q);
        tc::prefetch_tensormap(&map_k);
        tc::mbar_expect_tx(q_full, 2 * PT_HALF);
        tc::tma_load_4d(sm + PT_OFF_Q, &map_q, q_full, 0, q0, h0, b);
        tc::tma_load_4d(sm + PT_OFF_Q + PT_HALF, &map_q, q_full, 64, q0, h0, b);
      } else {
        tc::prefetch_tensormap(&map_v);
      }
      int issued = 0;
      for (int j = 0; j < ntiles; ++j) {
        const int s = j & 1;
        if (j >= 2 && !tc::mbar_wait(&empty[s], ((j - 2) >> 1) & 1)) {
          atomicExch(&g_attn_prefill_tc_status, tc::kTimeoutEmpty);
          *abort_flag = 1;
          break;
        }
        if (*abort_flag) break;
        issued = j + 1;
        uint8_t *st = sm + PT_OFF_KV + s * PT_KV_STAGE + (is_k ? 0u : 2 * PT_HALF);
        const int key0 = j * PT_N;
        tc::mbar_expect_tx(&full[s], 2 * PT_HALF);
        tc::tma_load_4d(st, map, &full[s], 0, key0, kvh, b);
        tc::tma_load_4d(st + PT_HALF, map, &full[s], 64, key0, kvh, b);
      }
      // No copy may land after the CTA exits: wait (bounded) for the last
      // fills of both stages (and Q).  On the normal path they are done.
      for (int j = max(0, issued - 2); j < issued; ++j) tc::mbar_wait(&full[j & 1], (j >> 1) & 1);
      if (is_k) tc::mbar_wait(q_full, 0);
    }
  } else if (warp == PT_MMA_WARP) {
    // ------------------------------ MMA issuer --------------------------------
    if (tc::elect_one()) {
      const uint32_t fmt = std::is_same<T, __half>::value ? 0u : 1u;
      const uint32_t id_s = tc::idesc(1, fmt, fmt, 0, 0, PT_M, PT_N);
      const uint32_t id_o = tc::idesc(1, fmt, fmt, 0, 1, PT_M, PT_D);
      const uint32_t q_base = tc::smem_u32(sm + PT_OFF_Q);
      bool ok = tc::mbar_wait(q_full, 0);
      constexpr bool kSplitP = !std::is_same<T, __half>::value;
      auto issue_pv = [&](int j) {
        // O (+)= P_j . V_j: A = P from TMEM (over S buffer j & 1), B = V
        // (MN-major over dims); BFLOAT16 adds P_lo . V_j
        if (!tc::mbar_wait(&p_full[j & 1], (j >> 1) & 1)) return false;
        if (!tc::mbar_wait(&v_full[j & 1], (j >> 1) & 1)) return false;
        tc::tc_fence_after();
        const uint32_t p_col = tmem + (uint32_t)(j & 1) * PT_N;
        const uint32_t v_base = tc::smem_u32(sm + PT_OFF_KV + (j & 1) * PT_KV_STAGE + 2 * PT_HALF);
#pragma unroll
        for (int kk = 0; kk < PT_N / 16; ++kk) {
          const uint64_t bd = tc::sdesc_sw128(v_base + kk * 16 * 128, PT_HALF, 1024);
          tc::mma_f16_ts(tmem + PT_COL_O, p_col + kk * 8, bd, id_o, (j > 0 || kk > 0) ? 1u : 0u);
          if (kSplitP) tc::mma_f16_ts(tmem + PT_COL_O, p_col + 64 + kk * 8, bd, id_o, 1u);
        }
        tc::tc_commit(&o_done[j & 1]);
        tc::tc_commit(&v_empty[j & 1]);
        return true;
      };
      for (int j = 0; ok && j < ntiles; ++j) {
        if (*abort_flag || !tc::mbar_wait(&k_full[j & 1], (j >> 1) & 1)) {
          ok = false;
          break;
        }
        // S buffer j & 1 holds P_{j-2} until P.V of tile j - 2 is done.
        if (j >= 2 && !tc::mbar_wait(&o_done[j & 1], ((j - 2) >> 1) & 1)) {
          ok = false;
          break;
        }
        tc::tc_fence_after();
        const uint32_t k_base = tc::smem_u32(sm + PT_OFF_KV + (j & 1) * PT_KV_STAGE);
#pragma unroll
        for (int kk = 0; kk < PT_D / 16; ++kk) {
          const uint64_t ad = tc::sdesc_sw128(q_base + (kk >> 2) * PT_HALF + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = tc::sdesc_sw128(k_base + (kk >> 2) * PT_HALF + (kk & 3) * 32, 16, 1024);
          tc::mma_f16(tmem + (j & 1) * PT_N, ad, bd, id_s, kk > 0 ? 1u : 0u);
        }
        tc::tc_commit(&s_full[j & 1]);
        tc::tc_commit(&k_empty[j & 1]);
        if (j >= 1 && !issue_pv(j - 1)) ok = false;
      }
      if (ok && ntiles > 0 && !issue_pv(ntiles - 1)) ok = false;
      if (!ok) {
        atomicExch(&g_attn_prefill_tc_status, tc::kTimeoutFull);
        *abort_flag = 1;
      }
      // TMEM is freed below: wait (bounded) until every issued MMA is done.
      tc::tc_commit(mma_done);
      tc::mbar_wait(mma_done, 0);
    }
  } else {
    // ------------------------------ softmax warps -----------------------------
    // Two threads per query row (warps w and w + 4 share TMEM lanes 32 (w % 4)
    // .. + 31), each on one 64-column half of S, P and O; the row maximum and
    // sum combine through shared memory.  Control flow stays warp-uniform
    // (the TMEM loads and stores are warp-collective), and every softmax warp
    // takes every named barrier even after a time-out, so none can hang.
    const int quarter = warp & 3, half = warp >> 2;
    const int row = quarter * 32 + lane;           // query row in the tile = TMEM lane
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const int pos = g.past + q0 + row % g.np_;     // absolute position of the row
    float m_ref = -INFINITY, l_part = 0.0f;
    // scores are kept raw and scaled inside the exponent's FMA when the scale
    // is positive and there is no softcap; otherwise transformed up front
    const float vk = (g.softcap <= 0.0f && g.scale_log2 > 0.0f) ? g.scale_log2 : 1.0f;
    bool ok = true;
    auto uniform_wait = [&](uint64_t *bar, uint32_t parity) {
      const bool w = ok && !*abort_flag && tc::mbar_wait(bar, parity);
      return __all_sync(0xffffffffu, w);
    };
    auto softmax_sync = [] { asm volatile("bar.sync 1, %0;" ::"n"(PT_SOFT_WARPS * 32) : "memory"); };
    for (int j = 0; j < ntiles; ++j) {
      if (!uniform_wait(&s_full[j & 1], (j >> 1) & 1)) ok = false;
      tc::tc_fence_after();
      const int key0 = j * PT_N;
      const bool need_mask = key0 + PT_N > g.L || (g.causal && key0 + PT_N - 1 > g.past + q0);
      const uint32_t s_col = tmem + lane_off + (j & 1) * PT_N + half * 64;
      // pass 1: the half row's 64 scores stay in registers (v, in units where
      // p = 2^(v * vk - m)); this half's maximum, then the row's through
      // shared memory
      float v[64];
      float mx = -INFINITY;
      if (ok) {
        uint32_t r0[32], r1[32];
        tc::tmem_ld32(s_col, r0);
        tc::tmem_ld32(s_col + 32, r1);
        tc::tmem_ld_wait();
        load_scores(r0, v, 0, g, need_mask, key0 + half * 64, pos);
        load_scores(r1, v, 32, g, need_mask, key0 + half * 64 + 32, pos);
#pragma unroll
        for (int e = 0; e < 64; e += 2) mx = max3f(mx, v[e], v[e + 1]);
        mx *= vk; // vk > 0: the maximum of the scaled scores
      }
      float *rm = red + (j & 1) * 2 * PT_M;
      rm[half * PT_M + row] = mx;
      softmax_sync();
      mx = fmaxf(mx, rm[(half ^ 1) * PT_M + row]);
      if (!ok) continue;
      // Re-base a row when its maximum grew by more than kRebase: l and its O
      // row (after the previous P.V finished) scale by 2^(m_old - m_new).
      const bool reb = mx > m_ref + kRebase;
      float corr = 1.0f;
      if (reb) {
        corr = m_ref == -INFINITY ? 0.0f : exp2f(m_ref - mx);
        l_part *= corr;
        m_ref = mx;
      }
      if (j >= 1 && __any_sync(0xffffffffu, reb)) {
        if (!uniform_wait(&o_done[(j - 1) & 1], ((j - 1) >> 1) & 1)) {
          ok = false;
          continue;
        }
        tc::tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          const uint32_t o_col = tmem + lane_off + PT_COL_O + half * 64 + c * 32;
          uint32_t r[32];
          tc::tmem_ld32(o_col, r);
          tc::tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * corr);
          tc::tmem_st32(o_col, r);
        }
        tc::tmem_st_wait();
      }
      // pass 2: P for this half (keys half * 64 .. + 63) over the S buffer
      // the scores came from (every thread of the row has read its S half
      // before the barrier above); masked scores are -inf and give 0
      // pairs of keys on the packed fp32x2 pipe: the exponent's argument, the
      // running sums (two lanes, added at the end) and the bf16 low parts
      const uint64_t nm2 = f2pack(-m_ref, -m_ref), vk2 = f2pack(vk, vk);
      uint64_t ls2 = f2pack(0.0f, 0.0f);
      const uint32_t p_col = tmem + lane_off + (j & 1) * PT_N + half * 32;
#pragma unroll
      for (int c = 0; c < 2; ++c) { // 32 keys (16 packed columns) at a time
        uint32_t ph[16];
        uint32_t pl[std::is_same<T, __half>::value ? 1 : 16];
#pragma unroll
        for (int u = 0; u < 16; ++u) {
          const float2 t = f2unpack(ffma2(f2pack(v[c * 32 + 2 * u], v[c * 32 + 2 * u + 1]), vk2, nm2));
          const float p0 = ex2(t.x), p1 = ex2(t.y);
          const uint64_t pp = f2pack(p0, p1);
          ls2 = fadd2(ls2, pp);
          ph[u] = pack2<T>(p0, p1);
          if constexpr (!std::is_same<T, __half>::value) {
            const float2 lo = f2unpack(fsub2(pp, f2pack(__uint_as_float(ph[u] << 16),
                                                        __uint_as_float(ph[u] & 0xffff0000u))));
            pl[u] = pack2<T>(lo.x, lo.y);
          }
        }
        tc::tmem_st16(p_col + c * 16, ph);
        if constexpr (!std::is_same<T, __half>::value) tc::tmem_st16(p_col + 64 + c * 16, pl);
      }
      tc::tmem_st_wait();
      {
        const float2 l2 = f2unpack(ls2);
        l_part += l2.x + l2.y;
      }
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&p_full[j & 1]);
    }
    // y = O / l, l = the two halves' sums (the reduction slots of tile parity 0
    // are free: every thread has passed the last tile's barrier)
    const int last = ntiles - 1;
    const bool fin = uniform_wait(&o_done[last & 1], (last >> 1) & 1);
    softmax_sync();
    red[half * PT_M + row] = l_part;
    softmax_sync();
    const float l_sum = l_part + red[(half ^ 1) * PT_M + row];
    if (fin) {
      tc::tc_fence_after();
      const int qrow = q0 + row % g.np_;
      const float inv = l_sum > 0.0f ? 1.0f / l_sum : 0.0f;
      T *yr = static_cast<T *>(g.y) + (int64_t)b * g.y_sb + (int64_t)(h0 + row / g.np_) * g.y_sh +
              (int64_t)qrow * g.y_ss + half * 64;
      uint32_t r[32];
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        tc::tmem_ld32(tmem + lane_off + PT_COL_O + half * 64 + c * 32, r);
        tc::tmem_ld_wait();
        if (qrow < g.Sq) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 o;
            o.x = pack2<T>(__uint_as_float(r[8 * q + 0]) * inv, __uint_as_float(r[8 * q + 1]) * inv);
            o.y = pack2<T>(__uint_as_float(r[8 * q + 2]) * inv, __uint_as_float(r[8 * q + 3]) * inv);
            o.z = pack2<T>(__uint_as_float(r[8 * q + 4]) * inv, __uint_as_float(r[8 * q + 5]) * inv);
            o.w = pack2<T>(__uint_as_float(r[8 * q + 6]) * inv, __uint_as_float(r[8 * q + 7]) * inv);
            *reinterpret_cast<uint4 *>(yr + c * 32 + q * 8) = o;
          }
        }
      }
    } else {
      atomicExch(&g_attn_prefill_tc_status, tc::kTimeoutFull);
      *abort_flag = 1;
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == PT_MMA_WARP) tc::tmem_dealloc(tmem, PT_TMEM_COLS);
}

} // namespace

// Eligible: FLOAT16 / BFLOAT16, head size 128, no mask, no sliding window,
// 16-byte aligned Q / K / V / Y rows and strides (the caller checks pointers).
bool attn_prefill_tc_eligible(int dtype, int64_t D, int64_t Sq, bool mask, int64_t left_window,
                              int64_t right_window, const int64_t *qs, const int64_t *ks,
                              const int64_t *ys, int64_t L) {
  if (!(dtype == kFloat16 || dtype == kBfloat16) || D != PT_D || Sq < 2 || mask ||
      left_window >= 0 || right_window >= 0 || L < 1 || L >= ((int64_t)1 << 30) ||
      Sq >= ((int64_t)1 << 30))
    return false;
  for (int i = 0; i < 3; ++i)
    if (qs[i] % 8 != 0 || ks[i] % 8 != 0 || ys[i] % 8 != 0) return false;
  return true;
}

int attn_prefill_tc_launch(int dtype, const void *q, const int64_t *qs, const void *kc,
                           const void *vc, const int64_t *ks, void *y, const int64_t *ys,
                           int64_t B, int64_t Hq, int64_t Hkv, int64_t Sq, int64_t L, int64_t past,
                           float scale, float softcap, int causal, cudaStream_t st) {
  // Q, K, V as 4-D {dim, row, head, batch}; strides in elements {batch, head, row}
  CUtensorMap map_q, map_k, map_v;
  const CUtensorMapDataType tdt =
      dtype == kFloat16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const uint32_t box[4] = {64, 128, 1, 1};
  // pk = query heads per CTA: the largest power of two up to 8 that divides
  // the GQA group; the Q box is {64 dims, 128 / pk positions, pk heads}.
  int pk = 1;
  const int64_t group = Hq / Hkv;
  while (pk < 8 && group % (2 * pk) == 0) pk *= 2;
  const int np = PT_M / pk;
  {
    const uint64_t dims[4] = {(uint64_t)PT_D, (uint64_t)Sq, (uint64_t)Hq, (uint64_t)B};
    const uint64_t strides[3] = {(uint64_t)qs[2] * 2, (uint64_t)qs[1] * 2, (uint64_t)qs[0] * 2};
    const uint32_t qbox[4] = {64, (uint32_t)np, (uint32_t)pk, 1};
    int rc = make_tensor_map(&map_q, tdt, 4, q, dims, strides, qbox, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  {
    const uint64_t dims[4] = {(uint64_t)PT_D, (uint64_t)L, (uint64_t)Hkv, (uint64_t)B};
    const uint64_t strides[3] = {(uint64_t)ks[2] * 2, (uint64_t)ks[1] * 2, (uint64_t)ks[0] * 2};
    int rc = make_tensor_map(&map_k, tdt, 4, kc, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    rc = make_tensor_map(&map_v, tdt, 4, vc, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  PtArgs a{};
  a.y = y;
  a.y_sb = ys[0];
  a.y_sh = ys[1];
  a.y_ss = ys[2];
  a.Hq = (int)Hq;
  a.group = (int)(Hq / Hkv);
  a.Sq = (int)Sq;
  a.L = (int)L;
  a.past = (int)past;
  a.pk = pk;
  a.np_ = np;
  a.hpacks = (int)(Hq / pk);
  a.qtiles = (int)((Sq + np - 1) / np);
  a.scale_log2 = scale * kLog2e;
  a.softcap = softcap;
  a.causal = causal;
  const int64_t ctas = (int64_t)a.qtiles * B * a.hpacks;
  if (ctas >= ((int64_t)1 << 31)) B2_FAIL(B2_ERR_UNSUPPORTED, "b2_attention: too many query tiles");
  auto kern = dtype == kFloat16 ? attn_prefill_tc<__half> : attn_prefill_tc<__nv_bfloat16>;
  B2_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)PT_SMEM));
  kern<<<(unsigned)ctas, PT_THREADS, PT_SMEM, st>>>(map_q, map_k, map_v, a);
  B2_LAUNCH_CHECK();
  return B2_OK;
}

} // namespace b2

namespace b2 {
// Host: the time-out code this file's kernels recorded (0: none); reset != 0
// clears it.  Synchronous (the copy waits for the device).
int status_read_attn_prefill_tc(int reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_attn_prefill_tc_status, sizeof(int)) != cudaSuccess) return -1;
  if (reset && v) {
    const int z = 0;
    if (cudaMemcpyToSymbol(g_attn_prefill_tc_status, &z, sizeof(int)) != cudaSuccess) return -1;
  }
  return v;
}
} // namespace b2
