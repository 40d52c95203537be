// Decode-step Attention (one new query token per sequence) on tensor cores:
// GQA flash decoding for FLOAT16, head size 128.
//
// Reference: kernel::Attention::operator() / ComputeAttentionRank4
// (onnx_light/onnx_extensions/kernels/kernels/nn/kernel_attention.cc:427-691,
// 767-852): scores q . k * scale (default 1/sqrt(D)), optional softcap, causal
// mask j <= past_len (every cached key, for a single new token), softmax with
// max subtraction, y = softmax . V, all in fp32 after promoting the fp16 inputs.
//
// Here the Hq / Hkv query heads of one KV head (a GQA group, at most 16) are
// the 16 rows of mma.sync m16n8k16 tiles (rows past the group are zero), so
// every K and V byte read from HBM serves the whole group:
//   S[16 x 16 keys] = Q[16 x 128] . K^T      (fp16 inputs, fp32 accumulation)
//   online softmax of S in fp32 registers (running max / sum per row)
//   O[16 x 128]    += P[16 x 16 keys] . V     (P rounded to fp16, fp32 accumulation)
// P is the only quantity rounded on the way (2^-11 relative per probability);
// the reference keeps it in fp32.  The difference is far inside the rel-L2
// 1e-3 contract.
//
// Data path: the KV cache [B, Hkv, capacity, D] is read by TMA in stages of
// 32 keys (K and V, two 64-dim halves each with the 128-byte swizzle, 16 KB)
// through a 10-stage ring filled by one producer warp; the tensor map's key
// extent is the valid length L, so keys past it read as zeros and are masked.
// Four consumer warps take stages in turn and read the tiles with ldmatrix
// (K) and ldmatrix.trans (V).  Work split: the (b, kv_head) x 32-key chunks
// are numbered pair-major and the CTAs (one per SM) take equal contiguous
// ranges ("stream-K"); each CTA merges its warps' (m, l, O) per pair, writes
// y directly for pairs it covers whole, and otherwise leaves a partial that
// the last CTA to arrive on the pair merges in CTA order (deterministic).
#include "b2_common.cuh"
#include "tc_common.cuh"

namespace b2 {

__device__ int g_attn_decode_status;

namespace {

constexpr int AD_D = 128;
constexpr int AD_KEYS = 32;                       // keys per stage
constexpr int AD_STAGES = 12;
constexpr int AD_WARPS = 4;                       // consumer warps
// Stage i is consumed by warp i % AD_WARPS.  With the ring a multiple of the
// warp count, every fill of a stage goes to the same warp, which has consumed
// the previous fill before it waits on the next one; a parity wait can then
// never be satisfied by the fill before last (a warp waiting one phase ahead
// of a fill still in flight would see its parity as complete).
static_assert(AD_STAGES % AD_WARPS == 0, "each ring stage must belong to one consumer warp");
constexpr int AD_THREADS = (AD_WARPS + 1) * 32;
constexpr uint32_t AD_HALF = AD_KEYS * 64 * 2;    // one 64-dim half of K or V: 4 KB
constexpr uint32_t AD_STAGE = 4 * AD_HALF;        // K lo, K hi, V lo, V hi: 16 KB
constexpr uint32_t AD_OFF_MERGE = AD_STAGES * AD_STAGE;
constexpr uint32_t AD_MERGE_BYTES = AD_WARPS * 16 * (AD_D + 2) * 4; // (m, l, O) per warp and row
constexpr uint32_t AD_OFF_BAR = AD_OFF_MERGE + AD_MERGE_BYTES;
constexpr size_t AD_SMEM = AD_OFF_BAR + 2 * AD_STAGES * 8 + 16 + 1024;
constexpr float kLog2e = 1.4426950408889634f;

struct AdArgs {
  const __half *q;
  __half *y;
  int64_t q_sb, q_sh, y_sb, y_sh; // strides (elements) of Q / Y over batch and head
  int Hkv, group, L;
  int nc;          // 32-key chunks per (b, kv_head) pair
  int units, grid; // pairs * nc, CTAs
  float scale_log2; // scale * log2(e)
  float softcap;
  float *partials;  // [grid][2][16][D + 2] (O, m, l)
  uint32_t *counters;
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2,
                                        uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2,
                                          uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                    uint32_t a3, uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, "
      "{%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t *>(&h);
}
__device__ __forceinline__ void consumers_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(AD_WARPS * 32) : "memory");
}
__device__ __forceinline__ uint32_t atom_add_acq_rel(uint32_t *p, uint32_t v) {
  uint32_t old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
__device__ __forceinline__ int unit_begin(int c, int U, int G) {
  return (int)((int64_t)c * U / G);
}
__device__ __forceinline__ int cta_of(int u, int U, int G) {
  return (int)(((int64_t)(u + 1) * G - 1) / U);
}
// Shared-memory byte offset of 16-byte chunk `chunk` (0..7) of key row `key`
// in a [keys][128 B] tile written with the 128-byte swizzle.
__device__ __forceinline__ uint32_t swz(int key, int chunk) {
  return (uint32_t)(key * 128 + ((chunk ^ (key & 7)) << 4));
}

__global__ void __launch_bounds__(AD_THREADS, 1)
    attn_decode_mma(const __grid_constant__ CUtensorMap map_k,
                    const __grid_constant__ CUtensorMap map_v, const AdArgs g) {
  extern __shared__ uint8_t dsm[];
  uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(dsm) + 1023) & ~uintptr_t(1023));
  uint64_t *full = reinterpret_cast<uint64_t *>(sm + AD_OFF_BAR);
  uint64_t *empty = full + AD_STAGES;
  volatile int *flags = reinterpret_cast<volatile int *>(empty + AD_STAGES); // [0] abort [1] last
  float *mrg = reinterpret_cast<float *>(sm + AD_OFF_MERGE);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.x;
  const int u0 = unit_begin(b, g.units, g.grid), u1 = unit_begin(b + 1, g.units, g.grid);
  const int nun = u1 - u0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < AD_STAGES; ++i) {
      tc::mbar_init(&full[i], 1);
      tc::mbar_init(&empty[i], 1); // one consumer warp per stage
    }
    flags[0] = 0;
    flags[1] = 0;
    tc::fence_barrier_init();
  }
  __syncthreads();

  if (warp == AD_WARPS) {
    // ------------------------------ producer ------------------------------
    if (lane == 0) {
      tc::prefetch_tensormap(&map_k);
      tc::prefetch_tensormap(&map_v);
      for (int i = 0; i < nun; ++i) {
        const int s = i % AD_STAGES;
        if (i >= AD_STAGES && !tc::mbar_wait(&empty[s], ((i / AD_STAGES) - 1) & 1)) {
          atomicExch(&g_attn_decode_status, tc::kTimeoutEmpty);
          flags[0] = 1;
          break;
        }
        const int u = u0 + i, pair = u / g.nc, key0 = (u % g.nc) * AD_KEYS;
        uint8_t *st = sm + s * AD_STAGE;
        tc::mbar_expect_tx(&full[s], AD_STAGE);
        tc::tma_load_3d(st, &map_k, &full[s], 0, key0, pair);
        tc::tma_load_3d(st + AD_HALF, &map_k, &full[s], 64, key0, pair);
        tc::tma_load_3d(st + 2 * AD_HALF, &map_v, &full[s], 0, key0, pair);
        tc::tma_load_3d(st + 3 * AD_HALF, &map_v, &full[s], 64, key0, pair);
      }
    }
    return;
  }

  // ------------------------------ consumers -------------------------------
  const int gq = lane >> 2, t = lane & 3;
  const int mi = lane >> 3, mr = lane & 7; // ldmatrix: matrix / row this lane addresses
  bool ok = true;
  const int first_pair = u0 / g.nc;

  int seg0 = 0;
  while (seg0 < nun) {
    const int pair = (u0 + seg0) / g.nc;
    const int seg1 = min(nun, (pair + 1) * g.nc - u0);
    const int bb = pair / g.Hkv, kvh = pair % g.Hkv;

    // Q fragments of this group (rows >= group are zero): 8 k16 steps x 4 regs.
    uint32_t qa[8][4];
    {
      const __half *qb = g.q + (int64_t)bb * g.q_sb;
      const int r0 = gq, r1 = gq + 8;
      const __half *q0 = qb + (int64_t)(kvh * g.group + r0) * g.q_sh;
      const __half *q1 = qb + (int64_t)(kvh * g.group + r1) * g.q_sh;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const int d = kk * 16 + 2 * t;
        qa[kk][0] = r0 < g.group ? *reinterpret_cast<const uint32_t *>(q0 + d) : 0u;
        qa[kk][1] = r1 < g.group ? *reinterpret_cast<const uint32_t *>(q1 + d) : 0u;
        qa[kk][2] = r0 < g.group ? *reinterpret_cast<const uint32_t *>(q0 + d + 8) : 0u;
        qa[kk][3] = r1 < g.group ? *reinterpret_cast<const uint32_t *>(q1 + d + 8) : 0u;
      }
    }
    float o[16][4];
#pragma unroll
    for (int n = 0; n < 16; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) o[n][e] = 0.0f;
    float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.0f, 0.0f}; // rows gq, gq + 8

    for (int i = seg0 + ((warp - seg0 % AD_WARPS + AD_WARPS) % AD_WARPS); i < seg1; i += AD_WARPS) {
      const int s = i % AD_STAGES;
      if (ok && flags[0]) ok = false;
      if (ok && !tc::mbar_wait(&full[s], (i / AD_STAGES) & 1)) {
        atomicExch(&g_attn_decode_status, tc::kTimeoutFull);
        flags[0] = 1;
        ok = false;
      }
      if (ok) {
        const uint32_t kbase = tc::smem_u32(sm + s * AD_STAGE);
        const uint32_t vbase = kbase + 2 * AD_HALF;
        const int key0 = ((u0 + i) % g.nc) * AD_KEYS;
        // ---- S = Q . K^T for the 32 keys (4 n8 tiles) ----
        float sc[4][4];
#pragma unroll
        for (int n = 0; n < 4; ++n)
#pragma unroll
          for (int e = 0; e < 4; ++e) sc[n][e] = 0.0f;
#pragma unroll
        for (int kt = 0; kt < 2; ++kt) { // 16-key tiles
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) { // 16-dim steps
            // matrices: (keys 0-7, dims lo), (keys 0-7, dims hi), (keys 8-15, lo), (keys 8-15, hi)
            const int key = kt * 16 + (mi >> 1) * 8 + mr;
            const int dim = kk * 16 + (mi & 1) * 8;
            const uint32_t addr = kbase + (dim >= 64 ? AD_HALF : 0) + swz(key, (dim & 63) >> 3);
            uint32_t b0, b1, b2, b3;
            ldsm_x4(addr, b0, b1, b2, b3);
            mma(sc[2 * kt], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], b0, b1);
            mma(sc[2 * kt + 1], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], b2, b3);
          }
        }
        // ---- scale, softcap, mask, online softmax (base 2) ----
        float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
        for (int n = 0; n < 4; ++n)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int key = key0 + n * 8 + 2 * t + (e & 1);
            float v = sc[n][e];
            if (g.softcap > 0.0f) v = g.softcap * tanhf(v * g.scale_log2 / kLog2e / g.softcap) * kLog2e;
            else v *= g.scale_log2;
            if (key >= g.L) v = -INFINITY;
            sc[n][e] = v;
            mx[e >> 1] = fmaxf(mx[e >> 1], v);
          }
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
          mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
        }
        float corr[2], mnew[2];
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          mnew[r] = fmaxf(m_run[r], mx[r]);
          corr[r] = mnew[r] == -INFINITY ? 1.0f : exp2f(m_run[r] - mnew[r]);
          m_run[r] = mnew[r];
        }
        float ls[2] = {0.0f, 0.0f};
#pragma unroll
        for (int n = 0; n < 4; ++n)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float v = sc[n][e];
            const float pv = v == -INFINITY ? 0.0f : exp2f(v - mnew[e >> 1]);
            sc[n][e] = pv;
            ls[e >> 1] += pv;
          }
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          ls[r] += __shfl_xor_sync(0xffffffffu, ls[r], 1);
          ls[r] += __shfl_xor_sync(0xffffffffu, ls[r], 2);
          l_run[r] = l_run[r] * corr[r] + ls[r];
        }
#pragma unroll
        for (int n = 0; n < 16; ++n) {
          o[n][0] *= corr[0];
          o[n][1] *= corr[0];
          o[n][2] *= corr[1];
          o[n][3] *= corr[1];
        }
        // ---- O += P . V ----
#pragma unroll
        for (int kt = 0; kt < 2; ++kt) {
          const uint32_t pa0 = pack_h2(sc[2 * kt][0], sc[2 * kt][1]);
          const uint32_t pa1 = pack_h2(sc[2 * kt][2], sc[2 * kt][3]);
          const uint32_t pa2 = pack_h2(sc[2 * kt + 1][0], sc[2 * kt + 1][1]);
          const uint32_t pa3 = pack_h2(sc[2 * kt + 1][2], sc[2 * kt + 1][3]);
#pragma unroll
          for (int nd = 0; nd < 8; ++nd) { // pairs of 8-dim tiles
            // matrices: (keys 0-7, dims n0), (keys 8-15, dims n0), (keys 0-7, n0+8), (keys 8-15, n0+8)
            const int key = kt * 16 + (mi & 1) * 8 + mr;
            const int dim = nd * 16 + (mi >> 1) * 8;
            const uint32_t addr = vbase + (dim >= 64 ? AD_HALF : 0) + swz(key, (dim & 63) >> 3);
            uint32_t b0, b1, b2, b3;
            ldsm_x4_t(addr, b0, b1, b2, b3);
            mma(o[2 * nd], pa0, pa1, pa2, pa3, b0, b1);
            mma(o[2 * nd + 1], pa0, pa1, pa2, pa3, b2, b3);
          }
        }
      }
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&empty[s]);
    }

    // ---------------- end of a (b, kv_head) segment: merge the 4 warps ----------------
    consumers_sync(); // the merge buffer is free (previous segment done)
    {
      float *mw = mrg + (size_t)warp * 16 * (AD_D + 2);
#pragma unroll
      for (int n = 0; n < 16; ++n) {
        const int d = n * 8 + 2 * t;
        mw[gq * (AD_D + 2) + d] = o[n][0];
        mw[gq * (AD_D + 2) + d + 1] = o[n][1];
        mw[(gq + 8) * (AD_D + 2) + d] = o[n][2];
        mw[(gq + 8) * (AD_D + 2) + d + 1] = o[n][3];
      }
      if (t == 0) {
        mw[gq * (AD_D + 2) + AD_D] = m_run[0];
        mw[gq * (AD_D + 2) + AD_D + 1] = l_run[0];
        mw[(gq + 8) * (AD_D + 2) + AD_D] = m_run[1];
        mw[(gq + 8) * (AD_D + 2) + AD_D + 1] = l_run[1];
      }
    }
    consumers_sync();
    const int pf = pair * g.nc, pl = pf + g.nc - 1;
    const int cf = cta_of(pf, g.units, g.grid), cl = cta_of(pl, g.units, g.grid);
    const bool whole = cf == cl;
    const int slot = pair == first_pair ? 0 : 1;
    float *part = g.partials + ((size_t)b * 2 + slot) * 16 * (AD_D + 2);
    for (int e = threadIdx.x; e < g.group * AD_D; e += AD_WARPS * 32) {
      const int r = e / AD_D, d = e % AD_D;
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < AD_WARPS; ++w) M = fmaxf(M, mrg[((size_t)w * 16 + r) * (AD_D + 2) + AD_D]);
      float l = 0.0f, acc = 0.0f;
#pragma unroll
      for (int w = 0; w < AD_WARPS; ++w) {
        const float* row = mrg + ((size_t)w * 16 + r) * (AD_D + 2);
        const float c = row[AD_D] == -INFINITY ? 0.0f : exp2f(row[AD_D] - M);
        l += row[AD_D + 1] * c;
        acc += row[d] * c;
      }
      if (whole) {
        if (ok)
          g.y[(int64_t)bb * g.y_sb + (int64_t)(kvh * g.group + r) * g.y_sh + d] =
              __float2half_rn(l > 0.0f ? acc / l : 0.0f);
      } else {
        part[r * (AD_D + 2) + d] = acc;
        if (d == 0) {
          part[r * (AD_D + 2) + AD_D] = M;
          part[r * (AD_D + 2) + AD_D + 1] = l;
        }
      }
    }
    if (!whole) {
      consumers_sync();
      if (threadIdx.x == 0) {
        // A CTA whose wait gave up arrives with kAbortMark, and then the last
        // one does not merge (the partials are not all valid).
        const uint32_t inc = flags[0] ? kAbortMark + 1u : 1u;
        const uint32_t now = atom_add_acq_rel(g.counters + pair, inc) + inc;
        const bool last = (now & (kAbortMark - 1u)) == (uint32_t)(cl - cf + 1);
        if (last) g.counters[pair] = 0u;
        flags[1] = last && (now >> 16) == 0u ? 1 : 0;
      }
      consumers_sync();
      if (flags[1] && ok) {
        // Last CTA on this pair: merge the contributors' partials in CTA order.
        for (int e = threadIdx.x; e < g.group * AD_D; e += AD_WARPS * 32) {
          const int r = e / AD_D, d = e % AD_D;
          float M = -INFINITY;
          for (int c = cf; c <= cl; ++c) {
            const int cs = unit_begin(c, g.units, g.grid) / g.nc == pair ? 0 : 1;
            M = fmaxf(M, __ldcg(g.partials + (((size_t)c * 2 + cs) * 16 + r) * (AD_D + 2) + AD_D));
          }
          float l = 0.0f, acc = 0.0f;
          for (int c = cf; c <= cl; ++c) {
            const int cs = unit_begin(c, g.units, g.grid) / g.nc == pair ? 0 : 1;
            const float *row = g.partials + (((size_t)c * 2 + cs) * 16 + r) * (AD_D + 2);
            const float mc = __ldcg(row + AD_D);
            const float cw = mc == -INFINITY ? 0.0f : exp2f(mc - M);
            l += __ldcg(row + AD_D + 1) * cw;
            acc += __ldcg(row + d) * cw;
          }
          g.y[(int64_t)bb * g.y_sb + (int64_t)(kvh * g.group + r) * g.y_sh + d] =
              __float2half_rn(l > 0.0f ? acc / l : 0.0f);
        }
      }
    }
    seg0 = seg1;
  }
}

} // namespace

// Eligible: FLOAT16, head size 128, one query token, GQA group <= 16, no mask,
// no sliding window, every key visible (not causal, or causal with the query
// at the last position: one new token), K / V rows contiguous
// [B, Hkv, rows, 128] with b-stride = Hkv * head-stride.
bool attn_decode_eligible(int dtype, int64_t D, int64_t Sq, int64_t group, bool mask,
                          int64_t left_window, int64_t right_window, int64_t k_sb, int64_t k_sh,
                          int64_t k_ss, int64_t Hkv, int64_t L, bool causal, int64_t new_tokens) {
  if (causal && new_tokens != 1) return false;
  return dtype == kFloat16 && D == AD_D && Sq == 1 && group >= 1 && group <= 16 && !mask &&
         left_window < 0 && right_window < 0 && k_ss == D && k_sb == Hkv * k_sh && L >= 1 &&
         L < (int64_t)1 << 30 && k_sh % 8 == 0;
}

size_t attn_decode_workspace(int64_t B, int64_t Hkv) {
  (void)B;
  (void)Hkv;
  return kCounterBytes + (size_t)sm_count() * 2 * 16 * (AD_D + 2) * 4;
}

int attn_decode_launch(const void *q, int64_t q_sb, int64_t q_sh, const void *kc, const void *vc,
                       int64_t kv_sh, int64_t B, int64_t Hkv, int64_t group, int64_t L, float scale,
                       float softcap, void *y, int64_t y_sb, int64_t y_sh, void *ws,
                       cudaStream_t st) {
  const int64_t pairs = B * Hkv;
  if (pairs > (int64_t)kMaxCounters)
    B2_FAIL(B2_ERR_UNSUPPORTED, "b2_attention: too many (batch, kv_head) pairs for the decode kernel");
  CUtensorMap map_k, map_v;
  // [B*Hkv][rows][128] fp16: dims {128, L, pairs}, strides {row 256 B, pair kv_sh * 2 B}
  const uint64_t dims[3] = {(uint64_t)AD_D, (uint64_t)L, (uint64_t)pairs};
  const uint64_t strides[2] = {(uint64_t)AD_D * 2, (uint64_t)kv_sh * 2};
  const uint32_t box[3] = {64, (uint32_t)AD_KEYS, 1};
  int rc = make_tensor_map(&map_k, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, kc, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = make_tensor_map(&map_v, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, vc, dims, strides, box,
                       CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  AdArgs a{};
  a.q = static_cast<const __half *>(q);
  a.y = static_cast<__half *>(y);
  a.q_sb = q_sb;
  a.q_sh = q_sh;
  a.y_sb = y_sb;
  a.y_sh = y_sh;
  a.Hkv = (int)Hkv;
  a.group = (int)group;
  a.L = (int)L;
  a.nc = (int)((L + AD_KEYS - 1) / AD_KEYS);
  const int64_t units = pairs * a.nc;
  if (units >= ((int64_t)1 << 31) / 2) B2_FAIL(B2_ERR_UNSUPPORTED, "b2_attention: KV cache too long");
  a.units = (int)units;
  a.grid = (int)std::min<int64_t>(units, sm_count());
  a.scale_log2 = scale * kLog2e;
  a.softcap = softcap;
  a.counters = static_cast<uint32_t *>(ws);
  a.partials = reinterpret_cast<float *>(static_cast<uint8_t *>(ws) + kCounterBytes);
  B2_CUDA(cudaFuncSetAttribute(attn_decode_mma, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)AD_SMEM));
  attn_decode_mma<<<a.grid, AD_THREADS, AD_SMEM, st>>>(map_k, map_v, a);
  B2_LAUNCH_CHECK();
  return B2_OK;
}

} // namespace b2

namespace b2 {
// Host: the time-out code this file's kernels recorded (0: none); reset != 0
// clears it.  Synchronous (the copy waits for the device).
int status_read_attn_decode(int reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_attn_decode_status, sizeof(int)) != cudaSuccess) return -1;
  if (reset && v) {
    const int z = 0;
    if (cudaMemcpyToSymbol(g_attn_decode_status, &z, sizeof(int)) != cudaSuccess) return -1;
  }
  return v;
}
} // namespace b2
