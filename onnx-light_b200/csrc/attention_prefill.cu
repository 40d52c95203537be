// Prefill Attention (many query tokens) on tensor cores: FlashAttention-style
// forward for FLOAT16 / BFLOAT16, head size 128, GQA, optional causal mask and
// softcap.
//
// Reference: kernel::Attention::operator() / ComputeAttentionRank4
// (onnx_light/onnx_extensions/kernels/kernels/nn/kernel_attention.cc:427-691,
// 767-852): per query row i (absolute position past_len + i) and key j,
// score = q . k * scale, softcap, causal mask j <= past_len + i, softmax with
// max subtraction, y = softmax . V -- in fp32 after promoting the inputs.
//
// One CTA owns 64 query rows of one query head (4 warps x 16 rows) and walks
// the key range in tiles of 64 (only up to the diagonal when causal):
//   S[16 x 64] = Q[16 x 128] . K^T   (mma.sync m16n8k16, fp32 accumulation)
//   online softmax of S in fp32 registers (base 2, running max / sum)
//   O[16 x 128] += P[16 x 64] . V    (P rounded to FLOAT16, or to BFLOAT16
//                                     plus its BFLOAT16 remainder)
// K and V tiles ([64 keys][128 dims], two 64-dim halves with the 128-byte
// swizzle, 32 KB per tile) arrive by TMA through a 2-stage ring; a 4-D tensor
// map {dim, key, kv_head, batch} reads both the rank-4 [B, H, S, D] and the
// rank-3 [B, S, H*D] layouts without a repack.  Keys past the valid length
// read as zeros and are masked.  P is the only value rounded on the way
// (2^-11 relative for fp16; about 2^-17 for bf16 with the remainder term).
#include <type_traits>

#include "b2_common.cuh"
#include "tc_common.cuh"

namespace b2 {

__device__ int g_attn_prefill_status;

namespace {

constexpr int AP_D = 128;
constexpr int AP_QROWS = 64;          // query rows per CTA (4 warps x 16)
constexpr int AP_KEYS = 64;           // keys per tile
constexpr int AP_WARPS = 4;
constexpr int AP_THREADS = AP_WARPS * 32;
#ifndef AP_STAGES_N
#define AP_STAGES_N 2
#endif
#ifndef AP_MINB
#define AP_MINB 3 // CTAs per SM
#endif
constexpr int AP_STAGES = AP_STAGES_N;
constexpr uint32_t AP_HALF = AP_KEYS * 128;       // one 64-dim half of K or V: 8 KB
constexpr uint32_t AP_STAGE = 4 * AP_HALF;        // K lo, K hi, V lo, V hi: 32 KB
constexpr uint32_t AP_OFF_BAR = AP_STAGES * AP_STAGE;
constexpr size_t AP_SMEM = AP_OFF_BAR + 2 * AP_STAGES * 8 + 1024;
constexpr float kLog2e = 1.4426950408889634f;

struct ApArgs {
  const void *q;
  void *y;
  int64_t q_sb, q_sh, q_ss; // strides (elements) of Q and Y
  int64_t y_sb, y_sh, y_ss;
  int Hq, Hkv, group, Sq, L, past;
  int qtiles;
  float scale_log2;
  float softcap;
  int causal;
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
template <typename T>
__device__ __forceinline__ void mma(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                    uint32_t a3, uint32_t b0, uint32_t b1) {
  if constexpr (std::is_same<T, __half>::value)
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, "
        "{%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  else
    asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, "
        "{%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
template <typename T> __device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if constexpr (std::is_same<T, __half>::value) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t *>(&h);
  } else {
    const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t *>(&h);
  }
}
__device__ __forceinline__ uint32_t swz(int key, int chunk) {
  return (uint32_t)(key * 128 + ((chunk ^ (key & 7)) << 4));
}

template <typename T>
__global__ void __launch_bounds__(AP_THREADS, AP_MINB)
    attn_prefill_mma(const __grid_constant__ CUtensorMap map_k,
                     const __grid_constant__ CUtensorMap map_v, const ApArgs g) {
  extern __shared__ uint8_t dsm[];
  uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(dsm) + 1023) & ~uintptr_t(1023));
  uint64_t *full = reinterpret_cast<uint64_t *>(sm + AP_OFF_BAR);
  uint64_t *empty = full + AP_STAGES;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gq = lane >> 2, t = lane & 3;
  const int mi = lane >> 3, mr = lane & 7;
  // heavy (late, causal) query tiles first
  const int qt = g.qtiles - 1 - (int)(blockIdx.x % g.qtiles);
  const int bh = (int)(blockIdx.x / g.qtiles);
  const int b = bh / g.Hq, h = bh % g.Hq, kvh = h / g.group;
  const int q0 = qt * AP_QROWS;
  const int wq0 = q0 + warp * 16; // this warp's first query row
  // keys this CTA needs: [0, kend)
  const int kend = g.causal ? min(g.L, g.past + q0 + AP_QROWS) : g.L;
  const int ntiles = (kend + AP_KEYS - 1) / AP_KEYS;

  if (threadIdx.x == 0) {
    for (int i = 0; i < AP_STAGES; ++i) {
      tc::mbar_init(&full[i], 1);
      tc::mbar_init(&empty[i], AP_WARPS);
    }
    tc::fence_barrier_init();
  }
  __syncthreads();
  auto issue = [&](int j) {
    const int s = j % AP_STAGES;
    uint8_t *st = sm + s * AP_STAGE;
    tc::mbar_expect_tx(&full[s], AP_STAGE);
    const int key0 = j * AP_KEYS;
    tc::tma_load_4d(st, &map_k, &full[s], 0, key0, kvh, b);
    tc::tma_load_4d(st + AP_HALF, &map_k, &full[s], 64, key0, kvh, b);
    tc::tma_load_4d(st + 2 * AP_HALF, &map_v, &full[s], 0, key0, kvh, b);
    tc::tma_load_4d(st + 3 * AP_HALF, &map_v, &full[s], 64, key0, kvh, b);
  };
  if (threadIdx.x == 0) {
    tc::prefetch_tensormap(&map_k);
    tc::prefetch_tensormap(&map_v);
    for (int j = 0; j < min(ntiles, AP_STAGES); ++j) issue(j);
  }

  // Q fragments of the warp's 16 rows (rows past Sq are zero).
  uint32_t qa[8][4];
  {
    const T *qb = static_cast<const T *>(g.q) + (int64_t)b * g.q_sb + (int64_t)h * g.q_sh;
    const int r0 = wq0 + gq, r1 = wq0 + gq + 8;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const int d = kk * 16 + 2 * t;
      qa[kk][0] = r0 < g.Sq ? *reinterpret_cast<const uint32_t *>(qb + (int64_t)r0 * g.q_ss + d) : 0u;
      qa[kk][1] = r1 < g.Sq ? *reinterpret_cast<const uint32_t *>(qb + (int64_t)r1 * g.q_ss + d) : 0u;
      qa[kk][2] = r0 < g.Sq ? *reinterpret_cast<const uint32_t *>(qb + (int64_t)r0 * g.q_ss + d + 8) : 0u;
      qa[kk][3] = r1 < g.Sq ? *reinterpret_cast<const uint32_t *>(qb + (int64_t)r1 * g.q_ss + d + 8) : 0u;
    }
  }
  float o[16][4];
#pragma unroll
  for (int n = 0; n < 16; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[n][e] = 0.0f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.0f, 0.0f};
  // absolute positions of the lane's two rows (for the causal mask)
  const int pos0 = g.past + wq0 + gq, pos1 = pos0 + 8;
  // keys this warp can see: up to its last row
  const int wkend = g.causal ? min(kend, g.past + wq0 + 16) : kend;
  bool ok = true;

  for (int j = 0; j < ntiles; ++j) {
    const int s = j % AP_STAGES;
    if (ok && !tc::mbar_wait(&full[s], (j / AP_STAGES) & 1)) {
      atomicExch(&g_attn_prefill_status, tc::kTimeoutFull);
      ok = false;
    }
    const int key0 = j * AP_KEYS;
    if (ok && key0 < wkend) {
      const uint32_t kbase = tc::smem_u32(sm + s * AP_STAGE);
      const uint32_t vbase = kbase + 2 * AP_HALF;
      float sc[8][4];
#pragma unroll
      for (int n = 0; n < 8; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) sc[n][e] = 0.0f;
#pragma unroll
      for (int kt = 0; kt < 4; ++kt) {
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const int key = kt * 16 + (mi >> 1) * 8 + mr;
          const int dim = kk * 16 + (mi & 1) * 8;
          uint32_t b0, b1, b2, b3;
          ldsm_x4(kbase + (dim >= 64 ? AP_HALF : 0) + swz(key, (dim & 63) >> 3), b0, b1, b2, b3);
          mma<T>(sc[2 * kt], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], b0, b1);
          mma<T>(sc[2 * kt + 1], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], b2, b3);
        }
      }
      // scale, softcap, mask, online softmax (base 2)
      const bool need_mask = key0 + AP_KEYS > g.L || (g.causal && key0 + AP_KEYS - 1 > pos0);
      float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
      for (int n = 0; n < 8; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float v = sc[n][e];
          if (g.softcap > 0.0f) v = g.softcap * tanhf(v * g.scale_log2 / kLog2e / g.softcap) * kLog2e;
          else v *= g.scale_log2;
          if (need_mask) {
            const int key = key0 + n * 8 + 2 * t + (e & 1);
            const int pos = (e >> 1) ? pos1 : pos0;
            if (key >= g.L || (g.causal && key > pos)) v = -INFINITY;
          }
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
      for (int n = 0; n < 8; ++n)
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
      // O += P . V
#pragma unroll
      for (int kt = 0; kt < 4; ++kt) {
        const uint32_t pa0 = pack2<T>(sc[2 * kt][0], sc[2 * kt][1]);
        const uint32_t pa1 = pack2<T>(sc[2 * kt][2], sc[2 * kt][3]);
        const uint32_t pa2 = pack2<T>(sc[2 * kt + 1][0], sc[2 * kt + 1][1]);
        const uint32_t pa3 = pack2<T>(sc[2 * kt + 1][2], sc[2 * kt + 1][3]);
        // BFLOAT16: the remainder p - bf16(p) as a second operand, so P
        // carries 16 significant bits (as in the tcgen05 kernel)
        constexpr bool kSplit = !std::is_same<T, __half>::value;
        uint32_t pl0 = 0, pl1 = 0, pl2 = 0, pl3 = 0;
        if constexpr (kSplit) {
          auto rem = [](uint32_t hi, float lo_v, float hi_v) {
            return pack2<T>(lo_v - __uint_as_float(hi << 16), hi_v - __uint_as_float(hi & 0xffff0000u));
          };
          pl0 = rem(pa0, sc[2 * kt][0], sc[2 * kt][1]);
          pl1 = rem(pa1, sc[2 * kt][2], sc[2 * kt][3]);
          pl2 = rem(pa2, sc[2 * kt + 1][0], sc[2 * kt + 1][1]);
          pl3 = rem(pa3, sc[2 * kt + 1][2], sc[2 * kt + 1][3]);
        }
#pragma unroll
        for (int nd = 0; nd < 8; ++nd) {
          const int key = kt * 16 + (mi & 1) * 8 + mr;
          const int dim = nd * 16 + (mi >> 1) * 8;
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(vbase + (dim >= 64 ? AP_HALF : 0) + swz(key, (dim & 63) >> 3), b0, b1, b2, b3);
          mma<T>(o[2 * nd], pa0, pa1, pa2, pa3, b0, b1);
          mma<T>(o[2 * nd + 1], pa0, pa1, pa2, pa3, b2, b3);
          if constexpr (kSplit) {
            mma<T>(o[2 * nd], pl0, pl1, pl2, pl3, b0, b1);
            mma<T>(o[2 * nd + 1], pl0, pl1, pl2, pl3, b2, b3);
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) tc::mbar_arrive(&empty[s]);
    // refill this stage with tile j + STAGES once every warp released it
    if (threadIdx.x == 0 && j + AP_STAGES < ntiles) {
      if (tc::mbar_wait(&empty[s], (j / AP_STAGES) & 1)) issue(j + AP_STAGES);
      else {
        atomicExch(&g_attn_prefill_status, tc::kTimeoutEmpty);
        ok = false;
      }
    }
    __syncwarp();
  }

  // y = O / l
  if (ok) {
    T *yb = static_cast<T *>(g.y) + (int64_t)b * g.y_sb + (int64_t)h * g.y_sh;
    const int r0 = wq0 + gq, r1 = r0 + 8;
    const float inv0 = l_run[0] > 0.0f ? 1.0f / l_run[0] : 0.0f;
    const float inv1 = l_run[1] > 0.0f ? 1.0f / l_run[1] : 0.0f;
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      const int d = n * 8 + 2 * t;
      if (r0 < g.Sq) {
        T *p = yb + (int64_t)r0 * g.y_ss + d;
        *reinterpret_cast<uint32_t *>(p) = pack2<T>(o[n][0] * inv0, o[n][1] * inv0);
      }
      if (r1 < g.Sq) {
        T *p = yb + (int64_t)r1 * g.y_ss + d;
        *reinterpret_cast<uint32_t *>(p) = pack2<T>(o[n][2] * inv1, o[n][3] * inv1);
      }
    }
  }
}

} // namespace

// Eligible: FLOAT16 / BFLOAT16, head size 128, no mask, no sliding window,
// K / V rows of 128 contiguous elements (rank-4 or rank-3 layouts).
bool attn_prefill_eligible(int dtype, int64_t D, int64_t Sq, bool mask, int64_t left_window,
                           int64_t right_window, int64_t k_ss, int64_t L) {
  return (dtype == kFloat16 || dtype == kBfloat16) && D == AP_D && Sq >= 2 && !mask &&
         left_window < 0 && right_window < 0 && k_ss % 8 == 0 && L >= 1 &&
         L < ((int64_t)1 << 30) && Sq < ((int64_t)1 << 30);
}

size_t attn_prefill_smem() { return AP_SMEM; }

int attn_prefill_launch(int dtype, const void *q, const int64_t *qs, const void *kc,
                        const void *vc, const int64_t *ks, void *y, const int64_t *ys, int64_t B,
                        int64_t Hq, int64_t Hkv, int64_t Sq, int64_t L, int64_t past, float scale,
                        float softcap, int causal, cudaStream_t st) {
  // K / V as 4-D {dim, key, kv_head, batch}; ks = element strides {batch, head, key}
  CUtensorMap map_k, map_v;
  const uint64_t dims[4] = {(uint64_t)AP_D, (uint64_t)L, (uint64_t)Hkv, (uint64_t)B};
  const uint64_t strides[3] = {(uint64_t)ks[2] * 2, (uint64_t)ks[1] * 2, (uint64_t)ks[0] * 2};
  const uint32_t box[4] = {64, (uint32_t)AP_KEYS, 1, 1};
  const CUtensorMapDataType tdt =
      dtype == kFloat16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  int rc = make_tensor_map(&map_k, tdt, 4, kc, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = make_tensor_map(&map_v, tdt, 4, vc, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  ApArgs a{};
  a.q = q;
  a.y = y;
  a.q_sb = qs[0];
  a.q_sh = qs[1];
  a.q_ss = qs[2];
  a.y_sb = ys[0];
  a.y_sh = ys[1];
  a.y_ss = ys[2];
  a.Hq = (int)Hq;
  a.Hkv = (int)Hkv;
  a.group = (int)(Hq / Hkv);
  a.Sq = (int)Sq;
  a.L = (int)L;
  a.past = (int)past;
  a.qtiles = (int)((Sq + AP_QROWS - 1) / AP_QROWS);
  a.scale_log2 = scale * kLog2e;
  a.softcap = softcap;
  a.causal = causal;
  const int64_t ctas = (int64_t)a.qtiles * B * Hq;
  if (ctas >= ((int64_t)1 << 31)) B2_FAIL(B2_ERR_UNSUPPORTED, "b2_attention: too many query tiles");
  auto kern = dtype == kFloat16 ? attn_prefill_mma<__half> : attn_prefill_mma<__nv_bfloat16>;
  B2_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)AP_SMEM));
  kern<<<(unsigned)ctas, AP_THREADS, AP_SMEM, st>>>(map_k, map_v, a);
  B2_LAUNCH_CHECK();
  return B2_OK;
}

} // namespace b2

namespace b2 {
// Host: the time-out code this file's kernels recorded (0: none); reset != 0
// clears it.  Synchronous (the copy waits for the device).
int status_read_attn_prefill(int reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_attn_prefill_status, sizeof(int)) != cudaSuccess) return -1;
  if (reset && v) {
    const int z = 0;
    if (cudaMemcpyToSymbol(g_attn_prefill_status, &z, sizeof(int)) != cudaSuccess) return -1;
  }
  return v;
}
} // namespace b2
