// Opset-23 Attention with GQA and a contiguous KV cache on sm_100a.
//
// Replaces kernel::Attention::operator() and ComputeAttentionRank4
// (onnx_light/onnx_extensions/kernels/kernels/nn/kernel_attention.cc:427-691, 767-852).
//
// Data layout in HBM
//  * KV cache: one buffer per K and V, [B, Hkv, capacity, D], the layout the
//    reference's persistent append uses (kernel_attention.cc:297-310).  New
//    tokens are appended in place by kv_append; with kv_capacity == 0 the
//    present buffers are fresh [B, Hkv, past+new, D] tensors and the past is
//    copied in first (the reference's ConcatAxis2 repack, :313-339).
//  * Q / Y: rank-4 [B, H, S, D] or rank-3 [B, S, H*D], read and written through
//    strides, so rank-3 inputs need no transpose pass (the reference repacks
//    them, :179-248).
//
// attn_fwd: split-KV flash attention on CUDA cores.  One CTA owns one
// (batch, kv_head) pair, up to 16 query rows of that group (the Hq/Hkv query
// heads of a GQA group share every K/V byte read, :587) and a contiguous
// range of keys.  K/V tiles of 32 keys stream through shared memory with
// cp.async double buffering; each lane scores one key against all rows
// (fp32), the online softmax (running max / sum) is kept per row, and for
// P.V each lane owns D/32 output dims.  Splits write (m, l, o) partials; the
// last CTA of a (b, kv_head, row-tile) merges them in split order.
// The decode configuration is HBM-bound: bytes = K and V cache + Q + Y.
#include "b2_common.cuh"

namespace b2 {

// Tensor-core decode kernel (attention_decode.cu).
bool attn_decode_eligible(int dtype, int64_t D, int64_t Sq, int64_t group, bool mask,
                          int64_t left_window, int64_t right_window, int64_t k_sb, int64_t k_sh,
                          int64_t k_ss, int64_t Hkv, int64_t L, bool causal, int64_t new_tokens);
size_t attn_decode_workspace(int64_t B, int64_t Hkv);
// Tensor-core prefill kernel (attention_prefill.cu).
bool attn_prefill_eligible(int dtype, int64_t D, int64_t Sq, bool mask, int64_t left_window,
                           int64_t right_window, int64_t k_ss, int64_t L);
bool attn_prefill_tc_eligible(int dtype, int64_t D, int64_t Sq, bool mask, int64_t left_window,
                              int64_t right_window, const int64_t *qs, const int64_t *ks,
                              const int64_t *ys, int64_t L);
int attn_prefill_tc_launch(int dtype, const void *q, const int64_t *qs, const void *kc,
                           const void *vc, const int64_t *ks, void *y, const int64_t *ys,
                           int64_t B, int64_t Hq, int64_t Hkv, int64_t Sq, int64_t L, int64_t past,
                           float scale, float softcap, int causal, cudaStream_t st);
int attn_prefill_launch(int dtype, const void *q, const int64_t *qs, const void *kc,
                        const void *vc, const int64_t *ks, void *y, const int64_t *ys, int64_t B,
                        int64_t Hq, int64_t Hkv, int64_t Sq, int64_t L, int64_t past, float scale,
                        float softcap, int causal, cudaStream_t st);
int attn_decode_launch(const void *q, int64_t q_sb, int64_t q_sh, const void *kc, const void *vc,
                       int64_t kv_sh, int64_t B, int64_t Hkv, int64_t group, int64_t L, float scale,
                       float softcap, void *y, int64_t y_sb, int64_t y_sh, void *ws,
                       cudaStream_t st);

constexpr int ATT_THREADS = 128; // 4 warps
constexpr int ATT_ROWS = 16;     // query rows per CTA
constexpr int ATT_TK = 32;       // keys per tile (one per lane)
constexpr int ATT_DMAX = 256; // largest head size handled

struct AttParams {
  const void *q;
  const void *k; // present / key view
  const void *v;
  void *y;
  const void *mask;         // FLOAT, BOOL, FLOAT16 or BFLOAT16 (mask_dt)
  int mask_dt;
  int64_t mask_shape[4];
  const int64_t *nonpad;    // nonpad_kv_seqlen [B] or nullptr
  int64_t B, Hq, Hkv, Sq, L, D, Dv; // Dv: V head size (may differ from D)
  int64_t q_sb, q_sh, q_ss; // strides (elements)
  int64_t k_sb, k_sh, k_ss;
  int64_t v_sb, v_sh, v_ss;
  int64_t y_sb, y_sh, y_ss;
  int64_t past_len;
  float scale, softcap;
  int causal;
  int64_t left_window, right_window;
  int group;      // Hq / Hkv
  int rows_total; // group * Sq
  int row_tiles;
  int splits;
  int64_t keys_per_split;
  float *ws_o;    // [splits][B*Hkv*rows_total][D]
  float *ws_ml;   // [splits][B*Hkv*rows_total][2]
  uint32_t *counters;
  int dt;
};

template <typename T> __device__ __forceinline__ float ld_act(const void *p, int64_t i);
template <> __device__ __forceinline__ float ld_act<float>(const void *p, int64_t i) {
  return reinterpret_cast<const float *>(p)[i];
}
template <> __device__ __forceinline__ float ld_act<__half>(const void *p, int64_t i) {
  return __half2float(reinterpret_cast<const __half *>(p)[i]);
}
template <> __device__ __forceinline__ float ld_act<__nv_bfloat16>(const void *p, int64_t i) {
  return __uint_as_float((uint32_t)reinterpret_cast<const uint16_t *>(p)[i] << 16);
}
template <typename T> __device__ __forceinline__ void st_act(void *p, int64_t i, float v);
template <> __device__ __forceinline__ void st_act<float>(void *p, int64_t i, float v) {
  reinterpret_cast<float *>(p)[i] = v;
}
template <> __device__ __forceinline__ void st_act<__half>(void *p, int64_t i, float v) {
  reinterpret_cast<uint16_t *>(p)[i] = f32_to_f16_bits(v);
}
template <> __device__ __forceinline__ void st_act<__nv_bfloat16>(void *p, int64_t i, float v) {
  reinterpret_cast<uint16_t *>(p)[i] = f32_to_bf16_bits(v);
}

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
  const uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;"); }
template <int N> __device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N));
}

// Mask value of a FLOAT, BOOL (true keeps, false masks), FLOAT16 or BFLOAT16
// mask element (BroadcastedMaskValue, kernel_attention.cc:371-394; the half
// types are promoted to FLOAT as the half-precision entry does, :797-801).
__device__ __forceinline__ float mask_elem(const void *m, int dt, int64_t i) {
  switch (dt) {
  case kBool: return reinterpret_cast<const uint8_t *>(m)[i] != 0 ? 0.0f : -INFINITY;
  case kFloat16: return f16_bits_to_f32(reinterpret_cast<const uint16_t *>(m)[i]);
  case kBfloat16: return __uint_as_float((uint32_t)reinterpret_cast<const uint16_t *>(m)[i] << 16);
  default: return reinterpret_cast<const float *>(m)[i];
  }
}

// Number of valid keys that precede the query block of batch b: the past
// length, or nonpad_kv_seqlen[b] - Sq without a past (kernel_attention.cc:572-582).
__device__ __forceinline__ int64_t causal_offset(const AttParams &p, int64_t b) {
  return (p.nonpad != nullptr && p.past_len == 0) ? p.nonpad[b] - p.Sq : p.past_len;
}

// Mask bias of (b, h, i, j) (kernel_attention.cc:398-410, 592-602): the mask
// (positions past its last axis masked), the causal frontier, the windows and
// the nonpad_kv_seqlen padding.
__device__ __forceinline__ float att_bias(const AttParams &p, int64_t b, int64_t h, int64_t i,
                                          int64_t j) {
  float bias = 0.0f;
  if (p.mask) {
    if (j >= p.mask_shape[3]) {
      bias = -INFINITY;
    } else {
      const int64_t idx[4] = {b, h, i, j};
      int64_t lin = 0, st = 1;
#pragma unroll
      for (int k = 3; k >= 0; --k) {
        lin += (p.mask_shape[k] == 1 ? 0 : idx[k]) * st;
        st *= p.mask_shape[k];
      }
      bias = mask_elem(p.mask, p.mask_dt, lin);
    }
  }
  const int64_t off = causal_offset(p, b);
  if (p.causal && j > i + off) bias = -INFINITY;
  const int64_t wd = i + off - j;
  if ((p.left_window >= 0 && wd > p.left_window) || (p.right_window >= 0 && -wd > p.right_window))
    bias = -INFINITY;
  if (p.nonpad != nullptr && j >= p.nonpad[b]) bias = -INFINITY;
  return bias;
}

template <typename T, int ROWS, int DPL>
__global__ void __launch_bounds__(ATT_THREADS) attn_fwd(const AttParams p) {
  extern __shared__ __align__(16) uint8_t att_smem[];
  const int D = (int)p.D, Dv = (int)p.Dv;
  const int DP = D + 8, DPv = Dv + 8; // padded rows (elements) to spread shared-memory banks
  T *ks = reinterpret_cast<T *>(att_smem);                  // [2][4 warps][32][DP]
  T *vs = ks + 2 * 4 * ATT_TK * DP;                         // [2][4][32][DPv]
  float *qs = reinterpret_cast<float *>(vs + 2 * 4 * ATT_TK * DPv); // [ROWS][D]
  float *ps = qs + ROWS * D;                            // [4 warps][ROWS][32]
  float *red = ps + 4 * ROWS * ATT_TK;                  // merge buffer

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int bh = blockIdx.x;
  const int64_t b = bh / p.Hkv, kvh = bh % p.Hkv;
  const int rt = blockIdx.z;
  const int split = blockIdx.y;
  const int row0 = rt * ROWS;
  const int nrows = min(ROWS, p.rows_total - row0);

  // Query rows: row r -> (head = kvh*group + r % group, query index r / group).
  for (int e = threadIdx.x; e < ROWS * D; e += ATT_THREADS) {
    const int r = e / D, d = e % D;
    float val = 0.0f;
    if (r < nrows) {
      const int rr = row0 + r;
      const int64_t h = kvh * p.group + rr % p.group, s = rr / p.group;
      val = ld_act<T>(p.q, b * p.q_sb + h * p.q_sh + s * p.q_ss + d);
    }
    qs[e] = val;
  }

  const int64_t kbeg = (int64_t)split * p.keys_per_split;
  const int64_t kend = min(p.L, kbeg + p.keys_per_split);
  // Each warp walks its own interleaved sequence of 32-key tiles.
  const int64_t ntiles = (kend - kbeg + ATT_TK - 1) / ATT_TK;
  const T *kbase = reinterpret_cast<const T *>(p.k) + b * p.k_sb + kvh * p.k_sh;
  const T *vbase = reinterpret_cast<const T *>(p.v) + b * p.v_sb + kvh * p.v_sh;
  const int chunks = D * (int)sizeof(T) / 16;   // 16-byte chunks per K row
  const int chunks_v = Dv * (int)sizeof(T) / 16; // and per V row

  auto issue = [&](int64_t tile, int buf) {
    T *kd = ks + (buf * 4 + warp) * ATT_TK * DP;
    T *vd = vs + (buf * 4 + warp) * ATT_TK * DPv;
    const int64_t j0 = kbeg + tile * ATT_TK;
    for (int e = lane; e < ATT_TK * chunks; e += 32) {
      const int kk = e / chunks, c = e % chunks;
      const int64_t j = j0 + kk;
      if (j < kend)
        cp_async16(reinterpret_cast<uint8_t *>(kd + kk * DP) + 16 * c,
                   reinterpret_cast<const uint8_t *>(kbase + j * p.k_ss) + 16 * c);
    }
    for (int e = lane; e < ATT_TK * chunks_v; e += 32) {
      const int kk = e / chunks_v, c = e % chunks_v;
      const int64_t j = j0 + kk;
      if (j < kend)
        cp_async16(reinterpret_cast<uint8_t *>(vd + kk * DPv) + 16 * c,
                   reinterpret_cast<const uint8_t *>(vbase + j * p.v_ss) + 16 * c);
    }
  };

  __syncthreads();
  float m_run[ROWS], l_run[ROWS];
  float acc[ROWS][DPL];
#pragma unroll
  for (int r = 0; r < ROWS; ++r) {
    m_run[r] = -INFINITY;
    l_run[r] = 0.0f;
#pragma unroll
    for (int t = 0; t < DPL; ++t) acc[r][t] = 0.0f;
  }
  const int dpl = (Dv + 31) / 32; // output dims per lane

  int64_t my_tile = warp;
  if (my_tile < ntiles) issue(my_tile, 0);
  cp_async_commit();
  int buf = 0;
  for (; my_tile < ntiles; my_tile += 4) {
    const int64_t next = my_tile + 4;
    if (next < ntiles) issue(next, buf ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncwarp();
    const T *kt = ks + (buf * 4 + warp) * ATT_TK * DP;
    const T *vt = vs + (buf * 4 + warp) * ATT_TK * DPv;
    const int64_t j = kbeg + my_tile * ATT_TK + lane;
    const bool valid = j < kend;
    // scores for this lane's key against every row
    float sc[ROWS];
#pragma unroll
    for (int r = 0; r < ROWS; ++r) sc[r] = 0.0f;
    if (valid) {
      const T *krow = kt + lane * DP;
      for (int d = 0; d < D; d += 8) {
        float kv[8];
        if (sizeof(T) == 2) {
          const uint4 raw = *reinterpret_cast<const uint4 *>(krow + d);
          const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            const uint16_t lo = (uint16_t)(w[t] & 0xffffu), hi = (uint16_t)(w[t] >> 16);
            if (p.dt == kFloat16) {
              kv[2 * t] = f16_bits_to_f32(lo);
              kv[2 * t + 1] = f16_bits_to_f32(hi);
            } else {
              kv[2 * t] = __uint_as_float((uint32_t)lo << 16);
              kv[2 * t + 1] = __uint_as_float((uint32_t)hi << 16);
            }
          }
        } else {
#pragma unroll
          for (int t = 0; t < 8; ++t) kv[t] = ld_act<T>(krow, d + t);
        }
#pragma unroll
        for (int r = 0; r < ROWS; ++r) {
          const float4 q0 = *reinterpret_cast<const float4 *>(qs + r * D + d);
          const float4 q1 = *reinterpret_cast<const float4 *>(qs + r * D + d + 4);
          float s = sc[r];
          s = fmaf(q0.x, kv[0], s); s = fmaf(q0.y, kv[1], s);
          s = fmaf(q0.z, kv[2], s); s = fmaf(q0.w, kv[3], s);
          s = fmaf(q1.x, kv[4], s); s = fmaf(q1.y, kv[5], s);
          s = fmaf(q1.z, kv[6], s); s = fmaf(q1.w, kv[7], s);
          sc[r] = s;
        }
      }
    }
    // scale, softcap, mask; online softmax per row
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
      float s = -INFINITY;
      if (valid && r < nrows) {
        const int rr = row0 + r;
        const int64_t h = kvh * p.group + rr % p.group, qi = rr / p.group;
        s = sc[r] * p.scale;
        if (p.softcap > 0.0f) s = p.softcap * tanhf(s / p.softcap);
        s += att_bias(p, b, h, qi, j);
      }
      float tmax = s;
#pragma unroll
      for (int o = 16; o; o >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, o));
      const float m_new = fmaxf(m_run[r], tmax);
      // all keys so far masked: keep zeros
      const float corr = m_new == -INFINITY ? 1.0f : __expf(m_run[r] - m_new);
      const float pj = (s == -INFINITY) ? 0.0f : __expf(s - m_new);
      float psum = pj;
#pragma unroll
      for (int o = 16; o; o >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, o);
      l_run[r] = l_run[r] * corr + psum;
      m_run[r] = m_new;
#pragma unroll
      for (int t = 0; t < DPL; ++t) acc[r][t] *= corr;
      ps[(warp * ROWS + r) * ATT_TK + lane] = pj;
    }
    __syncwarp();
    // P.V: lane owns dims d = lane + 32 t
    const int64_t rem_k = kend - (kbeg + my_tile * ATT_TK);
    const int nk = rem_k < ATT_TK ? (int)rem_k : ATT_TK;
    for (int kk = 0; kk < nk; ++kk) {
      float vv[DPL];
#pragma unroll
      for (int t = 0; t < DPL; ++t)
        vv[t] = (t < dpl && lane + 32 * t < Dv) ? ld_act<T>(vt + kk * DPv, lane + 32 * t) : 0.0f;
#pragma unroll
      for (int r = 0; r < ROWS; ++r) {
        const float pr = ps[(warp * ROWS + r) * ATT_TK + kk];
#pragma unroll
        for (int t = 0; t < DPL; ++t) acc[r][t] = fmaf(pr, vv[t], acc[r][t]);
      }
    }
    __syncwarp();
    buf ^= 1;
  }
  cp_async_wait<0>();

  // Merge the 4 warps of this CTA: red[warp][r] = (m, l), then o.
  float *red_ml = red;                        // [4][ROWS][2]
  float *red_o = red + 4 * ROWS * 2;       // [4][ROWS][Dv]
  if (lane == 0) {
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
      red_ml[(warp * ROWS + r) * 2] = m_run[r];
      red_ml[(warp * ROWS + r) * 2 + 1] = l_run[r];
    }
  }
#pragma unroll
  for (int r = 0; r < ROWS; ++r)
#pragma unroll
    for (int t = 0; t < DPL; ++t)
      if (t < dpl && lane + 32 * t < Dv) red_o[(warp * ROWS + r) * Dv + lane + 32 * t] = acc[r][t];
  __syncthreads();

  const int64_t row_base = (int64_t)bh * p.rows_total + row0; // global row id
  for (int e = threadIdx.x; e < nrows * Dv; e += ATT_THREADS) {
    const int r = e / Dv, d = e % Dv;
    float m = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) m = fmaxf(m, red_ml[(w * ROWS + r) * 2]);
    float l = 0.0f, o = 0.0f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float mw = red_ml[(w * ROWS + r) * 2];
      const float c = (mw == -INFINITY) ? 0.0f : __expf(mw - m);
      l += red_ml[(w * ROWS + r) * 2 + 1] * c;
      o += red_o[(w * ROWS + r) * Dv + d] * c;
    }
    const int64_t grow = row_base + r;
    if (p.splits == 1) {
      const int rr = row0 + r;
      const int64_t h = kvh * p.group + rr % p.group, qi = rr / p.group;
      st_act<T>(p.y, b * p.y_sb + h * p.y_sh + qi * p.y_ss + d, l != 0.0f ? o / l : 0.0f);
    } else {
      const int64_t nrow_all = p.B * p.Hkv * p.rows_total;
      p.ws_o[((int64_t)split * nrow_all + grow) * Dv + d] = o;
      if (d == 0) {
        p.ws_ml[((int64_t)split * nrow_all + grow) * 2] = m;
        p.ws_ml[((int64_t)split * nrow_all + grow) * 2 + 1] = l;
      }
    }
  }
  if (p.splits == 1) return;

  // Last split CTA of this (b, kv_head, row tile) merges all splits.
  __shared__ bool last;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    uint32_t *ctr = p.counters + (int64_t)bh * p.row_tiles + rt;
    const uint32_t prev = atomicAdd(ctr, 1u);
    last = prev + 1 == (uint32_t)p.splits;
    if (last) {
      __threadfence();
      *ctr = 0u;
    }
  }
  __syncthreads();
  if (!last) return;
  const int64_t nrow_all = p.B * p.Hkv * p.rows_total;
  for (int e = threadIdx.x; e < nrows * Dv; e += ATT_THREADS) {
    const int r = e / Dv, d = e % Dv;
    const int64_t grow = row_base + r;
    float m = -INFINITY;
    for (int s = 0; s < p.splits; ++s) m = fmaxf(m, __ldcg(p.ws_ml + ((int64_t)s * nrow_all + grow) * 2));
    float l = 0.0f, o = 0.0f;
    for (int s = 0; s < p.splits; ++s) {
      const float ms = __ldcg(p.ws_ml + ((int64_t)s * nrow_all + grow) * 2);
      const float c = (ms == -INFINITY) ? 0.0f : __expf(ms - m);
      l += __ldcg(p.ws_ml + ((int64_t)s * nrow_all + grow) * 2 + 1) * c;
      o += __ldcg(p.ws_o + ((int64_t)s * nrow_all + grow) * Dv + d) * c;
    }
    const int rr = row0 + r;
    const int64_t h = kvh * p.group + rr % p.group, qi = rr / p.group;
    st_act<T>(p.y, b * p.y_sb + h * p.y_sh + qi * p.y_ss + d, l != 0.0f ? o / l : 0.0f);
  }
}

// qk_matmul_output (kernel_attention.cc:615-668): one CTA per query row
// (b, h, i).  mode 0: the scaled scores Q.K^T * scale; 1: after the softcap;
// 2: after adding the mask bias; 3: the softmax probabilities (a fully
// masked row gives zeros).  Written as FLOAT, or demoted to FLOAT16 /
// BFLOAT16 (RNE) when Q is half precision, as the reference demotes it.
template <typename T>
__global__ void __launch_bounds__(128) attn_qk_out(const AttParams p, int mode, void *out,
                                                   int out_dt) {
  extern __shared__ float qrow[]; // [D]
  __shared__ float red[4];
  __shared__ int red_i[4];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t row = blockIdx.x; // ((b * Hq) + h) * Sq + i
  const int64_t i = row % p.Sq, bh = row / p.Sq, h = bh % p.Hq, b = bh / p.Hq;
  const int64_t kvh = h / p.group;
  const int D = (int)p.D;
  for (int d = threadIdx.x; d < D; d += blockDim.x)
    qrow[d] = ld_act<T>(p.q, b * p.q_sb + h * p.q_sh + i * p.q_ss + d);
  __syncthreads();
  const T *kb = reinterpret_cast<const T *>(p.k) + b * p.k_sb + kvh * p.k_sh;
  // score of key j at the stage `upto` (0 raw, 1 softcap, 2 masked); *bias_out
  // receives the mask bias.
  auto score = [&](int64_t j, int upto, float *bias_out) {
    float s = 0.0f;
    for (int d = 0; d < D; ++d) s = fmaf(qrow[d], ld_act<T>(kb, j * p.k_ss + d), s);
    s *= p.scale;
    if (upto >= 1 && p.softcap > 0.0f) s = p.softcap * tanhf(s / p.softcap);
    const float bias = att_bias(p, b, h, i, j);
    if (bias_out) *bias_out = bias;
    if (upto >= 2) s += bias;
    return s;
  };
  auto put = [&](int64_t j, float v) {
    const int64_t o = row * p.L + j;
    if (out_dt == kFloat) reinterpret_cast<float *>(out)[o] = v;
    else if (out_dt == kFloat16) reinterpret_cast<uint16_t *>(out)[o] = f32_to_f16_bits(v);
    else reinterpret_cast<uint16_t *>(out)[o] = f32_to_bf16_bits(v);
  };
  if (mode != 3) {
    for (int64_t j = threadIdx.x; j < p.L; j += blockDim.x) put(j, score(j, mode, nullptr));
    return;
  }
  // softmax: row maximum and "fully masked" flag, then the sum, then the values
  float mx = -INFINITY;
  int live = 0;
  for (int64_t j = threadIdx.x; j < p.L; j += blockDim.x) {
    float bias;
    const float s = score(j, 2, &bias);
    mx = fmaxf(mx, s);
    live |= !(isinf(bias) && bias < 0.0f);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    live |= __shfl_xor_sync(0xffffffffu, live, o);
  }
  if (lane == 0) {
    red[warp] = mx;
    red_i[warp] = live;
  }
  __syncthreads();
  mx = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
  live = red_i[0] | red_i[1] | red_i[2] | red_i[3];
  __syncthreads();
  float sum = 0.0f;
  if (live)
    for (int64_t j = threadIdx.x; j < p.L; j += blockDim.x) sum += expf(score(j, 2, nullptr) - mx);
#pragma unroll
  for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if (lane == 0) red[warp] = sum;
  __syncthreads();
  sum = red[0] + red[1] + red[2] + red[3];
  const float inv = sum != 0.0f ? 1.0f / sum : 0.0f;
  for (int64_t j = threadIdx.x; j < p.L; j += blockDim.x)
    put(j, live ? expf(score(j, 2, nullptr) - mx) * inv : 0.0f);
}

// present[b, h, dst_off + s, :] = src(b, h, s, :) for s < S; 16-byte chunks.
template <typename T>
__global__ void kv_copy(const T *__restrict__ src, int64_t s_sb, int64_t s_sh, int64_t s_ss,
                        T *__restrict__ dst, int64_t d_sb, int64_t d_sh, int64_t d_ss,
                        int64_t dst_off, int64_t B, int64_t H, int64_t S, int64_t D) {
  const int64_t chunks = D * (int64_t)sizeof(T) / 16;
  const int64_t total = B * H * S * chunks;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t c = e % chunks;
    int64_t t = e / chunks;
    const int64_t s = t % S;
    t /= S;
    const int64_t h = t % H, b = t / H;
    const uint4 val = *reinterpret_cast<const uint4 *>(src + b * s_sb + h * s_sh + s * s_ss + c * (16 / sizeof(T)));
    *reinterpret_cast<uint4 *>(dst + b * d_sb + h * d_sh + (dst_off + s) * d_ss + c * (16 / sizeof(T))) = val;
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

// ONNXL_B200_ATTN_KERNEL=cuda forces the CUDA-core kernel where the tensor-core
// decode kernel would run (tests compare both); returns 1 in that case.
// ONNXL_B200_ATTN_KERNEL: "cuda" forces the CUDA-core kernel, "mma" the
// mma.sync prefill kernel instead of the tcgen05 one (tests compare them).
static int forced_attention_kernel() {
  const char *e = getenv("ONNXL_B200_ATTN_KERNEL");
  if (e && !strcmp(e, "cuda")) return 1;
  if (e && !strcmp(e, "mma")) return 2;
  return 0;
}

struct View { int64_t sb, sh, ss; };

static View rank4_view(int64_t H, int64_t S, int64_t D) { return {H * S * D, S * D, D}; }
static View rank3_view(int64_t H, int64_t S, int64_t D) { return {S * H * D, D, H * D}; }

template <typename T>
static int launch_copy(const void *src, View sv, void *dst, View dv, int64_t off, int64_t B,
                       int64_t H, int64_t S, int64_t D, cudaStream_t st) {
  const int64_t total = B * H * S * (D * (int64_t)sizeof(T) / 16);
  if (total == 0) return B2_OK;
  int64_t blocks = (total + 255) / 256;
  if (blocks > sm_count() * 16) blocks = sm_count() * 16;
  kv_copy<T><<<(unsigned)blocks, 256, 0, st>>>(static_cast<const T *>(src), sv.sb, sv.sh, sv.ss,
                                                static_cast<T *>(dst), dv.sb, dv.sh, dv.ss, off, B,
                                                H, S, D);
  B2_LAUNCH_CHECK();
  return B2_OK;
}

template <typename T>
static int attention_t(const b2_tensor *q, const b2_tensor *k, const b2_tensor *v,
                       const b2_tensor *mask, const b2_tensor *past_k, const b2_tensor *past_v,
                       const b2_tensor *nonpad, const b2_attention_attrs *at, b2_tensor *y,
                       b2_tensor *pres_k, b2_tensor *pres_v, b2_tensor *qk, void *ws,
                       size_t *ws_bytes, cudaStream_t st) {
  const int rank = q->ndim;
  int64_t B, Hq, Sq, D, Dv, Hkv, Sk;
  View qv, kv, vv, yv;
  if (rank == 4) {
    B = q->shape[0]; Hq = q->shape[1]; Sq = q->shape[2]; D = q->shape[3];
    Hkv = k->shape[1]; Sk = k->shape[2];
    B2_ENFORCE(k->shape[0] == B && v->shape[0] == B,
               "kernel::Attention: Q, K, V must share the same batch size.");
    B2_ENFORCE(k->shape[3] == D, "kernel::Attention: K head_size must match Q head_size.");
    B2_ENFORCE(v->shape[1] == Hkv, "kernel::Attention: V num_heads must match K num_heads.");
    B2_ENFORCE(v->shape[2] == Sk, "kernel::Attention: V kv_seq_len must match K kv_seq_len.");
    Dv = v->shape[3]; // v_head_size (kernel_attention.cc:478)
    qv = rank4_view(Hq, Sq, D);
    kv = rank4_view(Hkv, Sk, D);
    vv = rank4_view(Hkv, Sk, Dv);
    yv = rank4_view(Hq, Sq, Dv);
  } else {
    B2_ENFORCE(at->q_num_heads > 0, "kernel::Attention: 'Q' needs a positive ``num_heads`` to promote rank-3.");
    B2_ENFORCE(at->kv_num_heads > 0, "kernel::Attention: 'K' needs a positive ``num_heads`` to promote rank-3.");
    B = q->shape[0]; Sq = q->shape[1]; Hq = at->q_num_heads;
    B2_ENFORCE(q->shape[2] % Hq == 0, "kernel::Attention: 'Q' hidden_size must be a multiple of ``num_heads``.");
    D = q->shape[2] / Hq;
    Hkv = at->kv_num_heads;
    Sk = k->shape[1];
    B2_ENFORCE(k->shape[2] % Hkv == 0, "kernel::Attention: 'K' hidden_size must be a multiple of ``num_heads``.");
    B2_ENFORCE(k->shape[2] / Hkv == D, "kernel::Attention: K head_size must match Q head_size.");
    B2_ENFORCE(v->shape[2] % Hkv == 0, "kernel::Attention: 'V' hidden_size must be a multiple of ``num_heads``.");
    B2_ENFORCE(k->shape[0] == B && v->shape[0] == B,
               "kernel::Attention: Q, K, V must share the same batch size.");
    B2_ENFORCE(v->shape[1] == Sk, "kernel::Attention: V kv_seq_len must match K kv_seq_len.");
    Dv = v->shape[2] / Hkv;
    qv = rank3_view(Hq, Sq, D);
    kv = rank3_view(Hkv, Sk, D);
    vv = rank3_view(Hkv, Sk, Dv);
    yv = rank3_view(Hq, Sq, Dv);
  }
  B2_ENFORCE(Hkv > 0 && Hq % Hkv == 0,
             "kernel::Attention: q_num_heads must be a positive multiple of kv_num_heads.");
  B2_ENFORCE(at->left_window_size >= -1,
             "kernel::Attention: 'left_window_size' must be -1 or nonnegative.");
  B2_ENFORCE(at->right_window_size >= -1,
             "kernel::Attention: 'right_window_size' must be -1 or nonnegative.");
  B2_ENFORCE((past_k == nullptr) == (past_v == nullptr),
             "kernel::Attention: past_key and past_value must be provided together.");
  if (qk)
    B2_ENFORCE(at->qk_matmul_output_mode >= 0 && at->qk_matmul_output_mode <= 3,
               "kernel::Attention: 'qk_matmul_output_mode' must be 0, 1, 2 or 3.");
  if (D % 8 != 0 || D > ATT_DMAX || Dv % 8 != 0 || Dv > ATT_DMAX)
    B2_FAIL(B2_ERR_UNSUPPORTED, "kernel::Attention: head sizes must be multiples of 8 and <= 256 on the GPU");
  const int64_t P = past_k ? past_k->shape[2] : 0;
  if (past_k) {
    B2_ENFORCE(past_k->ndim == 4 && past_v->ndim == 4, "kernel::Attention: concat inputs must be rank-4.");
    B2_ENFORCE(past_k->shape[0] == B && past_k->shape[1] == Hkv && past_k->shape[3] == D,
               "kernel::Attention: past KV shape must match current K/V on axes 0, 1, 3.");
    B2_ENFORCE(past_v->shape[0] == B && past_v->shape[1] == Hkv && past_v->shape[2] == P &&
                   past_v->shape[3] == Dv,
               "kernel::Attention: past KV shape must match current K/V on axes 0, 1, 3.");
  }
  const int64_t L = P + Sk;
  if (mask) {
    // FLOAT or BOOL; FLOAT16 / BFLOAT16 too when Q is half precision (the
    // reference's half-precision entry promotes such a mask, :797-801).
    const bool half_q = q->dtype == kFloat16 || q->dtype == kBfloat16;
    const bool half_m = mask->dtype == kFloat16 || mask->dtype == kBfloat16;
    B2_ENFORCE(mask->dtype == kFloat || mask->dtype == kBool || (half_q && half_m),
               "kernel::Attention: 'attn_mask' must be FLOAT or BOOL.");
    B2_ENFORCE(mask->ndim >= 1 && mask->ndim <= 4,
               "kernel::Attention: 'attn_mask' must have rank between 1 and 4.");
  }
  int64_t ms[4] = {1, 1, 1, 1};
  if (mask) {
    for (int i = 0; i < mask->ndim; ++i) ms[4 - mask->ndim + i] = mask->shape[i];
    const int64_t od[3] = {B, Hq, Sq};
    for (int i = 0; i < 3; ++i)
      B2_ENFORCE(ms[i] == 1 || ms[i] == od[i],
                 "kernel::Attention: 'attn_mask' is not broadcastable to (batch_size, q_num_heads, "
                 "q_seq_len); its last axis defines the mask KV length.");
  }
  // nonpad_kv_seqlen (kernel_attention.cc:484-496): an empty tensor is ignored.
  if (nonpad && numel(nonpad) == 0) nonpad = nullptr;
  B2_ENFORCE(nonpad == nullptr || past_k == nullptr,
             "kernel::Attention: nonpad_kv_seqlen cannot be combined with past cache.");
  if (nonpad) {
    B2_ENFORCE(nonpad->dtype == kInt64, "kernel::Attention: 'nonpad_kv_seqlen' must be INT64.");
    B2_ENFORCE(nonpad->ndim == 1 && nonpad->shape[0] == B,
               "kernel::Attention: 'nonpad_kv_seqlen' must be a 1-D tensor of length batch_size.");
  }
  // present buffers
  const bool alias = at->kv_capacity > 0;
  const bool have_present = pres_k && pres_v;
  if (past_k) B2_ENFORCE(have_present, "b2_attention: present_key/present_value are required with a past");
  int64_t cap = L;
  if (alias) {
    cap = at->kv_capacity;
    B2_ENFORCE(L <= cap, "b2_attention: past_len + new tokens exceed kv_capacity");
    B2_ENFORCE(past_k == nullptr || (past_k->data == pres_k->data && past_v->data == pres_v->data),
               "b2_attention: with kv_capacity the past and present tensors must share storage");
  }
  if (have_present) {
    B2_ENFORCE(pres_k->ndim == 4 && pres_k->shape[0] == B && pres_k->shape[1] == Hkv &&
                   pres_k->shape[2] == L && pres_k->shape[3] == D,
               "b2_attention: present_key must be [B, Hkv, past+new, D]");
    B2_ENFORCE(pres_v->ndim == 4 && pres_v->shape[0] == B && pres_v->shape[1] == Hkv &&
                   pres_v->shape[2] == L && pres_v->shape[3] == Dv,
               "b2_attention: present_value must be [B, Hkv, past+new, D]");
  }
  B2_ENFORCE(y->dtype == q->dtype, "kernel::Attention preallocated output must share Q's element type.");
  B2_ENFORCE(numel(y) == B * Hq * Sq * Dv,
             "kernel::Attention preallocated output shape must be (batch_size, q_num_heads, "
             "q_seq_len, v_head_size).");
  const int qk_dt = q->dtype; // FLOAT, or demoted to Q's half type (:831-832)
  if (qk)
    B2_ENFORCE(qk->dtype == qk_dt && qk->ndim == 4 && qk->shape[0] == B && qk->shape[1] == Hq &&
                   qk->shape[2] == Sq && qk->shape[3] == L,
               "b2_attention: qk_matmul_output must be [B, Hq, Sq, past+new] of Q's dtype");

  // plan
  const int group = (int)(Hq / Hkv);
  const int rows_total = (int)(group * Sq);
  const int rows_cta = rows_total <= 4 ? 4 : ATT_ROWS;
  const int row_tiles = (rows_total + rows_cta - 1) / rows_cta;
  const int64_t ctas_base = B * Hkv * row_tiles;
  const int sms = sm_count();
  int64_t splits = ctas_base >= 2 * sms || ctas_base > (int64_t)kMaxCounters
                       ? 1 : (2 * sms + ctas_base - 1) / ctas_base;
  int64_t kps = (L + splits - 1) / splits;
  kps = (kps + 4 * ATT_TK - 1) / (4 * ATT_TK) * (4 * ATT_TK);
  if (kps < 4 * ATT_TK) kps = 4 * ATT_TK;
  splits = (L + kps - 1) / kps;
  if (splits < 1) splits = 1;
  const int64_t nrow_all = B * Hkv * rows_total;
  View cache = {Hkv * cap * D, cap * D, D};
  const View cache_v = {Hkv * cap * Dv, cap * Dv, Dv};
  const View kv_src = have_present ? cache : kv;
  // The tensor-core kernels take equal head sizes and no nonpad_kv_seqlen.
  const bool tc_shape = Dv == D && nonpad == nullptr;
  const bool decode_tc =
      tc_shape && attn_decode_eligible(q->dtype, D, Sq, group, mask != nullptr, at->left_window_size,
                           at->right_window_size, kv_src.sb, kv_src.sh, kv_src.ss, Hkv, L,
                           at->is_causal != 0, Sk) &&
      vv.sb == kv.sb && vv.sh == kv.sh && vv.ss == kv.ss && B * Hkv <= (int64_t)kMaxCounters &&
      forced_attention_kernel() != 1;
  const bool prefill_tc =
      !decode_tc && tc_shape &&
      attn_prefill_eligible(q->dtype, D, Sq, mask != nullptr, at->left_window_size,
                            at->right_window_size, kv_src.ss, L) &&
      vv.sb == kv.sb && vv.sh == kv.sh && vv.ss == kv.ss && forced_attention_kernel() != 1 &&
      kv_src.sb % 8 == 0 && kv_src.sh % 8 == 0 && qv.sb % 2 == 0 && qv.sh % 2 == 0 &&
      qv.ss % 2 == 0 && yv.sb % 2 == 0 && yv.sh % 2 == 0 && yv.ss % 2 == 0 &&
      ((reinterpret_cast<uintptr_t>(q->data) | reinterpret_cast<uintptr_t>(y->data)) & 3) == 0 &&
      ((reinterpret_cast<uintptr_t>(have_present ? pres_k->data : k->data) |
        reinterpret_cast<uintptr_t>(have_present ? pres_v->data : v->data)) & 15) == 0;
  size_t need = 0;
  if (prefill_tc)
    need = 0;
  else if (decode_tc)
    need = attn_decode_workspace(B, Hkv);
  else if (splits > 1)
    need = kCounterBytes + (size_t)splits * nrow_all * (Dv + 2) * 4;
  int rc = workspace_check(ws, ws_bytes, need);
  if (rc < 0) return rc;
  if (rc == 1) return B2_OK;

  // 1) build present: copy the past unless it is already in place, append new K/V.
  if (have_present) {
    if (past_k && !alias) {
      rc = launch_copy<T>(past_k->data, rank4_view(Hkv, P, D), pres_k->data, cache, 0, B, Hkv, P, D, st);
      if (rc) return rc;
      rc = launch_copy<T>(past_v->data, rank4_view(Hkv, P, Dv), pres_v->data, cache_v, 0, B, Hkv, P, Dv, st);
      if (rc) return rc;
    }
    rc = launch_copy<T>(k->data, kv, pres_k->data, cache, P, B, Hkv, Sk, D, st);
    if (rc) return rc;
    rc = launch_copy<T>(v->data, vv, pres_v->data, cache_v, P, B, Hkv, Sk, Dv, st);
    if (rc) return rc;
  }
  if (B * Hq * Sq == 0) return B2_OK;

  AttParams p{};
  p.q = q->data;
  p.k = have_present ? pres_k->data : k->data;
  p.v = have_present ? pres_v->data : v->data;
  const View kview = have_present ? cache : kv;
  const View vview = have_present ? cache_v : vv;
  p.y = y->data;
  p.mask = mask ? mask->data : nullptr;
  p.mask_dt = mask ? mask->dtype : kFloat;
  for (int i = 0; i < 4; ++i) p.mask_shape[i] = ms[i];
  p.nonpad = nonpad ? static_cast<const int64_t *>(nonpad->data) : nullptr;
  p.B = B; p.Hq = Hq; p.Hkv = Hkv; p.Sq = Sq; p.L = L; p.D = D; p.Dv = Dv;
  p.q_sb = qv.sb; p.q_sh = qv.sh; p.q_ss = qv.ss;
  p.k_sb = kview.sb; p.k_sh = kview.sh; p.k_ss = kview.ss;
  p.v_sb = vview.sb; p.v_sh = vview.sh; p.v_ss = vview.ss;
  p.y_sb = yv.sb; p.y_sh = yv.sh; p.y_ss = yv.ss;
  p.past_len = P;
  p.scale = at->has_scale ? at->scale : 1.0f / sqrtf((float)D);
  p.softcap = at->softcap;
  p.causal = at->is_causal;
  p.left_window = at->left_window_size;
  p.right_window = at->right_window_size;
  p.group = group;
  p.rows_total = rows_total;
  p.row_tiles = row_tiles;
  p.splits = (int)splits;
  p.keys_per_split = kps;
  p.dt = q->dtype;
  if (splits > 1) {
    p.counters = static_cast<uint32_t *>(ws);
    p.ws_o = reinterpret_cast<float *>(static_cast<uint8_t *>(ws) + kCounterBytes);
    p.ws_ml = p.ws_o + (size_t)splits * nrow_all * Dv;
  }
  if (L == 0) {
    // No keys: every row is fully masked and the reference writes zeros.
    B2_CUDA(cudaMemsetAsync(y->data, 0, (size_t)B * Hq * Sq * Dv * sizeof(T), st));
    return B2_OK;
  }
  if (qk) {
    attn_qk_out<T><<<(unsigned)(B * Hq * Sq), 128, (size_t)D * 4, st>>>(
        p, at->qk_matmul_output_mode, qk->data, qk_dt);
    B2_LAUNCH_CHECK();
  }
  if (prefill_tc) {
    const int64_t qs[3] = {qv.sb, qv.sh, qv.ss}, ys[3] = {yv.sb, yv.sh, yv.ss};
    const int64_t ks[3] = {kview.sb, kview.sh, kview.ss};
    // tcgen05 kernel unless forced to the mma.sync one; it needs 16-byte
    // aligned Q / Y rows (TMA reads of Q, 16-byte stores of Y).
    const bool aligned16 =
        ((reinterpret_cast<uintptr_t>(q->data) | reinterpret_cast<uintptr_t>(y->data)) & 15) == 0;
    if (forced_attention_kernel() != 2 && aligned16 &&
        attn_prefill_tc_eligible(q->dtype, D, Sq, false, -1, -1, qs, ks, ys, L))
      return attn_prefill_tc_launch(q->dtype, q->data, qs, p.k, p.v, ks, y->data, ys, B, Hq, Hkv,
                                    Sq, L, P, p.scale, p.softcap, p.causal, st);
    return attn_prefill_launch(q->dtype, q->data, qs, p.k, p.v, ks, y->data, ys, B, Hq, Hkv, Sq,
                               L, P, p.scale, p.softcap, p.causal, st);
  }
  if (decode_tc)
    return attn_decode_launch(q->data, qv.sb, qv.sh, p.k, p.v, kview.sh, B, Hkv, group, L,
                              p.scale, p.softcap, y->data, yv.sb, yv.sh, ws, st);
  const int DP = (int)D + 8, DPv = (int)Dv + 8;
  const size_t smem = (size_t)2 * 4 * ATT_TK * (DP + DPv) * sizeof(T) + (size_t)rows_cta * D * 4 +
                      (size_t)4 * rows_cta * ATT_TK * 4 + (size_t)4 * rows_cta * 2 * 4 +
                      (size_t)4 * rows_cta * Dv * 4;
  dim3 grid((unsigned)(B * Hkv), (unsigned)splits, (unsigned)row_tiles);
  const int dpl = (int)((Dv + 31) / 32);
  void (*kern)(AttParams) = nullptr;
  if (rows_cta == 4) {
    kern = dpl <= 2 ? attn_fwd<T, 4, 2> : dpl <= 4 ? attn_fwd<T, 4, 4> : attn_fwd<T, 4, 8>;
  } else {
    kern = dpl <= 2 ? attn_fwd<T, ATT_ROWS, 2> : dpl <= 4 ? attn_fwd<T, ATT_ROWS, 4> : attn_fwd<T, ATT_ROWS, 8>;
  }
  B2_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  kern<<<grid, ATT_THREADS, smem, st>>>(p);
  B2_LAUNCH_CHECK();
  return B2_OK;
}

} // namespace b2

using namespace b2;

extern "C" int b2_attention_ex(const b2_tensor *q, const b2_tensor *k, const b2_tensor *v,
                               const b2_tensor *attn_mask, const b2_tensor *past_key,
                               const b2_tensor *past_value, const b2_tensor *nonpad_kv_seqlen,
                               const b2_attention_attrs *attrs, b2_tensor *y,
                               b2_tensor *present_key, b2_tensor *present_value,
                               b2_tensor *qk_matmul_output, void *workspace,
                               size_t *workspace_bytes, void *stream) {
  if (!q || !k || !v || !attrs || !y) B2_FAIL(B2_ERR_INVALID_ARGUMENT, "kernel::Attention: null tensor");
  B2_ENFORCE(q->dtype == kFloat || q->dtype == kFloat16 || q->dtype == kBfloat16,
             "kernel::Attention: 'Q' must be a FLOAT, FLOAT16 or BFLOAT16 tensor.");
  B2_ENFORCE(k->dtype == q->dtype && v->dtype == q->dtype,
             "kernel::Attention: Q, K, V must share the same dtype.");
  B2_ENFORCE(q->ndim == k->ndim && q->ndim == v->ndim,
             "kernel::Attention: Q, K, V must all share the same rank.");
  B2_ENFORCE(q->ndim == 3 || q->ndim == 4, "kernel::Attention: Q, K, V must be rank-3 or rank-4.");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (q->dtype == kFloat16)
    return attention_t<__half>(q, k, v, attn_mask, past_key, past_value, nonpad_kv_seqlen, attrs,
                               y, present_key, present_value, qk_matmul_output, workspace,
                               workspace_bytes, st);
  if (q->dtype == kBfloat16)
    return attention_t<__nv_bfloat16>(q, k, v, attn_mask, past_key, past_value, nonpad_kv_seqlen,
                                      attrs, y, present_key, present_value, qk_matmul_output,
                                      workspace, workspace_bytes, st);
  return attention_t<float>(q, k, v, attn_mask, past_key, past_value, nonpad_kv_seqlen, attrs, y,
                            present_key, present_value, qk_matmul_output, workspace,
                            workspace_bytes, st);
}

extern "C" int b2_attention(const b2_tensor *q, const b2_tensor *k, const b2_tensor *v,
                            const b2_tensor *attn_mask, const b2_tensor *past_key,
                            const b2_tensor *past_value, const b2_attention_attrs *attrs,
                            b2_tensor *y, b2_tensor *present_key, b2_tensor *present_value,
                            void *workspace, size_t *workspace_bytes, void *stream) {
  return b2_attention_ex(q, k, v, attn_mask, past_key, past_value, nullptr, attrs, y, present_key,
                         present_value, nullptr, workspace, workspace_bytes, stream);
}
