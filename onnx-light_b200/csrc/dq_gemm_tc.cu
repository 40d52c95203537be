// Fused DequantizeLinear -> [Cast] -> MatMul on tcgen05 tensor cores (sm_100a)
// for FLOAT16 / BFLOAT16 activations.
//
// Orientation ("swap AB"): the MMA computes D^T[n, m] = W^T[n, k] . A^T[k, m],
// so 128 weight columns fill the MMA's M = 128 side and the activation rows
// (BN = 16 .. 256 of them) are the MMA's N side.  Decode batches of 8..64
// rows therefore run at full tile height, and prefill uses BN = 256.
//
// Per CTA (one 128-column x BN-row output tile, K range of one split):
//   warp 0      TMA: raw packed weight tile [64 k x 128 n] (no swizzle) and the
//               activation tile [BN m x 64 k] (128-byte swizzle, K-major) into
//               a STAGES-deep ring;
//   warps 2-9   dequantize the raw weight tile in registers with the
//               reference's rounding (fp32 (q - zp) * s, rounded to the
//               DequantizeLinear output type and to the Cast type) and store
//               it as the MMA's A operand in the 128-byte-swizzled MN-major
//               layout (64-element rows of n, 8-row atoms along k);
//   warp 1      allocates TMEM and one thread issues tcgen05.mma.kind::f16
//               (M=128, N=BN, K=16, fp32 accumulation in TMEM), releasing each
//               stage with tcgen05.commit;
//   warps 2-5   finally read the accumulator (tcgen05.ld) and write y, or
//               split-K partials merged by the last-arriving CTA.
#include "dq_matmul.cuh"
#include "tc_common.cuh"

namespace b2 {

constexpr int DT_BM = 128;     // weight columns per tile (MMA M)
constexpr int DT_BK = 64;      // k per stage (one 128-byte swizzle row of fp16)
constexpr int DT_PROD_WARPS = 8; // dequantizing warps (2 .. 9)
constexpr int DT_THREADS = 64 + DT_PROD_WARPS * 32;
constexpr uint32_t DT_AOP_BYTES = DT_BM * DT_BK * 2; // 16 KB dequantized operand

// kModePre: the weight was dequantized (and cast) once into a 16-bit operand
// [K, N] in the workspace (large M: every weight tile is used by many
// activation tiles), and both operands stream in by TMA.
enum DqMode : int { kModeI4H = 0, kModeF8 = 1, kModeF4 = 2, kModeGeneric = 3, kModePre = 4 };

struct DqTcArgs {
  DqMmParams p;
  int bn;          // activation rows per tile (MMA N)
  int stages;
  int mode;
  uint32_t raw_bytes;   // raw weight bytes per stage
  uint32_t b_bytes;     // activation bytes per stage
  uint32_t stage_bytes; // raw + aop + b + scales
  uint32_t s_bytes;     // scale bytes per stage (0: scales read from global memory)
  int s_rows;           // scale rows per stage
  int op_bf16;          // MMA operand type: 1 bf16, 0 f16
  int group_m;          // activation tiles per rasterization group (1: plain order)
  uint64_t wait_ns;     // limit of every bounded wait (kWaitNs)
  int no_loads;         // self-test only: issue no TMA, so the first data wait runs out
};

// Time-out code of the last launch that gave up (0 = none); read and cleared
// by b2_kernel_status().
__device__ int g_dq_gemm_tc_status;

// Packs two fp32 values into fp16x2 / bf16x2 bits with the reference's RNE.
__device__ __forceinline__ uint32_t pack2(float lo, float hi, bool bf16) {
  if (bf16) return (uint32_t)f32_to_bf16_bits(lo) | ((uint32_t)f32_to_bf16_bits(hi) << 16);
  return (uint32_t)f32_to_f16_bits(lo) | ((uint32_t)f32_to_f16_bits(hi) << 16);
}

// Dequantizes the 8 weights (k, n..n+7) into 8 operand values (uint4).
// `srow` points at the staged scale row of this weight row (nullptr: read the
// scale tensor in global memory).
template <int MODE>
__device__ __forceinline__ uint4 dequant8(const DqTcArgs &a, const uint8_t *raw_row, int nl,
                                          int64_t k, int64_t n, const uint8_t *srow) {
  const DqMmParams &p = a.p;
  if constexpr (MODE == kModeI4H) {
    // int4/uint4 x fp16 scale (blocked along K or per column), fp16 operand.
    const uint32_t w = *reinterpret_cast<const uint32_t *>(raw_row + nl / 2);
    const int64_t kb = p.slayout == kScaleAxis0Block ? (int64_t)p.fdiv_block.div((uint32_t)k) : 0;
    const int64_t si = p.slayout == kScaleTensor ? 0 : p.slayout == kScaleAxis1 ? n : kb * p.N + n;
    const uint16_t *sp = reinterpret_cast<const uint16_t *>(p.scale);
    uint32_t s4[4];
    if (p.slayout == kScaleTensor) {
      const uint32_t s = sp[0];
      s4[0] = s4[1] = s4[2] = s4[3] = s | (s << 16);
    } else {
      const uint4 v = srow ? *reinterpret_cast<const uint4 *>(srow + nl * 2)
                           : *reinterpret_cast<const uint4 *>(sp + si);
      s4[0] = __byte_perm(v.x, v.z, 0x5410); // (0, 4)
      s4[1] = __byte_perm(v.x, v.z, 0x7632); // (1, 5)
      s4[2] = __byte_perm(v.y, v.w, 0x5410); // (2, 6)
      s4[3] = __byte_perm(v.y, v.w, 0x7632); // (3, 7)
    }
    const bool sgn = p.wdt == kInt4;
    const uint32_t x = sgn ? (w ^ 0x88888888u) : w;
    const uint32_t bias = sgn ? 0x64086408u : 0x64006400u;
    uint32_t r[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t h = ((x >> (4 * j)) & 0x000f000fu) | 0x64006400u;
      uint32_t q;
      asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(q) : "r"(h), "r"(bias));
      asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r[j]) : "r"(q), "r"(s4[j]));
    }
    // r[j] = (elem j, elem j+4) -> output order (0,1),(2,3),(4,5),(6,7)
    uint4 o;
    o.x = __byte_perm(r[0], r[1], 0x5410);
    o.y = __byte_perm(r[2], r[3], 0x5410);
    o.z = __byte_perm(r[0], r[1], 0x7632);
    o.w = __byte_perm(r[2], r[3], 0x7632);
    return o;
  }
  // fp32 path: value = (q - zp) * s in fp32, rounded to the DequantizeLinear
  // output type (fp16 when the scale is fp16), then to the operand type.
  float q[8];
  if constexpr (MODE == kModeF8) {
    const uint2 w = *reinterpret_cast<const uint2 *>(raw_row + nl);
#pragma unroll
    for (int j = 0; j < 8; ++j) q[j] = dec_f8e4m3fn(((j < 4 ? w.x : w.y) >> (8 * (j & 3))) & 0xffu);
  } else if constexpr (MODE == kModeF4) {
    const uint32_t w = *reinterpret_cast<const uint32_t *>(raw_row + nl / 2);
#pragma unroll
    for (int j = 0; j < 8; ++j) q[j] = dec_f4e2m1((w >> (4 * j)) & 0xfu);
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) q[j] = qval(p.wdt, p.w, k * p.N + n + j);
  }
  float v[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    int64_t si;
    switch (p.slayout) {
    case kScaleTensor: si = 0; break;
    case kScaleAxis0Block: si = (int64_t)p.fdiv_block.div((uint32_t)k) * p.N + n + j; break;
    case kScaleAxis0: si = k; break;
    case kScaleAxis1Block: si = k * p.s_alen + p.fdiv_block.div((uint32_t)(n + j)); break;
    default: si = n + j; break;
    }
    float s;
    if (srow) s = p.s_f16 ? f16_bits_to_f32(reinterpret_cast<const uint16_t *>(srow)[nl + j])
                          : reinterpret_cast<const float *>(srow)[nl + j];
    else s = p.s_f16 ? f16_bits_to_f32(reinterpret_cast<const uint16_t *>(p.scale)[si])
                     : reinterpret_cast<const float *>(p.scale)[si];
    const float z = p.zp ? qval(p.wdt, p.zp, si) : 0.0f;
    float x = x86_mul(x86_sub(q[j], z), s);
    if (p.s_f16) x = f16_bits_to_f32(f32_to_f16_bits(x));
    v[j] = x;
  }
  const bool bf = a.op_bf16 != 0;
  return make_uint4(pack2(v[0], v[1], bf), pack2(v[2], v[3], bf), pack2(v[4], v[5], bf),
                    pack2(v[6], v[7], bf));
}

__device__ __forceinline__ void store_val(const DqMmParams &p, int64_t m, int64_t n, float v) {
  if (p.ydt == kFloat16) reinterpret_cast<uint16_t *>(p.y)[m * p.N + n] = f32_to_f16_bits(v);
  else reinterpret_cast<uint16_t *>(p.y)[m * p.N + n] = f32_to_bf16_bits(v);
}

template <int MODE>
__global__ void __launch_bounds__(DT_THREADS, MODE == kModePre ? 1 : 2)
    dq_gemm_tc_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_a,
                      const __grid_constant__ CUtensorMap map_s, const DqTcArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const DqMmParams &p = args.p;
  const int S = args.stages;
  // ring layout per stage: [aop 16 KB][b bn*128 B][raw]
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + (size_t)S * args.stage_bytes);
  uint64_t *deq = full + S;
  uint64_t *empty = deq + S;
  uint64_t *done = empty + S;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);
  __shared__ volatile int abort_flag;
  __shared__ int issued; // stages the producer filled (for the drain after a give-up)
  __shared__ bool last_cta, skip_merge;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Grouped rasterization: CTAs in launch order cover group_m activation
  // tiles across every weight tile before the next group, so a wave's tiles
  // share their operands in L2 instead of sweeping all weights per row tile.
  int64_t tile_n = blockIdx.x, tile_m = blockIdx.y;
  if (args.group_m > 1) {
    const int64_t lin = (int64_t)blockIdx.y * gridDim.x + blockIdx.x;
    const int64_t per_group = (int64_t)args.group_m * gridDim.x;
    const int64_t first_m = lin / per_group * args.group_m;
    const int64_t gsz = min((int64_t)gridDim.y - first_m, (int64_t)args.group_m);
    const int64_t r = lin % per_group;
    tile_m = first_m + r % gsz;
    tile_n = r / gsz;
  }
  const int64_t n0 = tile_n * DT_BM;
  const int64_t m0 = tile_m * args.bn;
  const int split = blockIdx.z;
  const int64_t kbeg = (int64_t)split * p.kchunk;
  const int64_t kend = min(p.K, kbeg + p.kchunk);
  const int kt_count = (int)((kend - kbeg + DT_BK - 1) / DT_BK);
  const uint32_t tmem_cols = args.bn <= 32 ? 32 : args.bn <= 64 ? 64 : args.bn <= 128 ? 128 : 256;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    issued = 0;
    for (int s = 0; s < S; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&deq[s], DT_PROD_WARPS);
      tc::mbar_init(&empty[s], 1);
    }
    tc::mbar_init(done, 1);
    tc::fence_barrier_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, tmem_cols);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (tc::elect_one()) {
      tc::prefetch_tensormap(&map_w);
      tc::prefetch_tensormap(&map_a);
      if (args.s_bytes) tc::prefetch_tensormap(&map_s);
      for (int kt = 0; kt < (args.no_loads ? 0 : kt_count); ++kt) {
        const int s = kt % S;
        if (kt >= S && !tc::mbar_wait(&empty[s], ((kt / S) - 1) & 1, args.wait_ns)) {
          atomicExch(&g_dq_gemm_tc_status, tc::kTimeoutEmpty);
          abort_flag = 1;
          break;
        }
        if (abort_flag) break;
        issued = kt + 1;
        uint8_t *st = smem + (size_t)s * args.stage_bytes;
        const int32_t k = (int32_t)(kbeg + (int64_t)kt * DT_BK);
        if constexpr (MODE == kModePre) {
          // operand tile [64 k][128 n] as two 64-column boxes with the 128-byte
          // swizzle: exactly the MN-major layout the dequantizing warps write
          tc::mbar_expect_tx(&full[s], DT_AOP_BYTES + args.b_bytes);
          tc::tma_load_2d(st, &map_w, &full[s], (int32_t)n0, k);
          tc::tma_load_2d(st + 8192, &map_w, &full[s], (int32_t)n0 + 64, k);
          tc::tma_load_2d(st + DT_AOP_BYTES, &map_a, &full[s], k, (int32_t)m0);
          continue;
        }
        const bool raw_tma = MODE != kModeGeneric;
        tc::mbar_expect_tx(&full[s], (raw_tma ? args.raw_bytes : 0u) + args.b_bytes + args.s_bytes);
        tc::tma_load_2d(st + DT_AOP_BYTES, &map_a, &full[s], k, (int32_t)m0);
        if (args.s_bytes)
          tc::tma_load_2d(st + DT_AOP_BYTES + args.b_bytes + args.raw_bytes, &map_s, &full[s],
                          (int32_t)n0, (int32_t)(k / p.block));
        if (raw_tma) {
          // raw weights: [k rows][128 n] as bytes (int4: 64 bytes, 8-bit: 128 bytes per row)
          const int32_t xb = MODE == kModeF8 ? (int32_t)n0 : (int32_t)(n0 / 2);
          tc::tma_load_2d(st + DT_AOP_BYTES + args.b_bytes, &map_w, &full[s], xb, k);
        }
      }
    }
  } else if (warp == 1) {
    if (tc::elect_one()) {
      const uint32_t id = tc::idesc(1, args.op_bf16, args.op_bf16, 1, 0, DT_BM, (uint32_t)args.bn);
      for (int kt = 0; kt < kt_count; ++kt) {
        const int s = kt % S;
        if (!tc::mbar_wait(MODE == kModePre ? &full[s] : &deq[s], (kt / S) & 1, args.wait_ns)) {
          atomicExch(&g_dq_gemm_tc_status, tc::kTimeoutFull);
          abort_flag = 1;
          break;
        }
        tc::tc_fence_after();
        const uint32_t a_base = tc::smem_u32(smem + (size_t)s * args.stage_bytes);
        const uint32_t b_base = a_base + DT_AOP_BYTES;
#pragma unroll
        for (int kk = 0; kk < DT_BK / 16; ++kk) {
          // A: MN-major, 2 blocks of 64 n (8 KB apart), 8-row atoms along k (1 KB)
          const uint64_t ad = tc::sdesc_sw128(a_base + kk * 16 * 128, 8192, 1024);
          // B: K-major activation rows, 128-byte rows, 8-row atoms (1 KB)
          const uint64_t bd = tc::sdesc_sw128(b_base + kk * 32, 16, 1024);
          tc::mma_f16(tmem, ad, bd, id, (kt > 0 || kk > 0) ? 1u : 0u);
        }
        tc::tc_commit(&empty[s]);
      }
      tc::tc_commit(done);
    }
  } else {
    // ----- dequant producers (warps 2..9) -----
    constexpr int kRowStep = DT_PROD_WARPS * 32 / 16; // rows of the stage a pass covers
    const int t = threadIdx.x - 64;
    const int cc = t & 15;   // 8-column chunk (n_local = cc * 8)
    const int r0 = t >> 4;   // first k row, rows r0 + kRowStep i
    const uint32_t raw_row_bytes = MODE == kModeF8 ? 128 : 64;
    for (int kt = 0; kt < (MODE == kModePre ? 0 : kt_count) && !abort_flag; ++kt) {
      const int s = kt % S;
      if (!tc::mbar_wait(&full[s], (kt / S) & 1, args.wait_ns)) {
        atomicExch(&g_dq_gemm_tc_status, tc::kTimeoutFull);
        abort_flag = 1;
        break;
      }
      uint8_t *st = smem + (size_t)s * args.stage_bytes;
      const uint8_t *raw = st + DT_AOP_BYTES + args.b_bytes;
      const uint8_t *sst = args.s_bytes ? raw + args.raw_bytes : nullptr;
      const int64_t kst = kbeg + (int64_t)kt * DT_BK; // first k of the stage
      const uint32_t s_esz = p.s_f16 ? 2u : 4u;
      const uint32_t kst_b = sst ? p.fdiv_block.div((uint32_t)kst) : 0u;
      if constexpr (MODE == kModeI4H) {
        // int4 x fp16 scale: the 8 nibbles of a 32-bit word become exact fp16
        // values with 4 logic ops, 1 shift, 2 subtractions and 2 FMAs (low
        // nibbles: 1024 + code - bias; high nibbles: (1024 + 16 code) / 16 -
        // bias), then the correctly rounded product with the fp16 scale -- the
        // reference's FloatToFloat16Bits((q - 0) * s).  The pairs come out as
        // columns (0,4) (1,5) (2,6) (3,7) and are stored in that order: the
        // MMA row of shared position p of an 8-column chunk is column
        // (p >> 1) + 4 (p & 1), which the epilogue maps back.
        const bool sgn = p.wdt == kInt4;
        const uint32_t mlo = sgn ? 0x64086408u : 0x64006400u;
        const uint32_t mhi = sgn ? 0x64806480u : 0x64006400u;
        const uint32_t bhi = sgn ? 0xd480d480u : 0xd400d400u; // -(64 + 8) / -64
        const int nl = cc * 8;
        // Scale pairs (s0,s4) (s1,s5) (s2,s6) (s3,s7) of the chunk, reloaded
        // only when the row's scale block changes.
        int64_t cur_kb = -1;
        uint32_t sp[4] = {0u, 0u, 0u, 0u};
        const uint16_t *s16 = reinterpret_cast<const uint16_t *>(p.scale);
        if (p.slayout == kScaleTensor) {
          const uint32_t sv = s16[0];
          sp[0] = sp[1] = sp[2] = sp[3] = sv | (sv << 16);
        }
        // No row guard: split ranges are whole 64-row stages, and rows past K
        // (and columns past N) arrive from TMA as zero codes with zero staged
        // scales, which dequantize to 0.  Branch-free, the rows interleave.
        const bool col_ok = n0 + nl < p.N;
#pragma unroll
        for (int i = 0; i < DT_BK / kRowStep; ++i) {
          const int r = r0 + kRowStep * i;
          const int64_t k = kst + r;
          if (p.slayout != kScaleTensor) {
            const int64_t kb = p.slayout == kScaleAxis1 ? 0 : (int64_t)p.fdiv_block.div((uint32_t)k);
            if (kb != cur_kb) {
              cur_kb = kb;
              uint4 v = make_uint4(0, 0, 0, 0);
              if (sst) v = *reinterpret_cast<const uint4 *>(sst + (size_t)(kb - kst_b) * DT_BM * 2 + nl * 2);
              else if (col_ok && k < p.K) v = *reinterpret_cast<const uint4 *>(s16 + kb * p.N + n0 + nl);
              sp[0] = __byte_perm(v.x, v.z, 0x5410);
              sp[1] = __byte_perm(v.x, v.z, 0x7632);
              sp[2] = __byte_perm(v.y, v.w, 0x5410);
              sp[3] = __byte_perm(v.y, v.w, 0x7632);
            }
          }
          uint4 o;
          {
            const uint32_t w = *reinterpret_cast<const uint32_t *>(raw + r * raw_row_bytes + nl / 2);
            const uint32_t w8 = w >> 8;
            uint32_t q0, q1, q2, q3;
            asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(q0) : "r"((w & 0x000f000fu) ^ mlo), "r"(mlo));
            asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(q1) : "r"((w & 0x00f000f0u) ^ mhi), "r"(0x2c002c00u), "r"(bhi));
            asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(q2) : "r"((w8 & 0x000f000fu) ^ mlo), "r"(mlo));
            asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(q3) : "r"((w8 & 0x00f000f0u) ^ mhi), "r"(0x2c002c00u), "r"(bhi));
            asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(o.x) : "r"(q0), "r"(sp[0]));
            asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(o.y) : "r"(q1), "r"(sp[1]));
            asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(o.z) : "r"(q2), "r"(sp[2]));
            asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(o.w) : "r"(q3), "r"(sp[3]));
          }
          const int blk = nl >> 6, chunk = (nl & 63) >> 3;
          uint8_t *dst = st + blk * 8192 + r * 128 + ((chunk ^ (r & 7)) << 4);
          *reinterpret_cast<uint4 *>(dst) = o;
        }
      } else {
#pragma unroll 2
      for (int i = 0; i < DT_BK / kRowStep; ++i) {
        const int r = r0 + kRowStep * i; // k row within the stage
        const int64_t k = kst + r;
        const int nl = cc * 8;
        const uint8_t *srow =
            sst ? sst + (size_t)(p.fdiv_block.div((uint32_t)k) - kst_b) * DT_BM * s_esz : nullptr;
        uint4 o = make_uint4(0, 0, 0, 0);
        if (k < kend && n0 + nl < p.N) o = dequant8<MODE>(args, raw + r * raw_row_bytes, nl, k, n0 + nl, srow);
        // MN-major 128-byte swizzle: block (nl / 64) at 8 KB, row r at 128 B,
        // 16-byte chunk (nl % 64) / 8 XOR (r % 8)
        const int blk = nl >> 6, chunk = (nl & 63) >> 3;
        uint8_t *dst = st + blk * 8192 + r * 128 + ((chunk ^ (r & 7)) << 4);
        *reinterpret_cast<uint4 *>(dst) = o;
      }
      }
      tc::fence_proxy_async();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&deq[s]);
    }
    // ----- epilogue (warps 2..5: one TMEM lane group each) -----
    if (warp < 6) {
      const int g = warp & 3; // TMEM lane group
      const bool ok = tc::mbar_wait(done, 0, 2 * args.wait_ns);
      if (!ok) {
        atomicExch(&g_dq_gemm_tc_status, tc::kTimeoutMma);
        abort_flag = 1;
      }
      tc::tc_fence_after();
      // MMA row -> weight column (the int4 path stores each 8-column chunk
      // in the order 0 4 1 5 2 6 3 7)
      const int pos = g * 32 + lane;
      const int64_t n = n0 + (MODE == kModeI4H ? (pos & ~7) + (pos & 7) / 2 + (pos & 1) * 4 : pos);
      if (ok && !abort_flag) {
        float *part = p.ksplit > 1 ? p.partials + (int64_t)split * p.M * p.N : nullptr;
        for (int ch = 0; ch < args.bn / 32 + ((args.bn & 31) ? 1 : 0); ++ch) {
          uint32_t r[32];
          tc::tmem_ld32(tmem + ((uint32_t)(g * 32) << 16) + (uint32_t)(ch * 32), r);
          tc::tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int64_t m = m0 + ch * 32 + j;
            if (ch * 32 + j < args.bn && m < p.M && n < p.N) {
              const float v = __uint_as_float(r[j]);
              if (part) part[m * p.N + n] = v;
              else store_val(p, m, n, v);
            }
          }
        }
      }
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 1) tc::tmem_dealloc(tmem, tmem_cols);
  if (abort_flag && threadIdx.x == 0) {
    // A wait gave up: let this CTA's own copies in flight land before it
    // exits (the last fill of each stage; bounded again).
    const int n = issued;
    for (int kt = n > S ? n - S : 0; kt < n; ++kt)
      tc::mbar_wait(&full[kt % S], (kt / S) & 1, args.wait_ns / 4);
  }
  if (p.ksplit <= 1) return;
  // split-K: the last CTA of this output tile sums the partials in split
  // order, unless a contributor gave up (its partials are not valid)
  if (threadIdx.x == 0) {
    bool gave_up = false;
    last_cta = arrive_marked(p.counters + (blockIdx.y * gridDim.x + blockIdx.x),
                             (uint32_t)p.ksplit, abort_flag != 0, &gave_up);
    skip_merge = gave_up;
  }
  __syncthreads();
  if (!last_cta || skip_merge) return;
  for (int e = threadIdx.x; e < DT_BM * args.bn; e += DT_THREADS) {
    const int64_t m = m0 + e / DT_BM, n = n0 + e % DT_BM;
    if (m >= p.M || n >= p.N) continue;
    float s = 0.0f;
    for (int sp = 0; sp < p.ksplit; ++sp) s += __ldcg(p.partials + ((int64_t)sp * p.M + m) * p.N + n);
    store_val(p, m, n, s);
  }
}

// The 16-bit MMA operand of the whole weight: w16[k][n] = the reference's
// DequantizeLinear value rounded to its output type and to the Cast type,
// exactly as the dequantizing warps form it (8 columns per thread).
template <int MODE>
__global__ void __launch_bounds__(256) dq_operand_kernel(const DqTcArgs args, uint16_t *w16) {
  const DqMmParams &p = args.p;
  const int64_t groups = p.N / 8;
  const int64_t total = p.K * groups;
  const int64_t row_bytes = MODE == kModeF8 ? p.N : p.N / 2;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t k = e / groups, n = (e % groups) * 8;
    const uint4 o = dequant8<MODE>(args, p.w + k * row_bytes, (int)n, k, n, nullptr);
    *reinterpret_cast<uint4 *>(w16 + k * p.N + n) = o;
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

static int dq_tc_mode(const DqMmParams &p) {
  if ((p.wdt == kInt4 || p.wdt == kUint4) && p.s_f16 && p.zp == nullptr && p.ydt == kFloat16 &&
      (p.cast_dt == 0 || p.cast_dt == kFloat16) &&
      (p.slayout == kScaleTensor || (p.slayout == kScaleAxis0Block && p.block % 8 == 0) ||
       p.slayout == kScaleAxis1))
    return kModeI4H;
  if (p.wdt == kF8E4M3FN) return kModeF8;
  if (p.wdt == kF4E2M1) return kModeF4;
  return kModeGeneric;
}

struct TcPlan {
  int bn = 0, stages = 0, ksplit = 1, mode = 0, s_rows = 0;
  int pre = 0; // 1: dequantize the weight once into the workspace (kModePre)
  int group_m = 1; // activation tiles per rasterization group
  uint32_t s_bytes = 0;
  int64_t kchunk = 0;
  uint32_t raw_bytes = 0, b_bytes = 0, stage_bytes = 0;
  size_t smem = 0;
  dim3 grid;
};

constexpr int64_t kPreM = 2048; // rows of activations from which the weight is dequantized once

static TcPlan tc_plan(const DqMmParams &p) {
  TcPlan t;
  t.mode = dq_tc_mode(p);
  t.bn = p.M >= 256 ? 256 : (int)((p.M + 15) / 16 * 16);
  if (t.bn < 16) t.bn = 16;
  t.raw_bytes = (t.mode == kModeF8 ? 128u : 64u) * DT_BK;
  if (t.mode == kModeGeneric) t.raw_bytes = 64u * DT_BK; // raw tile unused, keep the ring uniform
  t.b_bytes = (uint32_t)t.bn * 128u;
  // Large M: each weight tile feeds M / 256 activation tiles, so dequantizing
  // it per tile would repeat the work that many times; form the operand once.
  t.pre = p.M >= kPreM && p.N % 8 == 0 && p.N >= 64 ? 1 : 0;
  if (t.pre) t.raw_bytes = 0;
  // Blocked-along-K scales are staged per stage by TMA: ceil(64 / block) rows
  // of 128 columns (the stage start is block-aligned when block >= 64).
  const uint32_t s_esz = p.s_f16 ? 2u : 4u;
  const bool s_ok = p.slayout == kScaleAxis0Block && t.mode != kModeGeneric &&
                    (p.block % DT_BK == 0 || DT_BK % p.block == 0) &&
                    ((uint64_t)p.N * s_esz) % 16 == 0;
  t.s_rows = s_ok && !t.pre ? (p.block >= DT_BK ? 1 : (int)(DT_BK / p.block)) : 0;
  t.s_bytes = (uint32_t)t.s_rows * DT_BM * s_esz;
  t.stage_bytes = DT_AOP_BYTES + t.b_bytes + t.raw_bytes + t.s_bytes;
  t.stage_bytes = (t.stage_bytes + 1023) & ~1023u;
  // Decode-range batches (bn <= 64) run two CTAs per SM (about 100 KB of ring
  // each), so two sets of dequantizing warps share an SM and split-K fills
  // both slots; wider activation tiles (a stage of 35 KB or more) keep one CTA
  // with a deeper ring, as does the prefill (pre-dequantized) GEMM.
  const size_t budget = (t.pre || t.bn > 64) ? 220 * 1024 : 100 * 1024;
  t.stages = (int)std::min<size_t>(6, budget / t.stage_bytes);
  t.smem = (size_t)t.stages * t.stage_bytes + 1024 + 256;
  const int64_t ntiles = (p.N + DT_BM - 1) / DT_BM, mtiles = (p.M + t.bn - 1) / t.bn;
  const int sms = sm_count();
  int64_t split = 1;
  if (ntiles * mtiles < 2 * sms && ntiles * mtiles <= (int64_t)kMaxCounters) {
    // one CTA per SM (the ring takes most of shared memory): stay within one wave
    split = (t.pre ? 1 : 2) * sms / (ntiles * mtiles);
    const int64_t maxsplit = (p.K + 4 * DT_BK - 1) / (4 * DT_BK); // >= 4 stages per split
    if (split > maxsplit) split = maxsplit;
    if (split < 1) split = 1;
  }
  int64_t kchunk = (p.K + split - 1) / split;
  kchunk = (kchunk + DT_BK - 1) / DT_BK * DT_BK;
  t.kchunk = kchunk;
  t.ksplit = (int)((p.K + kchunk - 1) / kchunk);
  t.grid = dim3((unsigned)ntiles, (unsigned)mtiles, (unsigned)t.ksplit);
  // About 32 MB of activation rows per group (L2 is 126 MB): the group's row
  // tiles stay resident while the weight tiles stream past them once.
  t.group_m = 1;
  if (t.ksplit == 1) {
    const int64_t tile_bytes = (int64_t)t.bn * p.K * 2;
    t.group_m = (int)std::max<int64_t>(1, std::min<int64_t>(mtiles, (32ll << 20) / tile_bytes));
  }
  return t;
}

bool dq_tc_supported(const DqMmParams &p) { return p.M > 4 && dq_tc_eligible(p); }

bool dq_tc_eligible(const DqMmParams &p) {
  if (p.ydt != kFloat16 && p.ydt != kBfloat16) return false;
  // TMA: activation rows K * 2 bytes and packed weight rows must be 16-byte multiples.
  if ((p.K * 2) % 16 != 0) return false;
  // Large M reads the weight through the dequantized 16-bit operand only.
  if (p.M >= kPreM && p.N % 8 == 0 && p.N >= 64 && p.K >= DT_BK) return true;
  const int mode = dq_tc_mode(p);
  const int64_t wrow = mode == kModeF8 ? p.N : p.N / 2;
  if (mode != kModeGeneric && ((wrow % 16) != 0 || (p.N % 2) != 0)) return false;
  if (mode == kModeGeneric && (p.N % 8) != 0) return false;
  if (mode == kModeI4H && p.slayout != kScaleTensor && (p.N % 8) != 0) return false;
  return p.K >= DT_BK && p.N >= 8;
}

size_t dq_tc_workspace(const DqMmParams &p) {
  const TcPlan t = tc_plan(p);
  size_t ws = kCounterBytes;
  if (t.pre) ws += ((size_t)p.K * p.N * 2 + 1023) & ~(size_t)1023; // 16-bit operand
  if (t.ksplit > 1) ws += (size_t)t.ksplit * p.M * p.N * 4;
  return ws;
}

int dq_tc_launch(const DqMmParams &pin, void *workspace, cudaStream_t st, uint64_t wait_ns,
                 bool no_loads) {
  const TcPlan t = tc_plan(pin);
  DqTcArgs a{};
  a.p = pin;
  a.p.kchunk = t.kchunk;
  a.p.ksplit = t.ksplit;
  a.wait_ns = wait_ns;
  a.no_loads = no_loads ? 1 : 0;
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  uint16_t *w16 = t.pre ? reinterpret_cast<uint16_t *>(ws + kCounterBytes) : nullptr;
  const size_t pre_bytes = t.pre ? (((size_t)pin.K * pin.N * 2 + 1023) & ~(size_t)1023) : 0;
  if (t.ksplit > 1) {
    a.p.counters = reinterpret_cast<uint32_t *>(ws);
    a.p.partials = reinterpret_cast<float *>(ws + kCounterBytes + pre_bytes);
  }
  a.bn = t.bn;
  a.stages = t.stages;
  a.mode = t.mode;
  a.raw_bytes = t.raw_bytes;
  a.b_bytes = t.b_bytes;
  a.stage_bytes = t.stage_bytes;
  a.s_bytes = t.s_bytes;
  a.s_rows = t.s_rows;
  a.op_bf16 = pin.ydt == kBfloat16;
  a.group_m = t.group_m;
  CUtensorMap map_a, map_w, map_s;
  if (t.s_bytes) {
    // scales [K / block, N] (FLOAT16 or FLOAT), box 128 columns x s_rows rows
    const uint64_t esz = pin.s_f16 ? 2 : 4;
    const uint64_t dims[2] = {(uint64_t)pin.N, (uint64_t)(pin.K / pin.block)};
    const uint64_t strides[1] = {(uint64_t)pin.N * esz};
    const uint32_t box[2] = {(uint32_t)DT_BM, (uint32_t)t.s_rows};
    int rc = make_tensor_map(&map_s, pin.s_f16 ? CU_TENSOR_MAP_DATA_TYPE_UINT16 : CU_TENSOR_MAP_DATA_TYPE_UINT32,
                             2, pin.scale, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
  }
  {
    // activations [M, K] 16-bit, K innermost; box 64 k x bn rows, 128-byte swizzle
    const uint64_t dims[2] = {(uint64_t)pin.K, (uint64_t)pin.M};
    const uint64_t strides[1] = {(uint64_t)pin.K * 2};
    const uint32_t box[2] = {64, (uint32_t)t.bn};
    int rc = make_tensor_map(&map_a, a.op_bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                             2, pin.a, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  {
    // packed weights as bytes [K, row_bytes]; box 128 n (64 or 128 bytes) x 64 k
    const bool is8 = t.mode == kModeF8;
    const uint64_t row = is8 ? (uint64_t)pin.N : (uint64_t)pin.N / 2;
    const uint64_t dims[2] = {row, (uint64_t)pin.K};
    const uint64_t strides[1] = {row};
    const uint32_t box[2] = {is8 ? 128u : 64u, (uint32_t)DT_BK};
    if (t.mode == kModeGeneric || t.pre) {
      // the generic path reads weights with plain loads; the pre path builds
      // its own map over the operand
      map_w = map_a;
    } else {
      int rc = make_tensor_map(&map_w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, pin.w, dims, strides, box,
                               CU_TENSOR_MAP_SWIZZLE_NONE);
      if (rc) return rc;
    }
  }
  if (!t.s_bytes) map_s = map_a; // unused
  if (t.pre) {
    // 1) the operand, once
    const int64_t groups = pin.K * (pin.N / 8);
    const unsigned blocks = (unsigned)std::min<int64_t>((groups + 255) / 256, (int64_t)sm_count() * 16);
    auto op_kern = t.mode == kModeI4H ? dq_operand_kernel<kModeI4H>
                   : t.mode == kModeF8 ? dq_operand_kernel<kModeF8>
                   : t.mode == kModeF4 ? dq_operand_kernel<kModeF4>
                                       : dq_operand_kernel<kModeGeneric>;
    op_kern<<<blocks, 256, 0, st>>>(a, w16);
    B2_LAUNCH_CHECK();
    // 2) the GEMM on it: [K, N] 16-bit, boxes of 64 n x 64 k with the 128-byte swizzle
    const uint64_t dims[2] = {(uint64_t)pin.N, (uint64_t)pin.K};
    const uint64_t strides[1] = {(uint64_t)pin.N * 2};
    const uint32_t box[2] = {64, (uint32_t)DT_BK};
    int rc = make_tensor_map(&map_w, a.op_bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                             2, w16, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    a.mode = kModePre;
    a.raw_bytes = 0;
    a.s_bytes = 0;
    auto kern = dq_gemm_tc_kernel<kModePre>;
    B2_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)t.smem));
    kern<<<t.grid, DT_THREADS, t.smem, st>>>(map_w, map_a, map_a, a);
    B2_LAUNCH_CHECK();
    return B2_OK;
  }
  auto kern = t.mode == kModeI4H ? dq_gemm_tc_kernel<kModeI4H>
              : t.mode == kModeF8  ? dq_gemm_tc_kernel<kModeF8>
              : t.mode == kModeF4  ? dq_gemm_tc_kernel<kModeF4>
                                   : dq_gemm_tc_kernel<kModeGeneric>;
  B2_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)t.smem));
  kern<<<t.grid, DT_THREADS, t.smem, st>>>(map_w, map_a, map_s, a);
  B2_LAUNCH_CHECK();
  return B2_OK;
}

int dq_tc_ksplit(const DqMmParams &p) { return tc_plan(p).ksplit; }

int status_read_dq_gemm_tc(int reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_dq_gemm_tc_status, sizeof(int)) != cudaSuccess) return -1;
  if (reset) {
    const int z = 0;
    if (cudaMemcpyToSymbol(g_dq_gemm_tc_status, &z, sizeof(int)) != cudaSuccess) return -1;
  }
  return v;
}

} // namespace b2
