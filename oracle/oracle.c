/*
 * CPU ORACLE — test infrastructure only.
 *
 * A plain-C restatement of onnx-light's CPU kernels for the quantized-inference
 * path (DequantizeLinear, MatMul, MatMulInteger, QLinearMatMul, Attention) plus
 * the reference's SplitMix64 input generators.  It is the checker the CUDA
 * path is compared against; nothing in the shipped library links or calls it.
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg may
 * load it.
 *
 * Parity pins: this file is checked against (a) the known-answer vectors
 * written in the reference's own tests (tests/golden/kat_reference_tests.json)
 * and (b) fixtures produced by the reference kernels themselves, compiled from
 * the reference sources into oracle/_ref (tests/golden/make_golden.py).
 *
 * Every function names the reference file:line it restates.  Paths are
 * relative to the onnx-light source tree.
 *
 * Build: gcc -O2 -std=c11 -fPIC -shared -ffp-contract=off -fno-fast-math
 * (no FMA contraction: the reference computes each product and sum with its
 * own rounding).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORC_OK 0
#define ORC_EINVAL -1
#define ORC_EDTYPE -2

/* ONNX TensorProto.DataType codes (onnx_proto/include/onnx_proto/onnx.h:300-330). */
enum {
  DT_FLOAT = 1, DT_UINT8 = 2, DT_INT8 = 3, DT_UINT16 = 4, DT_INT16 = 5, DT_INT32 = 6,
  DT_INT64 = 7, DT_BOOL = 9, DT_FLOAT16 = 10, DT_DOUBLE = 11, DT_UINT32 = 12, DT_UINT64 = 13,
  DT_BFLOAT16 = 16, DT_F8E4M3FN = 17, DT_F8E4M3FNUZ = 18, DT_F8E5M2 = 19, DT_F8E5M2FNUZ = 20,
  DT_UINT4 = 21, DT_INT4 = 22, DT_F4E2M1 = 23, DT_F8E8M0 = 24, DT_UINT2 = 25, DT_INT2 = 26,
  DT_F6E2M3 = 27, DT_F6E3M2 = 28
};

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* ------------------------------------------------------------------------ */
/* Scalar conversions                                                        */
/* ------------------------------------------------------------------------ */

/* IEEE binary32 -> binary16, round-to-nearest-even, subnormals kept, NaN
 * collapsed to sign|0x7e00 (cast_helper.cc:51-87). */
uint16_t orc_f32_to_f16(float f) {
  const uint32_t u = f2u(f);
  const uint32_t sign = (u >> 16) & 0x8000u;
  const int32_t exp32 = (int32_t)((u >> 23) & 0xffu);
  const uint32_t man = u & 0x7fffffu;
  if (exp32 == 0xff) return (uint16_t)(sign | 0x7c00u | (man ? 0x200u : 0u));
  const int32_t e = exp32 - 127 + 15;
  if (e >= 31) return (uint16_t)(sign | 0x7c00u);
  if (e <= 0) {
    if (e < -10) return (uint16_t)sign;
    const uint32_t full = man | 0x800000u;
    const uint32_t sh = (uint32_t)(14 - e);
    const uint32_t rem = full & ((1u << sh) - 1u);
    const uint32_t half = 1u << (sh - 1u);
    uint16_t h = (uint16_t)(sign | (full >> sh));
    if (rem > half || (rem == half && (h & 1u))) h = (uint16_t)(h + 1u);
    return h;
  }
  const uint32_t rem = man & 0x1fffu;
  uint16_t h = (uint16_t)(sign | ((uint32_t)e << 10) | (man >> 13));
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h = (uint16_t)(h + 1u);
  return h;
}

/* binary16 -> binary32, exact (cast_helper.cc:89-122). */
float orc_f16_to_f32(uint16_t h) {
  const uint32_t sign = ((uint32_t)h >> 15) & 1u;
  const uint32_t ex = ((uint32_t)h >> 10) & 0x1fu;
  const uint32_t man = (uint32_t)h & 0x3ffu;
  uint32_t out;
  if (ex == 0) {
    if (man == 0) {
      out = sign << 31;
    } else {
      uint32_t m = man;
      int32_t e = 1;
      while (!(m & 0x400u)) { m <<= 1; --e; }
      out = (sign << 31) | ((uint32_t)(e - 15 + 127) << 23) | ((m & 0x3ffu) << 13);
    }
  } else if (ex == 0x1f) {
    out = (sign << 31) | 0x7f800000u | (man << 13);
  } else {
    out = (sign << 31) | ((ex - 15 + 127) << 23) | (man << 13);
  }
  return u2f(out);
}

/* binary32 -> bfloat16, RNE with quiet NaN (cast_helper.cc:124-135). */
uint16_t orc_f32_to_bf16(float f) {
  const uint32_t u = f2u(f);
  if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x7fffffu)) return (uint16_t)((u >> 16) | 0x40u);
  return (uint16_t)((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
}

float orc_bf16_to_f32(uint16_t b) { return u2f((uint32_t)b << 16); }

/* FLOAT8E4M3FN -> binary32; 0x7f/0xff are NaN (cast_float8.cc:83-120). */
float orc_f8e4m3fn_to_f32(uint8_t v) {
  if (v == 0xff) return u2f(0xffc00000u);
  if (v == 0x7f) return u2f(0x7fc00000u);
  const uint32_t sign = (uint32_t)(v & 0x80u) << 24;
  const uint32_t ex = (v >> 3) & 0xfu, man = v & 7u;
  if (ex == 0) {
    /* subnormal: man * 2^-9 */
    if (man == 0) return u2f(sign);
    const float mag = (float)man * (1.0f / 512.0f);
    return u2f(sign | f2u(mag));
  }
  return u2f(sign | ((ex - 7u + 127u) << 23) | (man << 20));
}

/* FLOAT8E4M3FNUZ -> binary32; bias 8, 0x80 is NaN (cast_float8.cc:174-205). */
float orc_f8e4m3fnuz_to_f32(uint8_t v) {
  if (v == 0x80) return u2f(0xffc00000u);
  const uint32_t sign = (uint32_t)(v & 0x80u) << 24;
  const uint32_t ex = (v >> 3) & 0xfu, man = v & 7u;
  if (ex == 0) {
    if (man == 0) return u2f(sign);
    return u2f(sign | f2u((float)man * (1.0f / 1024.0f)));
  }
  return u2f(sign | ((ex - 8u + 127u) << 23) | (man << 20));
}

/* FLOAT8E5M2 -> binary32; infinities at 0x7c/0xfc, NaN above (cast_float8.cc:263-296). */
float orc_f8e5m2_to_f32(uint8_t v) {
  if (v >= 253) return u2f(0xffc00000u);
  if (v >= 125 && v <= 127) return u2f(0x7fc00000u);
  if (v == 252) return u2f(0xff800000u);
  if (v == 124) return u2f(0x7f800000u);
  const uint32_t sign = (uint32_t)(v & 0x80u) << 24;
  const uint32_t ex = (v >> 2) & 0x1fu, man = v & 3u;
  if (ex == 0) {
    if (man == 0) return u2f(sign);
    return u2f(sign | f2u((float)man * (1.0f / 65536.0f)));
  }
  return u2f(sign | ((ex - 15u + 127u) << 23) | (man << 21));
}

/* FLOAT8E5M2FNUZ -> binary32; bias 16, 0x80 is NaN (cast_float8.cc:347-375). */
float orc_f8e5m2fnuz_to_f32(uint8_t v) {
  if (v == 0x80) return u2f(0xffc00000u);
  const uint32_t sign = (uint32_t)(v & 0x80u) << 24;
  const uint32_t ex = (v >> 2) & 0x1fu, man = v & 3u;
  if (ex == 0) {
    if (man == 0) return u2f(sign);
    return u2f(sign | f2u((float)man * (1.0f / 131072.0f)));
  }
  return u2f(sign | ((ex - 16u + 127u) << 23) | (man << 21));
}

/* binary32 -> FLOAT8E4M3FN, saturating, round-to-nearest-even; NaN -> 0x7f|sign,
 * +-inf -> +-448.  Used to synthesise fp8 weights (the reference generator
 * applies FloatToFloat8E4M3FNBits, cast_float8.cc:27-80, to Randn samples). */
uint8_t orc_f32_to_f8e4m3fn(float f) {
  const uint32_t u = f2u(f);
  const uint8_t sign = (uint8_t)((u >> 24) & 0x80u);
  if ((u & 0x7fffffffu) == 0x7f800000u) return (uint8_t)(sign | 0x7eu);
  if ((u & 0x7f800000u) == 0x7f800000u) return (uint8_t)(sign | 0x7fu);
  const float a = fabsf(f);
  if (a >= 464.0f) return (uint8_t)(sign | 0x7eu); /* beyond the 448 rounding band */
  /* Representable grid: subnormals k*2^-9 (k<8), normals (8+m)*2^(e-10). */
  int e;
  frexpf(a, &e); /* a = fr * 2^e, fr in [0.5,1) */
  int q = e - 4;  /* spacing exponent for normals: ulp = 2^(e-1-3) */
  if (q < -9) q = -9;
  const float ulp = ldexpf(1.0f, q);
  const float k = a / ulp; /* exact: power-of-two division */
  float r = nearbyintf(k); /* default rounding mode is ties-to-even */
  float val = r * ulp;
  if (val > 448.0f) val = 448.0f;
  /* encode val */
  if (val == 0.0f) return sign;
  if (val < ldexpf(1.0f, -6)) return (uint8_t)(sign | (uint8_t)(val * 512.0f));
  int ve;
  const float fr = frexpf(val, &ve); /* val = fr*2^ve, fr in [0.5,1) */
  const uint32_t biased = (uint32_t)(ve - 1 + 7);
  const uint32_t man = (uint32_t)((fr * 2.0f - 1.0f) * 8.0f);
  return (uint8_t)(sign | (biased << 3) | man);
}

/* FLOAT4E2M1 nibble -> binary32 table (cast_helper.cc:161-166). */
static const float kF4[16] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f,
                              -0.0f, -0.5f, -1.0f, -1.5f, -2.0f, -3.0f, -4.0f, -6.0f};
float orc_f4e2m1_to_f32(uint8_t nib) { return kF4[nib & 0xfu]; }

/* FLOAT6 -> binary32 (cast_helper.cc:208-219). */
static float f6_to_f32(uint8_t bits, int dtype) {
  const int mb = dtype == DT_F6E2M3 ? 3 : 2;
  const int eb = 5 - mb;
  const int bias = (1 << (eb - 1)) - 1;
  const int ex = (bits >> mb) & ((1 << eb) - 1);
  const int man = bits & ((1 << mb) - 1);
  const float v = ex == 0 ? ldexpf((float)man, 1 - bias - mb)
                          : ldexpf(1.0f + (float)man / (float)(1 << mb), ex - bias);
  return (bits & 0x20u) ? -v : v;
}

/* Sub-byte readers (cast_sub_byte.h:57-60, 72-76; cast_helper.cc:247-255). */
static inline uint8_t read4(const uint8_t *p, int64_t i) {
  const uint8_t b = p[i / 2];
  return (uint8_t)((i % 2 == 0) ? (b & 0xfu) : ((b >> 4) & 0xfu));
}
static inline uint8_t read2(const uint8_t *p, int64_t i) {
  return (uint8_t)((p[i / 4] >> ((i % 4) * 2)) & 3u);
}
static inline uint8_t read6(const uint8_t *p, int64_t i) {
  const size_t bo = (size_t)i * 6, by = bo / 8;
  const int sh = (int)(bo % 8);
  uint16_t v = (uint16_t)(p[by] >> sh);
  if (sh > 2) v |= (uint16_t)(p[by + 1] << (8 - sh));
  return (uint8_t)(v & 0x3fu);
}

/* ------------------------------------------------------------------------ */
/* SplitMix64 generators (random.cc:38-45, 61-89, 92-107, 141-176)           */
/* ------------------------------------------------------------------------ */

static inline uint64_t sm_next(uint64_t *state) {
  *state += 0x9E3779B97F4A7C15ULL;
  uint64_t z = *state;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}
static inline double sm_unit(uint64_t v) { return (double)(v >> 11) * (1.0 / 9007199254740992.0); }

/* RandUniformInto<float>: low + float(u) * float(high-low). */
void orc_rand_uniform_f32(uint64_t seed, int64_t n, double lo, double hi, float *out) {
  uint64_t st = seed;
  const float span = (float)(hi - lo), lowf = (float)lo;
  for (int64_t i = 0; i < n; ++i) out[i] = lowf + (float)sm_unit(sm_next(&st)) * span;
}

/* RandNormalInto<float>: mean + float(sum of 12 uniforms - 6) * scale. */
void orc_randn_f32(uint64_t seed, int64_t n, double mean, double scale, float *out) {
  uint64_t st = seed;
  const float m = (float)mean, s = (float)scale;
  for (int64_t i = 0; i < n; ++i) {
    double acc = 0.0;
    for (int j = 0; j < 12; ++j) acc += sm_unit(sm_next(&st));
    out[i] = m + (float)(acc - 6.0) * s;
  }
}

/* RandInt(low, high): rejection sampling on [0, span). */
void orc_randint(uint64_t seed, int64_t n, int64_t lo, int64_t hi_exclusive, int64_t *out) {
  uint64_t st = seed;
  const uint64_t span = (uint64_t)(hi_exclusive - lo);
  const uint64_t mod = (0ULL - span) % span;
  const uint64_t limit = 0ULL - mod;
  for (int64_t i = 0; i < n; ++i) {
    uint64_t v;
    for (;;) {
      v = sm_next(&st);
      if (limit == 0 || v < limit) break;
    }
    out[i] = (int64_t)(v % span) + lo;
  }
}

/* ------------------------------------------------------------------------ */
/* Element decode helpers shared by the DequantizeLinear oracle              */
/* ------------------------------------------------------------------------ */

static int is_f8(int dt) {
  return dt == DT_F8E4M3FN || dt == DT_F8E4M3FNUZ || dt == DT_F8E5M2 || dt == DT_F8E5M2FNUZ;
}
static float dec_f8(int dt, uint8_t v) {
  switch (dt) {
  case DT_F8E4M3FN: return orc_f8e4m3fn_to_f32(v);
  case DT_F8E4M3FNUZ: return orc_f8e4m3fnuz_to_f32(v);
  case DT_F8E5M2: return orc_f8e5m2_to_f32(v);
  default: return orc_f8e5m2fnuz_to_f32(v);
  }
}

/* Value of element i of a quantized tensor as float, exactly as the
 * reference's typed loops convert it (kernel_dequantizelinear.cc:65-159,
 * 246-328): whole-byte/word integers via static_cast<float>, sub-byte via the
 * nibble converters, float8/float4/float6 via their decoders. */
static float qval(int dt, const uint8_t *p, int64_t i) {
  switch (dt) {
  case DT_UINT8: return (float)p[i];
  case DT_INT8: return (float)(int8_t)p[i];
  case DT_UINT16: { uint16_t v; memcpy(&v, p + 2 * i, 2); return (float)v; }
  case DT_INT16: { int16_t v; memcpy(&v, p + 2 * i, 2); return (float)v; }
  case DT_INT32: { int32_t v; memcpy(&v, p + 4 * i, 4); return (float)v; }
  case DT_UINT4: return (float)read4(p, i);
  case DT_INT4: { const uint8_t n = read4(p, i); return (float)((n & 8u) ? (int)n - 16 : (int)n); }
  case DT_UINT2: return (float)read2(p, i);
  case DT_INT2: { const uint8_t n = read2(p, i); return (float)((n & 2u) ? (int)n - 4 : (int)n); }
  case DT_F4E2M1: return kF4[read4(p, i)];
  case DT_F6E2M3: case DT_F6E3M2: return f6_to_f32(read6(p, i), dt);
  default: return dec_f8(dt, p[i]);
  }
}

static int dq_supported(int dt) {
  return dt == DT_UINT8 || dt == DT_INT8 || dt == DT_UINT16 || dt == DT_INT16 || dt == DT_INT32 ||
         is_f8(dt) || dt == DT_UINT4 || dt == DT_INT4 || dt == DT_UINT2 || dt == DT_INT2 ||
         dt == DT_F4E2M1 || dt == DT_F6E2M3 || dt == DT_F6E3M2;
}

static float read_scale(int sdt, const uint8_t *s, int64_t i) {
  if (sdt == DT_FLOAT16) { uint16_t h; memcpy(&h, s + 2 * i, 2); return orc_f16_to_f32(h); }
  float f; memcpy(&f, s + 4 * i, 4); return f;
}

static int64_t numel(const int64_t *shape, int nd) {
  int64_t n = 1;
  for (int d = 0; d < nd; ++d) n *= shape[d];
  return n;
}

/*
 * DequantizeLinear (kernel_dequantizelinear.cc:332-693).
 *
 * x: quantized bytes, dtype x_dt, shape x_shape[x_nd].
 * scale: FLOAT or FLOAT16 bytes with shape s_shape[s_nd].
 * zp: optional (NULL = absent, which the reference turns into a zero-filled
 *     zero point of the scale's shape, :670-693), dtype must equal x_dt.
 * y: output bytes, FLOAT when the scale is FLOAT, FLOAT16 when it is FLOAT16.
 *
 * Layout: scale element count 1 -> per-tensor (:349-502); rank(scale) ==
 * rank(x) -> blocked along `axis` with block x_shape[axis]/s_shape[axis]
 * (:548-559, :199-235); otherwise per-axis (:560-565, :237-243).  The value is
 * (float(x) - float(zp)) * scale in fp32, then rounded to fp16 when the
 * output is FLOAT16 (:57-63).
 */
int orc_dequantize_linear(const uint8_t *x, int x_dt, const int64_t *x_shape, int x_nd,
                          const uint8_t *scale, int s_dt, const int64_t *s_shape, int s_nd,
                          const uint8_t *zp, int zp_dt, const int64_t *zp_shape, int zp_nd,
                          int64_t axis, uint8_t *y) {
  if (s_dt != DT_FLOAT && s_dt != DT_FLOAT16) return ORC_EINVAL;
  const int64_t n = numel(x_shape, x_nd);
  const int64_t sn = numel(s_shape, s_nd);
  const int f16out = s_dt == DT_FLOAT16;
  if (zp && zp_dt != x_dt) return ORC_EINVAL;
  if (!dq_supported(x_dt)) return ORC_EDTYPE;
  if (sn == 1) {
    /* Per-tensor: zero point must be a scalar too (:430-431). */
    if (zp && numel(zp_shape, zp_nd) != 1) return ORC_EINVAL;
    const float s = read_scale(s_dt, scale, 0);
    const float z = zp ? qval(x_dt, zp, 0) : 0.0f;
    for (int64_t i = 0; i < n; ++i) {
      const float v = (qval(x_dt, x, i) - z) * s;
      if (f16out) { const uint16_t h = orc_f32_to_f16(v); memcpy(y + 2 * i, &h, 2); }
      else memcpy(y + 4 * i, &v, 4);
    }
    return ORC_OK;
  }
  if (axis < 0 || axis >= x_nd) return ORC_EINVAL;
  if (zp) {
    if (zp_nd != s_nd) return ORC_EINVAL;
    for (int d = 0; d < s_nd; ++d) if (zp_shape[d] != s_shape[d]) return ORC_EINVAL;
  }
  int64_t outer = 1, inner = 1;
  for (int d = 0; d < axis; ++d) outer *= x_shape[d];
  for (int d = (int)axis + 1; d < x_nd; ++d) inner *= x_shape[d];
  const int64_t alen = x_shape[axis];
  int64_t s_alen, block;
  if (s_nd == x_nd) {
    for (int d = 0; d < x_nd; ++d) {
      if (!(s_shape[d] > 0 && x_shape[d] % s_shape[d] == 0)) return ORC_EINVAL;
      if (!(d == axis || s_shape[d] == x_shape[d])) return ORC_EINVAL;
    }
    s_alen = s_shape[axis];
    block = alen / s_alen;
  } else {
    if (sn != alen) return ORC_EINVAL;
    s_alen = alen;
    block = 1;
  }
  for (int64_t i = 0; i < n; ++i) {
    const int64_t in = i % inner;
    const int64_t k = (i / inner) % alen;
    const int64_t o = i / (inner * alen);
    const int64_t si = (s_nd == x_nd) ? (o * s_alen + k / block) * inner + in : k;
    const float s = read_scale(s_dt, scale, si);
    const float z = zp ? qval(x_dt, zp, si) : 0.0f;
    const float v = (qval(x_dt, x, i) - z) * s;
    if (f16out) { const uint16_t h = orc_f32_to_f16(v); memcpy(y + 2 * i, &h, 2); }
    else memcpy(y + 4 * i, &v, 4);
  }
  return ORC_OK;
}

/* ------------------------------------------------------------------------ */
/* MatMul shape rules (matmul_shape_utils.h:24-108)                          */
/* ------------------------------------------------------------------------ */

typedef struct {
  int64_t M, K, N, batch;
  int out_nd;
  int64_t out_shape[16];
  int64_t *a_base, *b_base; /* per-batch element offsets (caller frees) */
} mm_plan;

static void plan_free(mm_plan *p) { free(p->a_base); free(p->b_base); }

static int mm_plan_make(const int64_t *as, int an, const int64_t *bs, int bn, mm_plan *p) {
  if (an < 1 || bn < 1 || an > 12 || bn > 12) return ORC_EINVAL;
  int64_t a2[14], b2[14];
  int a2n, b2n;
  if (an == 1) { a2[0] = 1; a2[1] = as[0]; a2n = 2; } else { memcpy(a2, as, an * 8); a2n = an; }
  if (bn == 1) { b2[0] = bs[0]; b2[1] = 1; b2n = 2; } else { memcpy(b2, bs, bn * 8); b2n = bn; }
  if (a2[a2n - 1] != b2[b2n - 2]) return ORC_EINVAL;
  p->M = a2[a2n - 2]; p->K = a2[a2n - 1]; p->N = b2[b2n - 1];
  const int ap = a2n - 2, bp = b2n - 2;
  const int r = ap > bp ? ap : bp;
  int64_t outp[12];
  for (int i = 0; i < r; ++i) {
    const int64_t da = i + ap >= r ? a2[i - (r - ap)] : 1;
    const int64_t db = i + bp >= r ? b2[i - (r - bp)] : 1;
    if (da == db || da == 1) outp[i] = db;
    else if (db == 1) outp[i] = da;
    else return ORC_EINVAL;
  }
  p->out_nd = 0;
  for (int i = 0; i < r; ++i) p->out_shape[p->out_nd++] = outp[i];
  if (an != 1) p->out_shape[p->out_nd++] = p->M;
  if (bn != 1) p->out_shape[p->out_nd++] = p->N;
  p->batch = 1;
  for (int i = 0; i < r; ++i) p->batch *= outp[i];
  p->a_base = (int64_t *)calloc((size_t)(p->batch ? p->batch : 1), 8);
  p->b_base = (int64_t *)calloc((size_t)(p->batch ? p->batch : 1), 8);
  /* row-major strides of the promoted operands */
  int64_t ast[14], bst[14];
  ast[a2n - 1] = 1;
  for (int i = a2n - 2; i >= 0; --i) ast[i] = ast[i + 1] * a2[i + 1];
  bst[b2n - 1] = 1;
  for (int i = b2n - 2; i >= 0; --i) bst[i] = bst[i + 1] * b2[i + 1];
  for (int64_t bt = 0; bt < p->batch; ++bt) {
    int64_t rem = bt, ab = 0, bb = 0;
    for (int d = r - 1; d >= 0; --d) {
      const int64_t c = rem % outp[d];
      rem /= outp[d];
      if (d + ap >= r) { const int ad = d - (r - ap); ab += (a2[ad] == 1 ? 0 : c) * ast[ad]; }
      if (d + bp >= r) { const int bd = d - (r - bp); bb += (b2[bd] == 1 ? 0 : c) * bst[bd]; }
    }
    p->a_base[bt] = ab;
    p->b_base[bt] = bb;
  }
  return ORC_OK;
}

/* MatMul output shape, for callers that allocate (matmul_shape_utils.h:86-106). */
int orc_matmul_shape(const int64_t *as, int an, const int64_t *bs, int bn, int64_t *out, int *out_nd) {
  mm_plan p;
  const int rc = mm_plan_make(as, an, bs, bn, &p);
  if (rc) return rc;
  memcpy(out, p.out_shape, (size_t)p.out_nd * 8);
  *out_nd = p.out_nd;
  plan_free(&p);
  return ORC_OK;
}

/*
 * MatMul for FLOAT / FLOAT16 / BFLOAT16 (kernel_matmul.cc:60-147, 181-223).
 * Half inputs are promoted to fp32 (float16_promote.cc), multiplied with fp32
 * accumulation in increasing k order per output element (:133-142), then
 * rounded back with RNE.
 */
int orc_matmul(const void *a, const int64_t *as, int an, const void *b, const int64_t *bs, int bn,
               int dt, void *y) {
  if (dt != DT_FLOAT && dt != DT_FLOAT16 && dt != DT_BFLOAT16) return ORC_EDTYPE;
  mm_plan p;
  int rc = mm_plan_make(as, an, bs, bn, &p);
  if (rc) return rc;
  const int64_t M = p.M, K = p.K, N = p.N;
  float *acc = (float *)malloc((size_t)(N ? N : 1) * 4);
  for (int64_t bt = 0; bt < p.batch; ++bt) {
    for (int64_t i = 0; i < M; ++i) {
      for (int64_t j = 0; j < N; ++j) acc[j] = 0.0f;
      for (int64_t k = 0; k < K; ++k) {
        const int64_t ai = p.a_base[bt] + i * K + k;
        float av;
        if (dt == DT_FLOAT) av = ((const float *)a)[ai];
        else if (dt == DT_FLOAT16) av = orc_f16_to_f32(((const uint16_t *)a)[ai]);
        else av = orc_bf16_to_f32(((const uint16_t *)a)[ai]);
        const int64_t brow = p.b_base[bt] + k * N;
        for (int64_t j = 0; j < N; ++j) {
          float bv;
          if (dt == DT_FLOAT) bv = ((const float *)b)[brow + j];
          else if (dt == DT_FLOAT16) bv = orc_f16_to_f32(((const uint16_t *)b)[brow + j]);
          else bv = orc_bf16_to_f32(((const uint16_t *)b)[brow + j]);
          const float prod = av * bv;
          acc[j] = acc[j] + prod;
        }
      }
      const int64_t yo = (bt * M + i) * N;
      for (int64_t j = 0; j < N; ++j) {
        if (dt == DT_FLOAT) ((float *)y)[yo + j] = acc[j];
        else if (dt == DT_FLOAT16) ((uint16_t *)y)[yo + j] = orc_f32_to_f16(acc[j]);
        else ((uint16_t *)y)[yo + j] = orc_f32_to_bf16(acc[j]);
      }
    }
  }
  free(acc);
  plan_free(&p);
  return ORC_OK;
}

/* Reads element idx of an INT8/UINT8 tensor as int32 (kernel_matmul_integer.cc:27-32). */
static inline int32_t rd8(int dt, const uint8_t *p, int64_t i) {
  return dt == DT_INT8 ? (int32_t)(int8_t)p[i] : (int32_t)p[i];
}

/*
 * MatMulInteger (kernel_matmul_integer.cc:89-229): int32 accumulation of
 * (a - a_zp[i]) * (b - b_zp[j]); a_zp scalar or per-row [M], b_zp scalar or
 * per-column [N]; absent zero points are 0.  Wraparound int32 arithmetic.
 */
int orc_matmul_integer(const uint8_t *a, int a_dt, const int64_t *as, int an,
                       const uint8_t *b, int b_dt, const int64_t *bs, int bn,
                       const uint8_t *azp, int64_t azp_n, const uint8_t *bzp, int64_t bzp_n,
                       int32_t *y) {
  if ((a_dt != DT_INT8 && a_dt != DT_UINT8) || (b_dt != DT_INT8 && b_dt != DT_UINT8)) return ORC_EINVAL;
  mm_plan p;
  int rc = mm_plan_make(as, an, bs, bn, &p);
  if (rc) return rc;
  const int64_t M = p.M, K = p.K, N = p.N;
  if (azp && !(azp_n == 1 || azp_n == M)) { plan_free(&p); return ORC_EINVAL; }
  if (bzp && !(bzp_n == 1 || bzp_n == N)) { plan_free(&p); return ORC_EINVAL; }
  for (int64_t bt = 0; bt < p.batch; ++bt)
    for (int64_t i = 0; i < M; ++i) {
      const int32_t za = azp ? rd8(a_dt, azp, azp_n > 1 ? i : 0) : 0;
      for (int64_t j = 0; j < N; ++j) {
        const int32_t zb = bzp ? rd8(b_dt, bzp, bzp_n > 1 ? j : 0) : 0;
        uint32_t acc = 0; /* int32 wraparound */
        for (int64_t k = 0; k < K; ++k) {
          const int32_t av = rd8(a_dt, a, p.a_base[bt] + i * K + k);
          const int32_t bv = rd8(b_dt, b, p.b_base[bt] + k * N + j);
          acc += (uint32_t)((av - za) * (bv - zb));
        }
        y[(bt * M + i) * N + j] = (int32_t)acc;
      }
    }
  plan_free(&p);
  return ORC_OK;
}

/*
 * QLinearMatMul (kernel_qlinearmatmul.cc:115-267): int64 accumulation, then
 * float(acc) * (a_s * b_s / y_s) in fp32, nearbyint (ties-to-even), + y_zp in
 * fp32, clamp to the output range, truncating cast.  All scalars per-tensor.
 */
int orc_qlinear_matmul(const uint8_t *a, int a_dt, const int64_t *as, int an, float a_s, int32_t a_zp,
                       const uint8_t *b, int b_dt, const int64_t *bs, int bn, float b_s, int32_t b_zp,
                       float y_s, int32_t y_zp, int y_dt, uint8_t *y) {
  if ((a_dt != DT_INT8 && a_dt != DT_UINT8) || (b_dt != DT_INT8 && b_dt != DT_UINT8) ||
      (y_dt != DT_INT8 && y_dt != DT_UINT8))
    return ORC_EINVAL;
  if (y_s == 0.0f) return ORC_EINVAL;
  mm_plan p;
  int rc = mm_plan_make(as, an, bs, bn, &p);
  if (rc) return rc;
  const int64_t M = p.M, K = p.K, N = p.N;
  const float comb = a_s * b_s / y_s;
  const float yz = (float)y_zp;
  const float lo = y_dt == DT_INT8 ? -128.0f : 0.0f, hi = y_dt == DT_INT8 ? 127.0f : 255.0f;
  for (int64_t bt = 0; bt < p.batch; ++bt)
    for (int64_t i = 0; i < M; ++i)
      for (int64_t j = 0; j < N; ++j) {
        int64_t acc = 0;
        for (int64_t k = 0; k < K; ++k)
          acc += (int64_t)(rd8(a_dt, a, p.a_base[bt] + i * K + k) - a_zp) *
                 (int64_t)(rd8(b_dt, b, p.b_base[bt] + k * N + j) - b_zp);
        float v = (float)acc * comb;
        v = nearbyintf(v) + yz;
        if (v < lo) v = lo; else if (v > hi) v = hi;
        int32_t q;
        if (isnan(v)) q = 0; /* x86 cvttss2si yields 0x80000000 -> low byte 0 */
        else q = (int32_t)v;
        y[(bt * M + i) * N + j] = (uint8_t)(q & 0xff);
      }
  plan_free(&p);
  return ORC_OK;
}

/*
 * Attention, rank-4 float32 core (kernel_attention.cc:427-691).
 *
 * Q [B,Hq,Sq,D], K [B,Hkv,L,D], V [B,Hkv,L,Dv] where L is the total KV length
 * (past already concatenated by the caller, kernel_attention.cc:469-471),
 * mask optional float [mb,mh,mq,ml] broadcast per :371-394 with positions
 * j >= ml masked (:396-412; BOOL and half masks are converted to this float
 * form by the caller, :391-392 and :797-801).  GQA kv_h = h / (Hq/Hkv) (:587);
 * causal frontier j > i + offset masked, offset = past_len, or
 * nonpad[b] - Sq when nonpad lengths are given without a past (:572-582);
 * windows measured from the same offset (:594-597); keys j >= nonpad[b]
 * masked (:598-599); softcap applied before the mask (:619-620); max-subtract
 * softmax with a fully-masked row producing zeros (:641-661); Y = sum p*V
 * (:670-678).  qk (optional, [B,Hq,Sq,L]) receives the scores of qk_mode
 * 0 (scaled), 1 (after softcap), 2 (after the mask) or 3 (softmax) (:613-668).
 * The extended-exponent rescue for non-finite scores (:33-158) is not
 * restated: it only triggers on overflowing inputs.
 */
int orc_attention_f32(const float *Q, const float *Kc, const float *Vc, int64_t B, int64_t Hq,
                      int64_t Hkv, int64_t Sq, int64_t L, int64_t D, int64_t Dv, float scale,
                      int is_causal, int64_t past_len, float softcap, const float *mask,
                      const int64_t *mask_shape4, int64_t left_window, int64_t right_window,
                      const int64_t *nonpad, float *qk, int qk_mode, float *Y) {
  if (Hkv <= 0 || Hq % Hkv) return ORC_EINVAL;
  const int64_t group = Hq / Hkv;
  float *sc = (float *)malloc((size_t)(L ? L : 1) * 4);
  for (int64_t b = 0; b < B; ++b)
    for (int64_t h = 0; h < Hq; ++h) {
      const int64_t kvh = h / group;
      const int64_t off = (nonpad && past_len == 0) ? nonpad[b] - Sq : past_len;
      const float *q = Q + ((b * Hq + h) * Sq) * D;
      const float *kk = Kc + ((b * Hkv + kvh) * L) * D;
      const float *vv = Vc + ((b * Hkv + kvh) * L) * Dv;
      float *yy = Y + ((b * Hq + h) * Sq) * Dv;
      for (int64_t i = 0; i < Sq; ++i) {
        float *qkr = qk ? qk + (((b * Hq + h) * Sq) + i) * L : NULL;
        int fully = 1;
        float mx = -INFINITY;
        for (int64_t j = 0; j < L; ++j) {
          float s = 0.0f;
          for (int64_t d = 0; d < D; ++d) s += q[i * D + d] * kk[j * D + d];
          s *= scale;
          if (qkr && qk_mode == 0) qkr[j] = s;
          if (softcap > 0.0f) s = softcap * tanhf(s / softcap);
          if (qkr && qk_mode == 1) qkr[j] = s;
          float bias = 0.0f;
          if (mask) {
            const int64_t ml = mask_shape4[3];
            if (j >= ml) bias = -INFINITY;
            else {
              const int64_t idx[4] = {b, h, i, j};
              int64_t lin = 0, st = 1;
              for (int k = 3; k >= 0; --k) {
                const int64_t c = mask_shape4[k] == 1 ? 0 : idx[k];
                lin += c * st;
                st *= mask_shape4[k];
              }
              bias = mask[lin];
            }
          }
          if (is_causal && j > i + off) bias = -INFINITY;
          const int64_t wd = i + off - j;
          if ((left_window >= 0 && wd > left_window) || (right_window >= 0 && -wd > right_window))
            bias = -INFINITY;
          if (nonpad && j >= nonpad[b]) bias = -INFINITY;
          fully &= isinf(bias) && bias < 0.0f;
          s += bias;
          sc[j] = s;
          if (qkr && qk_mode == 2) qkr[j] = s;
          if (s > mx) mx = s;
        }
        float den = 0.0f;
        for (int64_t j = 0; j < L; ++j) {
          const float e = fully ? 0.0f : expf(sc[j] - mx);
          sc[j] = e;
          den += e;
        }
        const float inv = den != 0.0f ? 1.0f / den : 0.0f;
        for (int64_t j = 0; j < L; ++j) sc[j] *= inv;
        if (qkr && qk_mode == 3)
          for (int64_t j = 0; j < L; ++j) qkr[j] = sc[j];
        for (int64_t dv = 0; dv < Dv; ++dv) {
          float acc = 0.0f;
          for (int64_t j = 0; j < L; ++j) acc += sc[j] * vv[j * Dv + dv];
          yy[i * Dv + dv] = acc;
        }
      }
    }
  free(sc);
  return ORC_OK;
}

/*
 * RMSNormalization on float rows (kernel_rmsnormalization.cc:83-214): for each
 * of `outer` rows of `norm` values, sum of squares in double (increasing
 * index), mean in double, rms = sqrtf((float)mean + eps), n = x / rms; half
 * types (half_dt 10 / 16) round n to their type first (:200-205); y = n * s
 * with the scale already expanded to one value per normalized element.  The
 * caller rounds y to the output type.
 */
void orc_rms_norm_f32(const float *x, const float *s, int64_t outer, int64_t norm, float eps,
                      int half_dt, float *y) {
  for (int64_t o = 0; o < outer; ++o) {
    const float *xr = x + o * norm;
    double sq = 0.0;
    for (int64_t i = 0; i < norm; ++i) sq += (double)xr[i] * (double)xr[i];
    const double mean = norm > 0 ? sq / (double)norm : 0.0;
    const float rms = sqrtf((float)mean + eps);
    for (int64_t i = 0; i < norm; ++i) {
      float n = xr[i] / rms;
      if (half_dt == 10) n = orc_f16_to_f32(orc_f32_to_f16(n));
      else if (half_dt == 16) n = orc_bf16_to_f32(orc_f32_to_bf16(n));
      y[o * norm + i] = n * s[i];
    }
  }
}

/*
 * RotaryEmbedding on float data (kernel_rotary_embedding.cc:151-218): x in the
 * canonical [B, H, S, D] order or, with rank3, stored [B, S, H, D]; cos / sin
 * rows of `half` values picked by pos[b * S + s] (pos != NULL) or by
 * (b * S + s); pairs (i, i + half) or, interleaved, (2i, 2i + 1);
 * y1 = c x1 - s x2, y2 = s x1 + c x2; channels from 2 * half on are copied.
 * Returns ORC_EINVAL for a position outside [0, cache_rows) (the reference
 * throws there).
 */
int orc_rotary_f32(const float *x, const float *cs, const float *sn, const int64_t *pos,
                   int64_t B, int64_t H, int64_t S, int64_t D, int64_t half, int rank3,
                   int interleaved, int64_t cache_rows, float *y) {
  for (int64_t b = 0; b < B; ++b)
    for (int64_t h = 0; h < H; ++h)
      for (int64_t s = 0; s < S; ++s) {
        const int64_t base = rank3 ? ((b * S + s) * H + h) * D : ((b * H + h) * S + s) * D;
        int64_t row = b * S + s;
        if (pos) {
          row = pos[b * S + s];
          if (row < 0 || row >= cache_rows) return ORC_EINVAL;
        }
        const float *cr = cs + row * half, *sr = sn + row * half;
        for (int64_t i = 0; i < half; ++i) {
          const int64_t i1 = interleaved ? base + 2 * i : base + i;
          const int64_t i2 = interleaved ? base + 2 * i + 1 : base + half + i;
          const float x1 = x[i1], x2 = x[i2], c = cr[i], sv = sr[i];
          y[i1] = c * x1 - sv * x2;
          y[i2] = sv * x1 + c * x2;
        }
        for (int64_t i = 2 * half; i < D; ++i) y[base + i] = x[base + i];
      }
  return ORC_OK;
}

/* SwiGLU on floats (kernel_swiglu.cc:13-20): a * (1 / (1 + exp(-alpha a))) * b. */
void orc_swiglu_f32(const float *a, const float *b, int64_t n, float alpha, float *y) {
  for (int64_t i = 0; i < n; ++i) {
    const float sg = 1.0f / (1.0f + expf(-alpha * a[i]));
    y[i] = a[i] * sg * b[i];
  }
}

/* Bulk conversions used by the Python wrapper. */
void orc_f16_to_f32_n(const uint16_t *in, float *out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = orc_f16_to_f32(in[i]);
}
void orc_f32_to_f16_n(const float *in, uint16_t *out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = orc_f32_to_f16(in[i]);
}
void orc_bf16_to_f32_n(const uint16_t *in, float *out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = orc_bf16_to_f32(in[i]);
}
void orc_f32_to_bf16_n(const float *in, uint16_t *out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = orc_f32_to_bf16(in[i]);
}
void orc_f32_to_f8e4m3fn_n(const float *in, uint8_t *out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = orc_f32_to_f8e4m3fn(in[i]);
}
void orc_decode_n(int dt, const uint8_t *in, float *out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = qval(dt, in, i);
}
