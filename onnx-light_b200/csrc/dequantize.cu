// DequantizeLinear on sm_100a, bit-exact with onnx-light's CPU kernel
// (onnx_light/onnx_extensions/kernels/kernels/quantization/kernel_dequantizelinear.cc).
//
// Layout in HBM: x is read as packed bytes, the output is written once.  The
// reference materialises an int64 scale index per element (:569-572); here the
// index is computed arithmetically from a (outer, axis, inner) decomposition:
// element i = (o * axis_len + k) * inner + in uses scale
//   blocked : (o * s_axis_len + k / block) * inner + in
//   per-axis: k
//   per-tensor: 0
// Each thread produces 8 consecutive elements: one 4/8/16-byte load of x for
// the common packed types, and 16 or 32 bytes of output in 128-bit stores.
// The kernel is HBM-bound: bytes = packed(x) + 4|2 bytes per output element
// (+ scales/zero points, 1/block of that).
#include "b2_common.cuh"
#include "dequantize.cuh"

namespace b2 {



__device__ __forceinline__ float load_scale(const DqParams &p, int64_t si) {
  if (p.f16) return f16_bits_to_f32(reinterpret_cast<const uint16_t *>(p.scale)[si]);
  return reinterpret_cast<const float *>(p.scale)[si];
}

// Loads the 8 quantized values of elements [i0, i0+8) (i0 % 8 == 0, all in range).
__device__ __forceinline__ void load8(const DqParams &p, int64_t i0, float v[8]) {
  const int dt = p.xdt;
  if (dt == kInt4 || dt == kUint4 || dt == kF4E2M1) {
    const uint32_t w = *reinterpret_cast<const uint32_t *>(p.x + (i0 >> 1));
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t nib = (w >> (4 * j)) & 0xfu;
      v[j] = dt == kUint4 ? (float)nib
             : dt == kInt4 ? (float)((int)nib - ((nib & 8u) ? 16 : 0))
                           : dec_f4e2m1(nib);
    }
    return;
  }
  if (dt == kInt8 || dt == kUint8 || is_f8(dt)) {
    const uint2 w = *reinterpret_cast<const uint2 *>(p.x + i0);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t b = ((j < 4 ? w.x : w.y) >> (8 * (j & 3))) & 0xffu;
      switch (dt) {
      case kUint8: v[j] = (float)b; break;
      case kInt8: v[j] = (float)(int8_t)b; break;
      case kF8E4M3FN: v[j] = dec_f8e4m3fn(b); break;
      case kF8E4M3FNUZ: v[j] = dec_f8e4m3fnuz(b); break;
      case kF8E5M2: v[j] = dec_f8e5m2(b); break;
      default: v[j] = dec_f8e5m2fnuz(b); break;
      }
    }
    return;
  }
  if (dt == kInt2 || dt == kUint2) {
    const uint32_t w = *reinterpret_cast<const uint16_t *>(p.x + (i0 >> 2));
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int c = (w >> (2 * j)) & 3;
      v[j] = dt == kUint2 ? (float)c : (float)(c >= 2 ? c - 4 : c);
    }
    return;
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) v[j] = qval(dt, p.x, i0 + j);
}

__device__ __forceinline__ void store1(const DqParams &p, int64_t i, float r) {
  if (p.f16) reinterpret_cast<uint16_t *>(p.y)[i] = f32_to_f16_bits(r);
  else reinterpret_cast<float *>(p.y)[i] = r;
}

// Decomposes flat index i into (o, k, in).
__device__ __forceinline__ void decompose(const DqParams &p, int64_t i, int64_t &o, int64_t &k,
                                          int64_t &in) {
  if (p.use32) {
    const uint32_t ii = (uint32_t)i;
    const uint32_t q1 = p.div_inner.div(ii);
    in = ii - q1 * (uint32_t)p.inner;
    const uint32_t q2 = p.div_alen.div(q1);
    k = q1 - q2 * (uint32_t)p.alen;
    o = q2;
  } else {
    in = i % p.inner;
    const int64_t q1 = i / p.inner;
    k = q1 % p.alen;
    o = q1 / p.alen;
  }
}

__device__ __forceinline__ int64_t scale_index(const DqParams &p, int64_t o, int64_t k,
                                               int64_t in) {
  if (p.layout == 0) return 0;
  if (p.layout == 1) return k;
  const int64_t kb = p.use32 ? (int64_t)p.div_block.div((uint32_t)k) : k / p.block;
  return (o * p.s_alen + kb) * p.inner + in;
}

__global__ void __launch_bounds__(256) dq_kernel(const DqParams p) {
  const int64_t nvec = (p.n + 7) / 8;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < nvec;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i0 = t * 8;
    float v[8];
    const bool full = i0 + 8 <= p.n;
    if (full) {
      load8(p, i0, v);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = (i0 + j < p.n) ? qval(p.xdt, p.x, i0 + j) : 0.0f;
    }
    int64_t o, k, in;
    decompose(p, i0, o, k, in);
    float r[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int64_t si = scale_index(p, o, k, in);
      const float s = load_scale(p, si);
      const float z = p.zp ? qval(p.xdt, p.zp, si) : 0.0f;
      r[j] = x86_mul(x86_sub(v[j], z), s);
      // advance the (o, k, in) odometer
      if (++in == p.inner) {
        in = 0;
        if (++k == p.alen) { k = 0; ++o; }
      }
    }
    if (full) {
      if (p.f16) {
        uint4 w;
        w.x = (uint32_t)f32_to_f16_bits(r[0]) | ((uint32_t)f32_to_f16_bits(r[1]) << 16);
        w.y = (uint32_t)f32_to_f16_bits(r[2]) | ((uint32_t)f32_to_f16_bits(r[3]) << 16);
        w.z = (uint32_t)f32_to_f16_bits(r[4]) | ((uint32_t)f32_to_f16_bits(r[5]) << 16);
        w.w = (uint32_t)f32_to_f16_bits(r[6]) | ((uint32_t)f32_to_f16_bits(r[7]) << 16);
        reinterpret_cast<uint4 *>(p.y)[t] = w;
      } else {
        float4 *dst = reinterpret_cast<float4 *>(p.y) + 2 * t;
        dst[0] = make_float4(r[0], r[1], r[2], r[3]);
        dst[1] = make_float4(r[4], r[5], r[6], r[7]);
      }
    } else {
      for (int j = 0; j < 8; ++j)
        if (i0 + j < p.n) store1(p, i0 + j, r[j]);
    }
  }
}

// ---------------------------------------------------------------------------
// Row kernel: the common layouts, where each group of 8 consecutive elements
// shares (o, k) -- per-tensor scale, or per-axis / blocked along an axis whose
// inner extent is a multiple of 8 (a weight [K, N] quantized along K, N % 8 ==
// 0).  A group then needs one scale (per-tensor, per-axis) or 8 consecutive
// scales (blocked: one vector load) and the same for the zero points, so
// nothing is decoded per element but the value itself.  Each thread handles
// two groups per iteration to keep more bytes in flight.  Same arithmetic as
// dq_kernel: x86 NaN rules, fp32 (q - zp) * s, RNE to fp16 when the scale is.
// ---------------------------------------------------------------------------
enum RowKind : int { kRowI4 = 0, kRowU4, kRowF4, kRowI8, kRowU8, kRowF8E4M3FN };

template <int XK>
__device__ __forceinline__ void dec8_row(const uint8_t *p, int64_t i0, float (&v)[8]) {
  if constexpr (XK == kRowI4 || XK == kRowU4 || XK == kRowF4) {
    const uint32_t w = __ldg(reinterpret_cast<const uint32_t *>(p + (i0 >> 1)));
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if constexpr (XK == kRowI4) v[j] = (float)((int32_t)(w << (28 - 4 * j)) >> 28);
      else if constexpr (XK == kRowU4) v[j] = (float)((w >> (4 * j)) & 0xfu);
      else v[j] = dec_f4e2m1((w >> (4 * j)) & 0xfu);
    }
  } else {
    const uint2 w = __ldg(reinterpret_cast<const uint2 *>(p + i0));
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t b = ((j < 4 ? w.x : w.y) >> (8 * (j & 3))) & 0xffu;
      if constexpr (XK == kRowI8) v[j] = (float)(int8_t)b;
      else if constexpr (XK == kRowU8) v[j] = (float)b;
      else v[j] = dec_f8e4m3fn(b);
    }
  }
}

template <int XK>
__device__ __forceinline__ float dec1_row(const uint8_t *p, int64_t i) {
  if constexpr (XK == kRowI4) return (float)((int32_t)((uint32_t)p[i >> 1] << (28 - 4 * (i & 1))) >> 28);
  else if constexpr (XK == kRowU4) return (float)((p[i >> 1] >> (4 * (i & 1))) & 0xfu);
  else if constexpr (XK == kRowF4) return dec_f4e2m1((p[i >> 1] >> (4 * (i & 1))) & 0xfu);
  else if constexpr (XK == kRowI8) return (float)(int8_t)p[i];
  else if constexpr (XK == kRowU8) return (float)p[i];
  else return dec_f8e4m3fn(p[i]);
}

template <int XK, bool F16>
__global__ void __launch_bounds__(256) dq_rows_kernel(const DqParams p) {
  const int64_t ngroups = p.n / 8; // full groups; a ragged tail (per-tensor only) below
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t t0 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t0 < ngroups; t0 += 2 * stride) {
    float v[2][8], s[2][8], z[2][8];
    int64_t gi[2];
    bool live[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      gi[u] = t0 + u * stride;
      live[u] = gi[u] < ngroups;
      if (!live[u]) continue;
      const int64_t i0 = gi[u] * 8;
      dec8_row<XK>(p.x, i0, v[u]);
      if (p.layout == 0) {
        const float sc = F16 ? f16_bits_to_f32(__ldg(reinterpret_cast<const uint16_t *>(p.scale)))
                             : __ldg(reinterpret_cast<const float *>(p.scale));
        const float zz = p.zp ? dec1_row<XK>(p.zp, 0) : 0.0f;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          s[u][j] = sc;
          z[u][j] = zz;
        }
        continue;
      }
      // (o, k, in) of the group's first element; in % 8 == 0
      const uint32_t ii = (uint32_t)i0;
      const uint32_t q1 = p.div_inner.div(ii);
      const uint32_t in = ii - q1 * (uint32_t)p.inner;
      const uint32_t q2 = p.div_alen.div(q1);
      const uint32_t k = q1 - q2 * (uint32_t)p.alen;
      if (p.layout == 1) {
        const float sc = F16 ? f16_bits_to_f32(__ldg(reinterpret_cast<const uint16_t *>(p.scale) + k))
                             : __ldg(reinterpret_cast<const float *>(p.scale) + k);
        const float zz = p.zp ? dec1_row<XK>(p.zp, k) : 0.0f;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          s[u][j] = sc;
          z[u][j] = zz;
        }
        continue;
      }
      const int64_t si = ((int64_t)q2 * p.s_alen + p.div_block.div(k)) * p.inner + in;
      if (F16) {
        const uint4 w = __ldg(reinterpret_cast<const uint4 *>(reinterpret_cast<const uint16_t *>(p.scale) + si));
        const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          s[u][2 * j] = f16_bits_to_f32((uint16_t)(ww[j] & 0xffffu));
          s[u][2 * j + 1] = f16_bits_to_f32((uint16_t)(ww[j] >> 16));
        }
      } else {
        const float4 a = __ldg(reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(p.scale) + si));
        const float4 b = __ldg(reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(p.scale) + si + 4));
        s[u][0] = a.x; s[u][1] = a.y; s[u][2] = a.z; s[u][3] = a.w;
        s[u][4] = b.x; s[u][5] = b.y; s[u][6] = b.z; s[u][7] = b.w;
      }
      if (p.zp) dec8_row<XK>(p.zp, si, z[u]);
      else {
#pragma unroll
        for (int j = 0; j < 8; ++j) z[u][j] = 0.0f;
      }
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      if (!live[u]) continue;
      float r[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) r[j] = x86_mul(x86_sub(v[u][j], z[u][j]), s[u][j]);
      if (F16) {
        uint4 w;
        w.x = (uint32_t)f32_to_f16_bits(r[0]) | ((uint32_t)f32_to_f16_bits(r[1]) << 16);
        w.y = (uint32_t)f32_to_f16_bits(r[2]) | ((uint32_t)f32_to_f16_bits(r[3]) << 16);
        w.z = (uint32_t)f32_to_f16_bits(r[4]) | ((uint32_t)f32_to_f16_bits(r[5]) << 16);
        w.w = (uint32_t)f32_to_f16_bits(r[6]) | ((uint32_t)f32_to_f16_bits(r[7]) << 16);
        __stcs(reinterpret_cast<uint4 *>(p.y) + gi[u], w);
      } else {
        float4 *dst = reinterpret_cast<float4 *>(p.y) + 2 * gi[u];
        __stcs(dst, make_float4(r[0], r[1], r[2], r[3]));
        __stcs(dst + 1, make_float4(r[4], r[5], r[6], r[7]));
      }
    }
  }
  // ragged tail of a per-tensor call (n % 8 elements), one thread each
  if (blockIdx.x == 0 && threadIdx.x < (p.n & 7)) {
    const int64_t i = (p.n & ~(int64_t)7) + threadIdx.x;
    const float sc = F16 ? f16_bits_to_f32(reinterpret_cast<const uint16_t *>(p.scale)[0])
                         : reinterpret_cast<const float *>(p.scale)[0];
    const float zz = p.zp ? dec1_row<XK>(p.zp, 0) : 0.0f;
    store1(p, i, x86_mul(x86_sub(dec1_row<XK>(p.x, i), zz), sc));
  }
}

// Row kernel variant for this call, or nullptr (then dq_kernel runs).
static void (*row_kernel(const DqParams &p))(DqParams) {
  if (!p.use32) return nullptr;
  if (p.layout != 0 && (p.inner % 8 != 0 || p.n % 8 != 0)) return nullptr;
  const uintptr_t sa = reinterpret_cast<uintptr_t>(p.scale), za = reinterpret_cast<uintptr_t>(p.zp);
  if (p.layout == 2 && ((sa & 15u) || (za & 7u))) return nullptr; // vector loads of 8 scales / zps
  int xk;
  switch (p.xdt) {
  case kInt4: xk = kRowI4; break;
  case kUint4: xk = kRowU4; break;
  case kF4E2M1: xk = kRowF4; break;
  case kInt8: xk = kRowI8; break;
  case kUint8: xk = kRowU8; break;
  case kF8E4M3FN: xk = kRowF8E4M3FN; break;
  default: return nullptr;
  }
  static void (*const table[6][2])(DqParams) = {
      {dq_rows_kernel<kRowI4, false>, dq_rows_kernel<kRowI4, true>},
      {dq_rows_kernel<kRowU4, false>, dq_rows_kernel<kRowU4, true>},
      {dq_rows_kernel<kRowF4, false>, dq_rows_kernel<kRowF4, true>},
      {dq_rows_kernel<kRowI8, false>, dq_rows_kernel<kRowI8, true>},
      {dq_rows_kernel<kRowU8, false>, dq_rows_kernel<kRowU8, true>},
      {dq_rows_kernel<kRowF8E4M3FN, false>, dq_rows_kernel<kRowF8E4M3FN, true>}};
  return table[xk][p.f16 ? 1 : 0];
}

static bool dq_supported(int dt) {
  return dt == kUint8 || dt == kInt8 || dt == kUint16 || dt == kInt16 || dt == kInt32 || is_f8(dt) ||
         dt == kUint4 || dt == kInt4 || dt == kUint2 || dt == kInt2 || dt == kF4E2M1 ||
         dt == kF6E2M3 || dt == kF6E3M2;
}

static bool same_shape(const b2_tensor *a, const b2_tensor *b) {
  if (a->ndim != b->ndim) return false;
  for (int i = 0; i < a->ndim; ++i)
    if (a->shape[i] != b->shape[i]) return false;
  return true;
}

// Validation of kernel_dequantizelinear.cc:332-693, in the reference's order.
// On success fills the kernel parameters (without pointers).
int dq_validate(const b2_tensor *x, const b2_tensor *s, const b2_tensor *zp, int64_t axis,
                int32_t out_dtype, const std::vector<int64_t> &out_shape, DqParams &p) {
  B2_ENFORCE(s->dtype == kFloat || s->dtype == kFloat16,
             "kernel::DequantizeLinear: x_scale must be FLOAT or FLOAT16.");
  const int64_t sn = numel(s);
  const int64_t n = numel(x);
  if (sn == 1) {
    if (zp) {
      B2_ENFORCE(numel(zp) == 1,
                 "kernel::DequantizeLinear: x_zero_point must be a scalar (per-tensor dequantization).");
      B2_ENFORCE(x->dtype == zp->dtype,
                 "kernel::DequantizeLinear: x_zero_point data_type must match x.");
    }
    B2_ENFORCE(out_dtype == s->dtype, "kernel::DequantizeLinear: output dtype must match x_scale.");
    B2_ENFORCE(out_shape == shape_of(x),
               "kernel::DequantizeLinear preallocated output shape must match x shape.");
    if (!dq_supported(x->dtype))
      B2_FAIL(B2_ERR_UNSUPPORTED_DTYPE,
              "unsupported data type %d, kernel::DequantizeLinear: only UINT8, INT8, UINT16, INT16, "
              "INT32, FLOAT8E4M3FN, FLOAT8E4M3FNUZ, FLOAT8E5M2, FLOAT8E5M2FNUZ, INT4, UINT4, INT2, "
              "UINT2 and FLOAT4E2M1 inputs are supported.",
              x->dtype);
    p.layout = 0;
    p.inner = 1;
    p.alen = n > 0 ? n : 1;
    p.s_alen = 1;
    p.block = 1;
  } else {
    B2_ENFORCE(axis >= 0 && axis < x->ndim, "kernel::DequantizeLinear: axis out of range.");
    if (zp)
      B2_ENFORCE(x->dtype == zp->dtype,
                 "kernel::DequantizeLinear: x_zero_point data_type must match x.");
    B2_ENFORCE(out_dtype == s->dtype, "kernel::DequantizeLinear: output dtype must match x_scale.");
    B2_ENFORCE(out_shape == shape_of(x),
               "kernel::DequantizeLinear preallocated output shape must match x shape.");
    if (zp)
      B2_ENFORCE(same_shape(s, zp),
                 "kernel::DequantizeLinear: x_scale and x_zero_point must have the same shape.");
    int64_t outer = 1, inner = 1;
    for (int d = 0; d < axis; ++d) outer *= x->shape[d];
    for (int d = (int)axis + 1; d < x->ndim; ++d) inner *= x->shape[d];
    const int64_t alen = x->shape[axis];
    if (s->ndim == x->ndim) {
      for (int d = 0; d < x->ndim; ++d) {
        const int64_t sd = s->shape[d];
        B2_ENFORCE(sd > 0 && x->shape[d] % sd == 0,
                   "kernel::DequantizeLinear: blocked x_scale dimension must divide the matching x "
                   "dimension.");
        B2_ENFORCE(d == axis || sd == x->shape[d],
                   "kernel::DequantizeLinear: blocked x_scale may only differ from x along the "
                   "quantization axis.");
      }
      p.layout = 2;
      p.s_alen = s->shape[axis];
      p.block = alen / p.s_alen;
    } else {
      B2_ENFORCE(sn == alen,
                 "kernel::DequantizeLinear: x_scale element count must equal axis dimension.");
      p.layout = 1;
      p.s_alen = alen;
      p.block = 1;
    }
    if (!dq_supported(x->dtype))
      B2_FAIL(B2_ERR_UNSUPPORTED_DTYPE,
              "unsupported data type %d, kernel::DequantizeLinear (per-axis): only UINT8, INT8, "
              "UINT16, INT16, INT32, FLOAT8E4M3FN, FLOAT8E4M3FNUZ, FLOAT8E5M2, FLOAT8E5M2FNUZ, INT4, "
              "UINT4, INT2, UINT2 and FLOAT4E2M1 inputs are supported.",
              x->dtype);
    p.inner = inner > 0 ? inner : 1;
    p.alen = alen > 0 ? alen : 1;
    (void)outer;
  }
  p.n = n;
  p.xdt = x->dtype;
  p.f16 = s->dtype == kFloat16;
  p.use32 = n < (int64_t(1) << 31) ? 1u : 0u;
  if (p.use32) {
    p.div_inner = FastDiv((uint32_t)p.inner);
    p.div_alen = FastDiv((uint32_t)p.alen);
    p.div_block = FastDiv((uint32_t)p.block);
  }
  return B2_OK;
}

int dq_launch(const DqParams &p, cudaStream_t stream) {
  if (p.n == 0) return B2_OK;
  const int64_t nvec = (p.n + 7) / 8;
  const int threads = 256;
  if (auto rk = row_kernel(p)) {
    // two groups of 8 per thread and iteration; 8 CTAs of 256 per SM
    int64_t blocks = (nvec + 2 * threads - 1) / (2 * threads);
    const int64_t cap = (int64_t)sm_count() * 8;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    rk<<<(unsigned)blocks, threads, 0, stream>>>(p);
    B2_LAUNCH_CHECK();
    return B2_OK;
  }
  int64_t blocks = (nvec + threads - 1) / threads;
  const int64_t cap = (int64_t)sm_count() * 16;
  if (blocks > cap) blocks = cap;
  dq_kernel<<<(unsigned)blocks, threads, 0, stream>>>(p);
  B2_LAUNCH_CHECK();
  return B2_OK;
}

} // namespace b2

using namespace b2;

extern "C" int b2_dequantize_linear(const b2_tensor *x, const b2_tensor *x_scale,
                                    const b2_tensor *x_zero_point, int64_t axis, b2_tensor *y,
                                    void *stream) {
  if (!x || !x_scale || !y) B2_FAIL(B2_ERR_INVALID_ARGUMENT, "kernel::DequantizeLinear: null tensor");
  DqParams p{};
  int rc = dq_validate(x, x_scale, x_zero_point, axis, y->dtype, shape_of(y), p);
  if (rc) return rc;
  p.x = static_cast<const uint8_t *>(x->data);
  p.scale = static_cast<const uint8_t *>(x_scale->data);
  p.zp = x_zero_point ? static_cast<const uint8_t *>(x_zero_point->data) : nullptr;
  p.y = y->data;
  // The vector load/store path needs 16-byte aligned output and 4-byte aligned x.
  if ((reinterpret_cast<uintptr_t>(p.y) & 15u) || (reinterpret_cast<uintptr_t>(p.x) & 7u))
    B2_FAIL(B2_ERR_INVALID_ARGUMENT,
            "kernel::DequantizeLinear: x must be 8-byte and y 16-byte aligned on the device");
  return dq_launch(p, static_cast<cudaStream_t>(stream));
}
