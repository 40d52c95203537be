// Library-wide pieces of the C ABI: version string, per-thread last error,
// device properties, and the seeded input generators.
#include "b2_common.cuh"


namespace b2 {

namespace {
thread_local int g_status = B2_OK;
thread_local char g_message[1024] = {0};
} // namespace

void set_error(int status, const char *fmt, ...) {
  g_status = status;
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_message, sizeof(g_message), fmt, ap);
  va_end(ap);
}

int last_status() { return g_status; }

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (!cached[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = n > 0 ? n : 148;
  }
  return cached[dev];
}

// ---------------------------------------------------------------------------
// SplitMix64 generators.  Element i of a stream seeded with `seed` is
// mix(seed + (i+1) * golden) (random.cc:38-45), so every element is computed
// independently on the device.
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint64_t sm_mix(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}
__device__ __forceinline__ uint64_t sm_draw(uint64_t seed, uint64_t idx) {
  return sm_mix(seed + (idx + 1) * 0x9E3779B97F4A7C15ULL);
}
__device__ __forceinline__ double sm_unit(uint64_t v) {
  return (double)(v >> 11) * (1.0 / 9007199254740992.0);
}

__global__ void synth_kernel(int kind, uint64_t seed, int64_t n, double lo, double hi, void *out,
                             uint64_t span) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    if (kind == 0) {
      // RandUniformInto<float> (random.cc:141-152)
      const float span_f = (float)(hi - lo), low_f = (float)lo;
      reinterpret_cast<float *>(out)[i] =
          __fadd_rn(low_f, __fmul_rn((float)sm_unit(sm_draw(seed, (uint64_t)i)), span_f));
    } else if (kind == 1) {
      // RandNormalInto<float> (random.cc:159-176): 12 draws per sample.
      double acc = 0.0;
      for (int j = 0; j < 12; ++j) acc = __dadd_rn(acc, sm_unit(sm_draw(seed, (uint64_t)i * 12 + j)));
      reinterpret_cast<float *>(out)[i] =
          __fadd_rn((float)lo, __fmul_rn((float)__dsub_rn(acc, 6.0), (float)hi));
    } else {
      // RandInt (random.cc:61-89); spans are small enough that the
      // reference never rejects a draw, so element i uses draw i.
      const uint64_t v = sm_draw(seed, (uint64_t)i);
      reinterpret_cast<int64_t *>(out)[i] = (int64_t)(v % span) + (int64_t)lo;
    }
  }
}

// FLOAT -> FLOAT8E4M3FN, saturating round-to-nearest-even (the encoding
// onnx_light/onnx_core/runtime/kernels/cast_float8.cc:27-80 produces).
__device__ __forceinline__ uint8_t enc_f8e4m3fn(float f) {
  const uint32_t u = __float_as_uint(f);
  const uint8_t sign = (uint8_t)((u >> 24) & 0x80u);
  if ((u & 0x7fffffffu) == 0x7f800000u) return (uint8_t)(sign | 0x7eu);
  if ((u & 0x7f800000u) == 0x7f800000u) return (uint8_t)(sign | 0x7fu);
  const float a = fabsf(f);
  if (a >= 464.0f) return (uint8_t)(sign | 0x7eu);
  int e;
  frexpf(a, &e);
  int q = e - 4;
  if (q < -9) q = -9;
  const float ulp = ldexpf(1.0f, q);
  float val = rintf(a / ulp) * ulp;
  if (val > 448.0f) val = 448.0f;
  if (val == 0.0f) return sign;
  if (val < 0.015625f) return (uint8_t)(sign | (uint8_t)(val * 512.0f));
  int ve;
  const float fr = frexpf(val, &ve);
  return (uint8_t)(sign | ((uint32_t)(ve + 6) << 3) | (uint32_t)((fr * 2.0f - 1.0f) * 8.0f));
}

__global__ void convert_kernel(const void *src, int sdt, void *dst, int ddt, int64_t n) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t t0 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (sdt == kFloat && (ddt == kFloat16 || ddt == kBfloat16 || ddt == kF8E4M3FN)) {
    for (int64_t i = t0; i < n; i += stride) {
      const float f = reinterpret_cast<const float *>(src)[i];
      if (ddt == kFloat16) reinterpret_cast<uint16_t *>(dst)[i] = f32_to_f16_bits(f);
      else if (ddt == kBfloat16) reinterpret_cast<uint16_t *>(dst)[i] = f32_to_bf16_bits(f);
      else reinterpret_cast<uint8_t *>(dst)[i] = enc_f8e4m3fn(f);
    }
    return;
  }
  const int64_t *s = reinterpret_cast<const int64_t *>(src);
  uint8_t *d = reinterpret_cast<uint8_t *>(dst);
  if (ddt == kInt8 || ddt == kUint8) {
    for (int64_t i = t0; i < n; i += stride) d[i] = (uint8_t)(s[i] & 0xff);
  } else if (ddt == kInt4 || ddt == kUint4 || ddt == kF4E2M1) {
    const int64_t nb = (n + 1) / 2;
    for (int64_t b = t0; b < nb; b += stride) {
      const uint32_t lo = (uint32_t)(s[2 * b] & 0xf);
      const uint32_t hi = 2 * b + 1 < n ? (uint32_t)(s[2 * b + 1] & 0xf) : 0u;
      d[b] = (uint8_t)(lo | (hi << 4));
    }
  } else if (ddt == kInt2 || ddt == kUint2) {
    const int64_t nb = (n + 3) / 4;
    for (int64_t b = t0; b < nb; b += stride) {
      uint32_t v = 0;
      for (int j = 0; j < 4; ++j)
        if (4 * b + j < n) v |= (uint32_t)(s[4 * b + j] & 3) << (2 * j);
      d[b] = (uint8_t)v;
    }
  }
}

} // namespace b2

using namespace b2;

extern "C" const char *b2_version(void) { return "onnxl_b200 0.1 sm_100a"; }

extern "C" int b2_last_error(char *buf, size_t len) {
  if (buf && len) {
    strncpy(buf, g_message, len - 1);
    buf[len - 1] = 0;
  }
  return g_status;
}

extern "C" int b2_synth_fill(int32_t kind, uint64_t seed, int64_t n, double lo, double hi,
                             void *out, void *stream) {
  if (kind < 0 || kind > 2 || n < 0) B2_FAIL(B2_ERR_INVALID_ARGUMENT, "b2_synth_fill: bad kind or size");
  if (n == 0) return B2_OK;
  uint64_t span = 0;
  if (kind == 2) {
    B2_ENFORCE(hi > lo, "high must be greater than low.");
    span = (uint64_t)((int64_t)hi + 1 - (int64_t)lo);
    // The reference rejects a draw only when it lands in the top (2^64 mod
    // span) values; for spans up to 2^16 that is below 2^-48 per draw, so the
    // counter-based stream (draw i for element i) reproduces it.  Wider spans
    // are refused rather than risk a silent divergence.
    if (span > 65536) B2_FAIL(B2_ERR_UNSUPPORTED, "b2_synth_fill: integer span above 2^16");
    lo = (double)(int64_t)lo;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int64_t blocks = (n + 255) / 256;
  if (blocks > sm_count() * 32) blocks = sm_count() * 32;
  synth_kernel<<<(unsigned)blocks, 256, 0, st>>>(kind, seed, n, lo, hi, out, span);
  B2_LAUNCH_CHECK();
  return B2_OK;
}

extern "C" int b2_convert(const void *src, int32_t src_dtype, void *dst, int32_t dst_dtype,
                          int64_t n, void *stream) {
  const bool f2x = src_dtype == kFloat &&
                   (dst_dtype == kFloat16 || dst_dtype == kBfloat16 || dst_dtype == kF8E4M3FN);
  const bool i2x = src_dtype == kInt64 &&
                   (dst_dtype == kInt8 || dst_dtype == kUint8 || dst_dtype == kInt4 ||
                    dst_dtype == kUint4 || dst_dtype == kF4E2M1 || dst_dtype == kInt2 ||
                    dst_dtype == kUint2);
  if (!f2x && !i2x) B2_FAIL(B2_ERR_UNSUPPORTED_DTYPE, "b2_convert: %s -> %s not supported",
                            dtype_name(src_dtype), dtype_name(dst_dtype));
  if (n == 0) return B2_OK;
  int64_t blocks = (n + 255) / 256;
  if (blocks > sm_count() * 32) blocks = sm_count() * 32;
  convert_kernel<<<(unsigned)blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      src, src_dtype, dst, dst_dtype, n);
  B2_LAUNCH_CHECK();
  return B2_OK;
}
