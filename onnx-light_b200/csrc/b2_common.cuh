// Shared definitions for the onnxl_b200 CUDA sources: dtype codes, status
// handling, shape helpers and the bit-exact scalar conversions the
// DequantizeLinear path needs.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <string>
#include <vector>

#include "../../include/onnxl_b200.h"

namespace b2 {

// ONNX TensorProto.DataType codes.
enum DType : int32_t {
  kFloat = 1, kUint8 = 2, kInt8 = 3, kUint16 = 4, kInt16 = 5, kInt32 = 6, kInt64 = 7,
  kBool = 9, kFloat16 = 10, kDouble = 11, kBfloat16 = 16, kF8E4M3FN = 17, kF8E4M3FNUZ = 18,
  kF8E5M2 = 19, kF8E5M2FNUZ = 20, kUint4 = 21, kInt4 = 22, kF4E2M1 = 23, kF8E8M0 = 24,
  kUint2 = 25, kInt2 = 26, kF6E2M3 = 27, kF6E3M2 = 28
};

// ---------------------------------------------------------------------------
// Host-side status handling
// ---------------------------------------------------------------------------

void set_error(int status, const char *fmt, ...);
int last_status();

struct Status {
  int code = B2_OK;
  bool ok() const { return code == B2_OK; }
};

#define B2_FAIL(code, ...)            \
  do {                                \
    ::b2::set_error((code), __VA_ARGS__); \
    return (code);                    \
  } while (0)

#define B2_ENFORCE(cond, ...)                                   \
  do {                                                          \
    if (!(cond)) B2_FAIL(B2_ERR_INVALID_ARGUMENT, __VA_ARGS__); \
  } while (0)

#define B2_CUDA(expr)                                                              \
  do {                                                                             \
    cudaError_t e__ = (expr);                                                      \
    if (e__ != cudaSuccess)                                                        \
      B2_FAIL(B2_ERR_CUDA, "CUDA error %s at %s:%d (%s)", cudaGetErrorString(e__), \
              __FILE__, __LINE__, #expr);                                          \
  } while (0)

// Checks the launch that was just issued.
#define B2_LAUNCH_CHECK() B2_CUDA(cudaGetLastError())

inline int64_t numel(const b2_tensor *t) {
  int64_t n = 1;
  for (int i = 0; i < t->ndim; ++i) n *= t->shape[i];
  return n;
}

inline std::vector<int64_t> shape_of(const b2_tensor *t) {
  return std::vector<int64_t>(t->shape, t->shape + t->ndim);
}

__host__ __device__ inline bool is_f8(int dt) {
  return dt == kF8E4M3FN || dt == kF8E4M3FNUZ || dt == kF8E5M2 || dt == kF8E5M2FNUZ;
}

// Storage bytes of n elements (onnx_light/onnx_core/runtime/memory/simple_tensor.cc:205-231).
inline int64_t packed_bytes(int dt, int64_t n) {
  switch (dt) {
  case kInt4: case kUint4: case kF4E2M1: return n / 2 + (n % 2);
  case kInt2: case kUint2: return n / 4 + (n % 4 != 0);
  case kF6E2M3: case kF6E3M2: return n / 4 * 3 + (n % 4 * 6 + 7) / 8;
  case kUint8: case kInt8: case kBool: return n;
  case kUint16: case kInt16: case kFloat16: case kBfloat16: return 2 * n;
  case kInt32: case kFloat: return 4 * n;
  case kInt64: case kDouble: return 8 * n;
  default: return is_f8(dt) ? n : -1;
  }
}

inline const char *dtype_name(int dt) {
  switch (dt) {
  case kFloat: return "FLOAT"; case kUint8: return "UINT8"; case kInt8: return "INT8";
  case kUint16: return "UINT16"; case kInt16: return "INT16"; case kInt32: return "INT32";
  case kInt64: return "INT64"; case kBool: return "BOOL"; case kFloat16: return "FLOAT16";
  case kDouble: return "DOUBLE"; case kBfloat16: return "BFLOAT16";
  case kF8E4M3FN: return "FLOAT8E4M3FN"; case kF8E4M3FNUZ: return "FLOAT8E4M3FNUZ";
  case kF8E5M2: return "FLOAT8E5M2"; case kF8E5M2FNUZ: return "FLOAT8E5M2FNUZ";
  case kUint4: return "UINT4"; case kInt4: return "INT4"; case kF4E2M1: return "FLOAT4E2M1";
  case kF6E2M3: return "FLOAT6E2M3"; case kF6E3M2: return "FLOAT6E3M2";
  case kUint2: return "UINT2"; case kInt2: return "INT2";
  default: return "?";
  }
}

// Workspace layout shared by every entry point: the first kCounterBytes hold
// uint32 arrival counters (split-K / split-KV "last CTA" detection).  Every
// kernel that uses counters returns them to zero before it exits, and no
// kernel ever writes anything else there, so the region stays all-zero across
// calls of any shape.  Per-call partial results follow the counter region.
constexpr size_t kCounterBytes = 64 * 1024;
// The last 16 bytes of the counter region are reserved (no kernel writes
// there); counters stop short of them.  Time-out codes live in per-kernel
// device words that b2_kernel_status() reads, never in the caller's workspace.
constexpr size_t kStatusOffset = kCounterBytes - 16;
constexpr size_t kMaxCounters = kStatusOffset / 4;

// Wall-clock limit of a bounded device-side wait (mbarrier, arrival flag).
constexpr uint64_t kWaitNs = 2000000000ull;

// Split-K arrival with a give-up mark.  Every contributor of a tile adds 1 to
// the tile's counter, plus kAbortMark when a bounded wait of its own gave up
// (its partial sums are then not valid).  The contributor whose arrival
// completes the count is the last; it resets the counter to zero, so the
// counters stay all-zero across calls even after a time-out, and it learns
// whether any contributor gave up (then it must not merge).  Called by one
// thread, after the caller's own partial stores are ordered before it.
constexpr uint32_t kAbortMark = 1u << 16;
__device__ __forceinline__ bool arrive_marked(uint32_t *counter, uint32_t expected, bool gave_up,
                                              bool *any_gave_up) {
  __threadfence();
  const uint32_t inc = gave_up ? kAbortMark + 1u : 1u;
  const uint32_t now = atomicAdd(counter, inc) + inc;
  const bool last = (now & (kAbortMark - 1u)) == expected;
  if (last) {
    __threadfence();
    *counter = 0u;
  }
  *any_gave_up = (now >> 16) != 0u;
  return last;
}

// Workspace protocol shared by every entry point that needs scratch.
// Returns 1 when the call is a size query (workspace == NULL), 0 when the
// caller offered enough, and a negative status otherwise.
inline int workspace_check(void *ws, size_t *ws_bytes, size_t need) {
  if (ws == nullptr) {
    if (ws_bytes == nullptr) {
      if (need == 0) return 0;
      set_error(B2_ERR_WORKSPACE, "workspace of %zu bytes required", need);
      return B2_ERR_WORKSPACE;
    }
    *ws_bytes = need; // size query: nothing runs, whatever the size
    return 1;
  }
  if (ws_bytes == nullptr || *ws_bytes < need) {
    set_error(B2_ERR_WORKSPACE, "workspace too small: %zu bytes required, %zu offered", need,
              ws_bytes ? *ws_bytes : (size_t)0);
    return B2_ERR_WORKSPACE;
  }
  return 0;
}

// Number of SMs of the current device (cached per device).
int sm_count();

// ---------------------------------------------------------------------------
// Device-side conversions
// ---------------------------------------------------------------------------

__device__ __forceinline__ float u2f(uint32_t u) { return __uint_as_float(u); }
__device__ __forceinline__ uint32_t f2u(float f) { return __float_as_uint(f); }

// x86 SSE binary-op NaN propagation, which the reference's compiled CPU loops
// follow: the first NaN operand is returned quieted; an invalid operation on
// non-NaN operands returns the "real indefinite" 0xffc00000.
__device__ __forceinline__ float nan_result(float a, float b) {
  if (a != a) return u2f(f2u(a) | 0x00400000u);
  if (b != b) return u2f(f2u(b) | 0x00400000u);
  return u2f(0xffc00000u);
}
__device__ __forceinline__ float x86_sub(float a, float b) {
  const float r = __fsub_rn(a, b);
  return r == r ? r : nan_result(a, b);
}
__device__ __forceinline__ float x86_mul(float a, float b) {
  const float r = __fmul_rn(a, b);
  return r == r ? r : nan_result(a, b);
}

// binary32 -> binary16 bits as onnx_light/onnx_core/runtime/kernels/cast_helper.cc:51-87
// (IEEE RNE; NaN collapses to sign|0x7e00).
__device__ __forceinline__ uint16_t f32_to_f16_bits(float f) {
  if (f != f) return (uint16_t)(((f2u(f) >> 16) & 0x8000u) | 0x7e00u);
  return __half_as_ushort(__float2half_rn(f));
}
// binary32 -> bfloat16 bits as cast_helper.cc:124-135 (RNE; NaN keeps payload | 0x40).
__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
  const uint32_t u = f2u(f);
  if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x7fffffu)) return (uint16_t)((u >> 16) | 0x40u);
  return (uint16_t)((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
}
__device__ __forceinline__ float f16_bits_to_f32(uint16_t h) {
  return __half2float(__ushort_as_half(h));
}

// 8-bit float decoders; NaN bit patterns follow
// onnx_light/onnx_core/runtime/kernels/cast_float8.cc:83-375.
__device__ __forceinline__ float dec_f8e4m3fn(uint32_t v) {
  if ((v & 0x7fu) == 0x7fu) return u2f((v & 0x80u) ? 0xffc00000u : 0x7fc00000u);
  const uint32_t sign = (v & 0x80u) << 24, ex = (v >> 3) & 0xfu, man = v & 7u;
  if (ex == 0) return u2f(sign | f2u((float)man * 0.001953125f));
  return u2f(sign | ((ex + 120u) << 23) | (man << 20));
}
__device__ __forceinline__ float dec_f8e4m3fnuz(uint32_t v) {
  if (v == 0x80u) return u2f(0xffc00000u);
  const uint32_t sign = (v & 0x80u) << 24, ex = (v >> 3) & 0xfu, man = v & 7u;
  if (ex == 0) return u2f(sign | f2u((float)man * 0.0009765625f));
  return u2f(sign | ((ex + 119u) << 23) | (man << 20));
}
__device__ __forceinline__ float dec_f8e5m2(uint32_t v) {
  if (v >= 253u) return u2f(0xffc00000u);
  if (v >= 125u && v <= 127u) return u2f(0x7fc00000u);
  if (v == 252u) return u2f(0xff800000u);
  if (v == 124u) return u2f(0x7f800000u);
  const uint32_t sign = (v & 0x80u) << 24, ex = (v >> 2) & 0x1fu, man = v & 3u;
  if (ex == 0) return u2f(sign | f2u((float)man * 1.52587890625e-05f));
  return u2f(sign | ((ex + 112u) << 23) | (man << 21));
}
__device__ __forceinline__ float dec_f8e5m2fnuz(uint32_t v) {
  if (v == 0x80u) return u2f(0xffc00000u);
  const uint32_t sign = (v & 0x80u) << 24, ex = (v >> 2) & 0x1fu, man = v & 3u;
  if (ex == 0) return u2f(sign | f2u((float)man * 7.62939453125e-06f));
  return u2f(sign | ((ex + 111u) << 23) | (man << 21));
}
// FLOAT4E2M1 value table (cast_helper.cc:161-166), as bit patterns.
__device__ __forceinline__ float dec_f4e2m1(uint32_t nib) {
  // magnitudes 0, .5, 1, 1.5, 2, 3, 4, 6 for codes 0..7
  const uint32_t m = nib & 7u;
  const float mag = m < 2 ? 0.5f * (float)m : (m < 4 ? 0.5f * (float)m : (float)(1u << ((m >> 1) - 1)) * (1.0f + 0.5f * (float)(m & 1u)));
  return u2f(f2u(mag) | ((nib & 8u) << 28));
}
// FLOAT6 (cast_helper.cc:208-219).
__device__ __forceinline__ float dec_f6(uint32_t bits, int dt) {
  const int mb = dt == kF6E2M3 ? 3 : 2;
  const int eb = 5 - mb;
  const int bias = (1 << (eb - 1)) - 1;
  const int ex = (bits >> mb) & ((1 << eb) - 1);
  const int man = bits & ((1 << mb) - 1);
  const float v = ex == 0 ? ldexpf((float)man, 1 - bias - mb)
                          : ldexpf(1.0f + (float)man / (float)(1 << mb), ex - bias);
  return (bits & 0x20u) ? -v : v;
}

// Reads element i of a quantized tensor as float, as the reference's typed
// loops convert it (kernel_dequantizelinear.cc:65-159, 246-328).
__device__ __forceinline__ float qval(int dt, const uint8_t *__restrict__ p, int64_t i) {
  switch (dt) {
  case kUint8: return (float)p[i];
  case kInt8: return (float)(int8_t)p[i];
  case kUint16: return (float)reinterpret_cast<const uint16_t *>(p)[i];
  case kInt16: return (float)reinterpret_cast<const int16_t *>(p)[i];
  case kInt32: return __int2float_rn(reinterpret_cast<const int32_t *>(p)[i]);
  case kUint4: return (float)((p[i >> 1] >> ((i & 1) * 4)) & 0xfu);
  case kInt4: { const int n = (p[i >> 1] >> ((i & 1) * 4)) & 0xf; return (float)(n >= 8 ? n - 16 : n); }
  case kUint2: return (float)((p[i >> 2] >> ((i & 3) * 2)) & 3u);
  case kInt2: { const int n = (p[i >> 2] >> ((i & 3) * 2)) & 3; return (float)(n >= 2 ? n - 4 : n); }
  case kF4E2M1: return dec_f4e2m1((p[i >> 1] >> ((i & 1) * 4)) & 0xfu);
  case kF8E4M3FN: return dec_f8e4m3fn(p[i]);
  case kF8E4M3FNUZ: return dec_f8e4m3fnuz(p[i]);
  case kF8E5M2: return dec_f8e5m2(p[i]);
  case kF8E5M2FNUZ: return dec_f8e5m2fnuz(p[i]);
  case kF6E2M3: case kF6E3M2: {
    const uint64_t bo = (uint64_t)i * 6, by = bo / 8;
    const int sh = (int)(bo % 8);
    uint32_t v = p[by] >> sh;
    if (sh > 2) v |= (uint32_t)p[by + 1] << (8 - sh);
    return dec_f6(v & 0x3fu, dt);
  }
  default: return 0.0f;
  }
}

// Fast unsigned 32-bit division by a runtime constant (Granlund-Montgomery
// round-up method: q = umulhi(n, m) + n >> s for divisors > 1).
struct FastDiv {
  uint32_t d = 1, m = 0, s = 0;
  FastDiv() = default;
  explicit FastDiv(uint32_t div) : d(div) {
    if (d <= 1) { m = 0; s = 0; return; }
    uint32_t l = 0;
    while ((1ull << l) < d) ++l;
    m = (uint32_t)((((1ull << 32) * ((1ull << l) - d)) / d) + 1);
    s = l - 1;
  }
  __device__ __forceinline__ uint32_t div(uint32_t n) const {
    if (d == 1) return n;
    const uint32_t t = __umulhi(n, m);
    return (t + ((n - t) >> 1)) >> s;
  }
};

} // namespace b2
