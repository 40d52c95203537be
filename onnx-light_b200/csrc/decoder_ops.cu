// The decoder-layer operators around the quantized projections, so that a
// Llama layer's ONNX graph stays on the device: RMSNormalization,
// RotaryEmbedding and SwiGLU (opset 23 / onnx-light), with the reference's
// operation order and rounding.
//
//  * b2_rms_normalization -- kernel::RMSNormalization
//    (onnx_light/onnx_extensions/kernels/kernels/nn/kernel_rmsnormalization.cc:83-214):
//    per row of the normalized axes, the sum of squares in double, mean in
//    double, rms = sqrt(float(mean) + epsilon) in float, x / rms, times the
//    broadcast scale (half types: the normalized value is rounded to the type
//    before the scale multiplies it, :200-205).  One CTA per row; the row is
//    read twice (the second time from L2 for rows up to tens of KB), HBM-bound.
//  * b2_rotary_embedding -- kernel::RotaryEmbedding
//    (.../nn/kernel_rotary_embedding.cc:47-218): rank-4 [B, H, S, D] or
//    rank-3 [B, S, H*D], rotate-half or interleaved pairs over the first
//    rotary_embedding_dim channels, cos/sin rows by position_ids or by
//    (batch, position); y1 = c x1 - s x2, y2 = s x1 + c x2 with separately
//    rounded products (no FMA contraction), half types through float.  One
//    thread per output element.
//  * b2_swiglu -- kernel::SwiGLU (.../math/kernel_swiglu.cc:13-20):
//    a * sigmoid(alpha a) * b with sigmoid = 1 / (1 + exp(-alpha a)).
//    CUDA's expf / exp differ from the host library's by at most a couple of
//    ulps, so FLOAT agrees to about 1e-7 relative rather than bit for bit.
#include "b2_common.cuh"

namespace b2 {

// Positions outside the cos/sin cache seen by the rotary kernel since the last
// reset (the reference throws, kernel_rotary_embedding.cc:177-180; a device
// kernel cannot, so it writes zeros and records it here).
__device__ int g_rotary_status;

namespace {

template <typename T> struct Act;
template <> struct Act<float> {
  static __device__ __forceinline__ float ld(const void *p, int64_t i) {
    return reinterpret_cast<const float *>(p)[i];
  }
  static __device__ __forceinline__ void st(void *p, int64_t i, float v) {
    reinterpret_cast<float *>(p)[i] = v;
  }
  static __device__ __forceinline__ float round(float v) { return v; }
};
template <> struct Act<__half> {
  static __device__ __forceinline__ float ld(const void *p, int64_t i) {
    return f16_bits_to_f32(reinterpret_cast<const uint16_t *>(p)[i]);
  }
  static __device__ __forceinline__ void st(void *p, int64_t i, float v) {
    reinterpret_cast<uint16_t *>(p)[i] = f32_to_f16_bits(v);
  }
  static __device__ __forceinline__ float round(float v) { return f16_bits_to_f32(f32_to_f16_bits(v)); }
};
template <> struct Act<__nv_bfloat16> {
  static __device__ __forceinline__ float ld(const void *p, int64_t i) {
    return __uint_as_float((uint32_t)reinterpret_cast<const uint16_t *>(p)[i] << 16);
  }
  static __device__ __forceinline__ void st(void *p, int64_t i, float v) {
    reinterpret_cast<uint16_t *>(p)[i] = f32_to_bf16_bits(v);
  }
  static __device__ __forceinline__ float round(float v) {
    return __uint_as_float((uint32_t)f32_to_bf16_bits(v) << 16);
  }
};

// Scale index of normalized-block element i: scale broadcast against the
// trailing axes (dims / strides of the normalized block, stride 0 where the
// scale dimension is 1).
struct ScaleMap {
  int mode;  // 0 scalar, 1 same shape (index i), 2 general
  int nd;
  int64_t dims[8], strides[8];
};

__device__ __forceinline__ int64_t scale_index(const ScaleMap &m, int64_t i) {
  if (m.mode == 0) return 0;
  if (m.mode == 1) return i;
  int64_t si = 0;
  for (int d = m.nd - 1; d >= 0; --d) {
    const int64_t c = i % m.dims[d];
    i /= m.dims[d];
    si += c * m.strides[d];
  }
  return si;
}

constexpr int RMS_THREADS = 256;

template <typename T>
__global__ void __launch_bounds__(RMS_THREADS) rms_norm_kernel(const void *x, const void *scale,
                                                               void *y, int64_t norm, float eps,
                                                               const ScaleMap sm) {
  __shared__ double red[RMS_THREADS / 32];
  __shared__ float rms_s;
  const int64_t base = (int64_t)blockIdx.x * norm;
  double acc = 0.0;
  for (int64_t i = threadIdx.x; i < norm; i += RMS_THREADS) {
    const double v = (double)Act<T>::ld(x, base + i);
    acc = fma(v, v, acc); // v * v is exact in double, so the FMA adds the exact square
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double s = 0.0;
    for (int w = 0; w < RMS_THREADS / 32; ++w) s += red[w];
    const double mean = norm > 0 ? s / (double)norm : 0.0;
    rms_s = __fsqrt_rn(__fadd_rn((float)mean, eps));
  }
  __syncthreads();
  const float rms = rms_s;
  for (int64_t i = threadIdx.x; i < norm; i += RMS_THREADS) {
    const float n = __fdiv_rn(Act<T>::ld(x, base + i), rms);
    const float s = Act<T>::ld(scale, scale_index(sm, i));
    Act<T>::st(y, base + i, __fmul_rn(Act<T>::round(n), s));
  }
}

struct RotaryArgs {
  const void *x, *cos, *sin;
  const int64_t *pos; // [B, S] or nullptr
  void *y;
  int64_t B, H, S, D, half, cache_rows;
  int rank3, interleaved;
};

// One warp per row of D channels (a (batch, head, position) triple): the row
// index is split into (b, s) once, and each lane computes both outputs of its
// rotation pairs from one load of x1, x2, cos and sin; channels past the
// rotary dimension are copied.
template <typename T> __global__ void __launch_bounds__(256) rotary_kernel(const RotaryArgs a) {
  const int64_t rows = a.B * a.H * a.S;
  const int lane = threadIdx.x & 31;
  for (int64_t r = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5; r < rows;
       r += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    int64_t b, s;
    if (a.rank3) { // storage [B, S, H, D]: r = (b S + s) H + h
      const int64_t bs = r / a.H;
      b = bs / a.S;
      s = bs - b * a.S;
    } else { // [B, H, S, D]: r = (b H + h) S + s
      const int64_t bh = r / a.S;
      s = r - bh * a.S;
      b = bh / a.H;
    }
    const int64_t base = r * a.D;
    int64_t crow = b * a.S + s;
    bool valid = true;
    if (a.pos) {
      crow = a.pos[b * a.S + s];
      if (crow < 0 || crow >= a.cache_rows) {
        valid = false;
        if (lane == 0) atomicExch(&g_rotary_status, 1);
      }
    }
    for (int64_t i = lane; i < a.half; i += 32) {
      int64_t i1, i2;
      if (a.interleaved) {
        i1 = base + 2 * i;
        i2 = i1 + 1;
      } else {
        i1 = base + i;
        i2 = base + a.half + i;
      }
      if (!valid) {
        Act<T>::st(a.y, i1, 0.0f);
        Act<T>::st(a.y, i2, 0.0f);
        continue;
      }
      const float cv = Act<T>::ld(a.cos, crow * a.half + i);
      const float sv = Act<T>::ld(a.sin, crow * a.half + i);
      const float x1 = Act<T>::ld(a.x, i1), x2 = Act<T>::ld(a.x, i2);
      Act<T>::st(a.y, i1, __fsub_rn(__fmul_rn(cv, x1), __fmul_rn(sv, x2)));
      Act<T>::st(a.y, i2, __fadd_rn(__fmul_rn(sv, x1), __fmul_rn(cv, x2)));
    }
    for (int64_t c = 2 * a.half + lane; c < a.D; c += 32) Act<T>::st(a.y, base + c, Act<T>::ld(a.x, base + c));
  }
}

template <typename T>
__global__ void swiglu_kernel(const void *a, const void *b, void *y, int64_t n, float alpha) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float av = Act<T>::ld(a, i), bv = Act<T>::ld(b, i);
    const float s = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(__fmul_rn(-alpha, av))));
    Act<T>::st(y, i, __fmul_rn(__fmul_rn(av, s), bv));
  }
}

__global__ void swiglu_f64_kernel(const double *a, const double *b, double *y, int64_t n,
                                  double alpha) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const double s = __ddiv_rn(1.0, __dadd_rn(1.0, exp(__dmul_rn(-alpha, a[i]))));
    y[i] = __dmul_rn(__dmul_rn(a[i], s), b[i]);
  }
}

unsigned grid_for(int64_t n, int threads) {
  int64_t blocks = (n + threads - 1) / threads;
  const int64_t cap = (int64_t)sm_count() * 16;
  if (blocks > cap) blocks = cap;
  return (unsigned)(blocks < 1 ? 1 : blocks);
}

bool is_float_type(int dt) { return dt == kFloat || dt == kFloat16 || dt == kBfloat16; }

} // namespace

int status_read_rotary(int reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_rotary_status, sizeof(int)) != cudaSuccess) return -1;
  if (reset && v) {
    const int z = 0;
    if (cudaMemcpyToSymbol(g_rotary_status, &z, sizeof(int)) != cudaSuccess) return -1;
  }
  return v;
}

} // namespace b2

using namespace b2;

extern "C" int b2_rms_normalization(const b2_tensor *x, const b2_tensor *scale, int64_t axis,
                                    float epsilon, b2_tensor *y, void *stream) {
  if (!x || !scale || !y) B2_FAIL(B2_ERR_INVALID_ARGUMENT, "kernel::RMSNormalization: null tensor");
  B2_ENFORCE(is_float_type(x->dtype), "kernel::RMSNormalization: X must be FLOAT, FLOAT16 or BFLOAT16.");
  B2_ENFORCE(scale->dtype == x->dtype, "kernel::RMSNormalization: scale must have the same dtype as X.");
  B2_ENFORCE(y->dtype == x->dtype, "kernel::RMSNormalization: output must have the same dtype as X.");
  B2_ENFORCE(shape_of(y) == shape_of(x), "kernel::RMSNormalization: output must have the same shape as X.");
  const int64_t rank = x->ndim;
  B2_ENFORCE(rank >= 1, "kernel::RMSNormalization: X must have rank >= 1.");
  if (axis < 0) axis += rank;
  B2_ENFORCE(axis >= 0 && axis < rank, "kernel::RMSNormalization: axis out of range for X's rank.");
  const int64_t nrank = rank - axis;
  B2_ENFORCE(scale->ndim <= nrank, "kernel::RMSNormalization: scale rank cannot exceed normalized rank.");
  const int64_t off = nrank - scale->ndim;
  for (int i = 0; i < scale->ndim; ++i) {
    const int64_t xd = x->shape[axis + off + i], sd = scale->shape[i];
    B2_ENFORCE(sd == xd || sd == 1,
               "kernel::RMSNormalization: scale shape is not broadcastable to X's normalized shape.");
  }
  int64_t outer = 1, norm = 1;
  for (int64_t i = 0; i < axis; ++i) outer *= x->shape[i];
  for (int64_t i = axis; i < rank; ++i) norm *= x->shape[i];
  if (nrank > 8) B2_FAIL(B2_ERR_UNSUPPORTED, "kernel::RMSNormalization: more than 8 normalized axes");
  ScaleMap sm{};
  const int64_t sn = numel(scale);
  sm.mode = sn == 1 ? 0 : sn == norm ? 1 : 2;
  sm.nd = (int)nrank;
  {
    int64_t st = 1;
    for (int64_t d = nrank - 1; d >= 0; --d) {
      sm.dims[d] = x->shape[axis + d];
      const int64_t sdim = d >= off ? scale->shape[d - off] : 1;
      sm.strides[d] = sdim == 1 ? 0 : st;
      st *= sdim;
    }
  }
  if (outer == 0 || norm == 0) return B2_OK;
  if (outer >= (int64_t)1 << 31) B2_FAIL(B2_ERR_UNSUPPORTED, "kernel::RMSNormalization: too many rows");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (x->dtype == kFloat16)
    rms_norm_kernel<__half><<<(unsigned)outer, RMS_THREADS, 0, st>>>(x->data, scale->data, y->data, norm, epsilon, sm);
  else if (x->dtype == kBfloat16)
    rms_norm_kernel<__nv_bfloat16><<<(unsigned)outer, RMS_THREADS, 0, st>>>(x->data, scale->data, y->data, norm, epsilon, sm);
  else
    rms_norm_kernel<float><<<(unsigned)outer, RMS_THREADS, 0, st>>>(x->data, scale->data, y->data, norm, epsilon, sm);
  B2_LAUNCH_CHECK();
  return B2_OK;
}

extern "C" int b2_rotary_embedding(const b2_tensor *x, const b2_tensor *cos_cache,
                                   const b2_tensor *sin_cache, const b2_tensor *position_ids,
                                   int32_t interleaved, int64_t rotary_embedding_dim,
                                   int64_t num_heads, b2_tensor *y, void *stream) {
  if (!x || !cos_cache || !sin_cache || !y)
    B2_FAIL(B2_ERR_INVALID_ARGUMENT, "kernel::RotaryEmbedding: null tensor");
  B2_ENFORCE(is_float_type(x->dtype), "kernel::RotaryEmbedding: X must be FLOAT, FLOAT16 or BFLOAT16.");
  B2_ENFORCE(x->ndim == 3 || x->ndim == 4, "kernel::RotaryEmbedding: X must have rank 3 or 4.");
  RotaryArgs a{};
  a.rank3 = x->ndim == 3;
  a.B = x->shape[0];
  if (a.rank3) {
    a.S = x->shape[1];
    B2_ENFORCE(num_heads > 0, "kernel::RotaryEmbedding: num_heads attribute is required for rank-3 X.");
    a.H = num_heads;
    B2_ENFORCE(x->shape[2] % num_heads == 0,
               "kernel::RotaryEmbedding: hidden_size must be divisible by num_heads.");
    a.D = x->shape[2] / num_heads;
  } else {
    a.H = x->shape[1];
    a.S = x->shape[2];
    a.D = x->shape[3];
  }
  B2_ENFORCE(a.D % 2 == 0, "kernel::RotaryEmbedding: head_size must be even.");
  int64_t rot = rotary_embedding_dim == 0 ? a.D : rotary_embedding_dim;
  B2_ENFORCE(rot > 0 && rot % 2 == 0 && rot <= a.D,
             "kernel::RotaryEmbedding: rotary_embedding_dim must be even and <= head_size.");
  a.half = rot / 2;
  const bool has_pos = position_ids != nullptr && position_ids->ndim > 0;
  if (has_pos) {
    B2_ENFORCE(position_ids->dtype == kInt64, "kernel::RotaryEmbedding: position_ids must be INT64.");
    B2_ENFORCE(position_ids->ndim == 2 && position_ids->shape[0] == a.B &&
                   position_ids->shape[1] == a.S,
               "kernel::RotaryEmbedding: position_ids must have shape (batch, seq).");
  }
  const b2_tensor *caches[2] = {cos_cache, sin_cache};
  const char *names[2] = {"cos_cache", "sin_cache"};
  for (int c = 0; c < 2; ++c) {
    const b2_tensor *t = caches[c];
    B2_ENFORCE(t->dtype == x->dtype, "kernel::RotaryEmbedding: %s must have the same dtype as X.", names[c]);
    if (has_pos) {
      B2_ENFORCE(t->ndim == 2, "kernel::RotaryEmbedding: %s must be rank-2 when position_ids is provided.",
                 names[c]);
      B2_ENFORCE(t->shape[1] == a.half,
                 "kernel::RotaryEmbedding: last dim of %s (%lld) must equal rotary_embedding_dim/2 (%lld).",
                 names[c], (long long)t->shape[1], (long long)a.half);
    } else {
      B2_ENFORCE(t->ndim == 3, "kernel::RotaryEmbedding: %s must be rank-3 when position_ids is omitted.",
                 names[c]);
      B2_ENFORCE(t->shape[0] == a.B && t->shape[1] == a.S && t->shape[2] == a.half,
                 "kernel::RotaryEmbedding: %s has unexpected shape; expected (batch, seq, rotary_dim/2).",
                 names[c]);
    }
  }
  B2_ENFORCE(y->dtype == x->dtype && shape_of(y) == shape_of(x),
             "kernel::RotaryEmbedding: output buffer has mismatched type or shape.");
  a.x = x->data;
  a.cos = cos_cache->data;
  a.sin = sin_cache->data;
  a.pos = has_pos ? static_cast<const int64_t *>(position_ids->data) : nullptr;
  a.cache_rows = has_pos ? cos_cache->shape[0] : 0;
  a.y = y->data;
  a.interleaved = interleaved != 0;
  const int64_t total = a.B * a.H * a.S * a.D;
  if (total == 0) return B2_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // one warp per (batch, head, position) row
  const unsigned grid = grid_for(total / a.D * 32, 256);
  if (x->dtype == kFloat16) rotary_kernel<__half><<<grid, 256, 0, st>>>(a);
  else if (x->dtype == kBfloat16) rotary_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(a);
  else rotary_kernel<float><<<grid, 256, 0, st>>>(a);
  B2_LAUNCH_CHECK();
  return B2_OK;
}

extern "C" int b2_swiglu(const b2_tensor *a, const b2_tensor *b, float alpha, b2_tensor *y,
                         void *stream) {
  if (!a || !b || !y) B2_FAIL(B2_ERR_INVALID_ARGUMENT, "kernel::SwiGLU: null tensor");
  if (!(is_float_type(a->dtype) || a->dtype == kDouble))
    B2_FAIL(B2_ERR_UNSUPPORTED_DTYPE,
            "kernel::SwiGLU: unsupported data type %d only supports FLOAT, DOUBLE, FLOAT16 and "
            "BFLOAT16 tensors.",
            a->dtype);
  B2_ENFORCE(shape_of(a) == shape_of(b),
             "kernel::SwiGLU: inputs A and B must have identical shapes (broadcasting is not applied).");
  B2_ENFORCE(b->dtype == a->dtype && y->dtype == a->dtype && shape_of(y) == shape_of(a),
             "kernel::SwiGLU: output must have the dtype and shape of A.");
  const int64_t n = numel(a);
  if (n == 0) return B2_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned grid = grid_for(n, 256);
  switch (a->dtype) {
  case kFloat16: swiglu_kernel<__half><<<grid, 256, 0, st>>>(a->data, b->data, y->data, n, alpha); break;
  case kBfloat16: swiglu_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(a->data, b->data, y->data, n, alpha); break;
  case kDouble:
    swiglu_f64_kernel<<<grid, 256, 0, st>>>(static_cast<const double *>(a->data),
                                            static_cast<const double *>(b->data),
                                            static_cast<double *>(y->data), n, (double)alpha);
    break;
  default: swiglu_kernel<float><<<grid, 256, 0, st>>>(a->data, b->data, y->data, n, alpha); break;
  }
  B2_LAUNCH_CHECK();
  return B2_OK;
}
