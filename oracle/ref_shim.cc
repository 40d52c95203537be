// oracle/_ref C entry points — test infrastructure only.
//
// Wraps onnx-light's own kernel classes, compiled from the reference sources
// (see oracle/Makefile), behind plain C functions so that the Python tests can
// (1) generate golden fixtures from the real reference, (2) check the C
// restatement in oracle/oracle.c against it, and (3) time the reference CPU
// path for bench.py's reference arm.  Calls go straight to each kernel's
// operator() with no RuntimeContext, exactly as the reference's unit tests do
// (unittests/cc/onnx_extensions/kernels/kernels/test_kernels_quantization.cc:263-430).
//
// Every function returns 0 on success and -1 when the reference raised an
// exception; the message is copied into `err`.
#include "onnx_core/runtime/kernels/cast_float8.h"
#include "onnx_core/runtime/kernels/float16_promote.h"
#include "onnx_core/runtime/kernels/parallel_for.h"
#include "onnx_extensions/kernels/kernels/math/include_math_kernels.h"
#include "onnx_extensions/kernels/kernels/nn/include_nn_kernels.h"
#include "onnx_extensions/kernels/kernels/quantization/include_quantization_kernels.h"

#include <cstring>
#include <exception>
#include <string>
#include <vector>

using namespace onnx_light::onnx_kernels;
using onnx_light::core::runtime::DemoteFromFloat32;
using onnx_light::core::runtime::PackedByteSize;
using onnx_light::core::runtime::PromoteToFloat32;

namespace {

kernel::KernelContext Ctx() { return kernel::KernelContext{kernel::DefaultOpset(23)}; }

Shape MakeShape(const int64_t *s, int nd) {
  Shape out;
  for (int i = 0; i < nd; ++i) out.push_back(s[i]);
  return out;
}

Tensor MakeTensor(const void *data, int dt, const int64_t *s, int nd) {
  Shape shape = MakeShape(s, nd);
  int64_t n = 1;
  for (int i = 0; i < nd; ++i) n *= s[i];
  const size_t bytes = PackedByteSize(dt, n);
  std::vector<uint8_t> buf(bytes);
  if (bytes) std::memcpy(buf.data(), data, bytes);
  return Tensor("", dt, shape, std::move(buf));
}

void Fail(const std::exception &e, char *err, size_t errlen) {
  if (err && errlen) {
    std::strncpy(err, e.what(), errlen - 1);
    err[errlen - 1] = 0;
  }
}

int CopyOut(const Tensor &t, void *out, size_t out_bytes, int64_t *out_shape, int *out_nd) {
  if (t.size_bytes() > out_bytes) throw std::runtime_error("oracle/_ref: output buffer too small");
  if (t.size_bytes()) std::memcpy(out, t.bytes(), t.size_bytes());
  if (out_nd) {
    *out_nd = static_cast<int>(t.shape.size());
    for (size_t i = 0; i < t.shape.size(); ++i) out_shape[i] = t.shape[i];
  }
  return 0;
}

} // namespace

extern "C" {

int ref_thread_count() { return static_cast<int>(onnx_light::core::runtime::ParallelForThreadCount()); }

// kernel::DequantizeLinear::operator()(x, x_scale[, x_zero_point], axis)
// (kernel_dequantizelinear.cc:504-520, 653-668).
int ref_dequantize_linear(const void *x, int x_dt, const int64_t *x_shape, int x_nd,
                          const void *s, int s_dt, const int64_t *s_shape, int s_nd,
                          const void *zp, const int64_t *zp_shape, int zp_nd, int64_t axis,
                          void *y, size_t y_bytes, char *err, size_t errlen) {
  try {
    const kernel::KernelContext ctx = Ctx();
    kernel::DequantizeLinear k(ctx);
    Tensor tx = MakeTensor(x, x_dt, x_shape, x_nd);
    Tensor ts = MakeTensor(s, s_dt, s_shape, s_nd);
    Tensor out;
    if (zp) {
      Tensor tz = MakeTensor(zp, x_dt, zp_shape, zp_nd);
      out = k(tx, ts, tz, axis);
    } else {
      out = k(tx, ts, axis);
    }
    return CopyOut(out, y, y_bytes, nullptr, nullptr);
  } catch (const std::exception &e) {
    Fail(e, err, errlen);
    return -1;
  }
}

// kernel::MatMul::operator()(a, b) (kernel_matmul.cc:181-223).
int ref_matmul(const void *a, const int64_t *as, int an, const void *b, const int64_t *bs, int bn,
               int dt, void *y, size_t y_bytes, int64_t *y_shape, int *y_nd, char *err,
               size_t errlen) {
  try {
    const kernel::KernelContext ctx = Ctx();
    kernel::MatMul k(ctx);
    Tensor out = k(MakeTensor(a, dt, as, an), MakeTensor(b, dt, bs, bn));
    return CopyOut(out, y, y_bytes, y_shape, y_nd);
  } catch (const std::exception &e) {
    Fail(e, err, errlen);
    return -1;
  }
}

// kernel::MatMulInteger::operator()(a, b, a_zp, b_zp) (kernel_matmul_integer.cc:212-229);
// a null zero point is passed as an empty Tensor, as MatMulInteger::Run does (:244-248).
int ref_matmul_integer(const void *a, int a_dt, const int64_t *as, int an, const void *b, int b_dt,
                       const int64_t *bs, int bn, const void *azp, const int64_t *azs, int azn,
                       const void *bzp, const int64_t *bzs, int bzn, void *y, size_t y_bytes,
                       int64_t *y_shape, int *y_nd, char *err, size_t errlen) {
  try {
    const kernel::KernelContext ctx = Ctx();
    kernel::MatMulInteger k(ctx);
    Tensor ta = MakeTensor(a, a_dt, as, an), tb = MakeTensor(b, b_dt, bs, bn);
    Tensor tza = azp ? MakeTensor(azp, a_dt, azs, azn) : Tensor{};
    Tensor tzb = bzp ? MakeTensor(bzp, b_dt, bzs, bzn) : Tensor{};
    Tensor out = k(ta, tb, tza, tzb);
    return CopyOut(out, y, y_bytes, y_shape, y_nd);
  } catch (const std::exception &e) {
    Fail(e, err, errlen);
    return -1;
  }
}

// kernel::QLinearMatMul::operator() (kernel_qlinearmatmul.cc:221-240).  Scales are
// scalars of dtype s_dt (FLOAT or FLOAT16, given as raw bytes); zero points are
// scalars of the matching integer dtype.
int ref_qlinear_matmul(const void *a, int a_dt, const int64_t *as, int an, const void *a_s,
                       const void *a_zp, const void *b, int b_dt, const int64_t *bs, int bn,
                       const void *b_s, const void *b_zp, const void *y_s, const void *y_zp,
                       int y_dt, int s_dt, void *y, size_t y_bytes, int64_t *y_shape, int *y_nd,
                       char *err, size_t errlen) {
  try {
    const kernel::KernelContext ctx = Ctx();
    kernel::QLinearMatMul k(ctx);
    const int64_t none[1] = {0};
    Tensor out = k(MakeTensor(a, a_dt, as, an), MakeTensor(a_s, s_dt, none, 0),
                   MakeTensor(a_zp, a_dt, none, 0), MakeTensor(b, b_dt, bs, bn),
                   MakeTensor(b_s, s_dt, none, 0), MakeTensor(b_zp, b_dt, none, 0),
                   MakeTensor(y_s, s_dt, none, 0), MakeTensor(y_zp, y_dt, none, 0));
    return CopyOut(out, y, y_bytes, y_shape, y_nd);
  } catch (const std::exception &e) {
    Fail(e, err, errlen);
    return -1;
  }
}

// kernel::Attention::operator()(Q, K, V, attrs, mask, past_key, past_value,
// nonpad_kv_seqlen) (kernel_attention.cc:767-852).  For FLOAT16/BFLOAT16
// inputs this mirrors the kernel's own half-precision path (:783-835): every
// input (a half-precision mask too) is promoted with PromoteToFloat32, the
// float32 kernel runs, and Y / present_key / present_value /
// qk_matmul_output are demoted with DemoteFromFloat32.  (That path builds a
// scratch RuntimeContext, which this link-light build does not carry, so the
// calls are made here instead.)  Without a node or context all four outputs
// are produced (:855-861).
int ref_attention(const void *q, const int64_t *qs, const void *k, const int64_t *ks, const void *v,
                  const int64_t *vs, int rank, int dt, const void *mask, int mask_dt,
                  const int64_t *ms, int mn, const void *past_k, const void *past_v,
                  const int64_t *ps, const int64_t *pvs, const int64_t *nonpad, int64_t nonpad_n,
                  int has_scale, float scale, int is_causal, float softcap, int64_t q_num_heads,
                  int64_t kv_num_heads, int64_t left_window, int64_t right_window, int qk_mode,
                  void *y, size_t y_bytes, void *present_k, void *present_v,
                  size_t present_k_bytes, size_t present_v_bytes, void *qk, size_t qk_bytes,
                  char *err, size_t errlen) {
  try {
    const kernel::KernelContext ctx = Ctx();
    kernel::Attention att(ctx);
    kernel::Attention::Attributes attrs;
    attrs.has_scale = has_scale != 0;
    attrs.scale = scale;
    attrs.is_causal = is_causal != 0;
    attrs.softcap = softcap;
    attrs.q_num_heads = q_num_heads;
    attrs.kv_num_heads = kv_num_heads;
    attrs.left_window_size = left_window;
    attrs.right_window_size = right_window;
    attrs.qk_matmul_output_mode = qk_mode;
    const bool half = dt != 1;
    auto up = [&](const void *p, const int64_t *s, int n, int t) {
      Tensor x = MakeTensor(p, t, s, n);
      return (t == 10 || t == 16) ? PromoteToFloat32(x) : x;
    };
    Tensor tq = up(q, qs, rank, dt), tk = up(k, ks, rank, dt), tv = up(v, vs, rank, dt);
    Tensor tm, tpk, tpv, tnp;
    // A half-precision mask is promoted only on the half-precision entry
    // (kernel_attention.cc:797-801); BOOL and FLOAT masks pass unchanged.
    if (mask) tm = half ? up(mask, ms, mn, mask_dt) : MakeTensor(mask, mask_dt, ms, mn);
    if (past_k) {
      tpk = up(past_k, ps, 4, dt);
      tpv = up(past_v, pvs, 4, dt);
    }
    if (nonpad) tnp = MakeTensor(nonpad, 7, &nonpad_n, 1);
    kernel::Attention::Result r =
        att(tq, tk, tv, attrs, mask ? &tm : nullptr, past_k ? &tpk : nullptr,
            past_v ? &tpv : nullptr, nonpad ? &tnp : nullptr);
    Tensor ty = half ? DemoteFromFloat32(r.Y, dt) : r.Y;
    CopyOut(ty, y, y_bytes, nullptr, nullptr);
    if (present_k && r.present_key.size_bytes()) {
      Tensor pk = half ? DemoteFromFloat32(r.present_key, dt) : r.present_key;
      Tensor pv = half ? DemoteFromFloat32(r.present_value, dt) : r.present_value;
      CopyOut(pk, present_k, present_k_bytes, nullptr, nullptr);
      CopyOut(pv, present_v, present_v_bytes, nullptr, nullptr);
    }
    if (qk && r.qk_matmul_output.size_bytes()) {
      Tensor tqk = half ? DemoteFromFloat32(r.qk_matmul_output, dt) : r.qk_matmul_output;
      CopyOut(tqk, qk, qk_bytes, nullptr, nullptr);
    }
    return 0;
  } catch (const std::exception &e) {
    Fail(e, err, errlen);
    return -1;
  }
}

// kernel::RMSNormalization::operator()(x, scale, axis, epsilon)
// (kernel_rmsnormalization.cc:68-214).
int ref_rms_normalization(const void *x, const int64_t *xs, int xn, int dt, const void *scale,
                          const int64_t *ss, int sn, int64_t axis, float epsilon, void *y,
                          size_t y_bytes, char *err, size_t errlen) {
  try {
    kernel::RMSNormalization k(Ctx());
    Tensor r = k(MakeTensor(x, dt, xs, xn), MakeTensor(scale, dt, ss, sn), axis, epsilon);
    CopyOut(r, y, y_bytes, nullptr, nullptr);
    return 0;
  } catch (const std::exception &e) {
    Fail(e, err, errlen);
    return -1;
  }
}

// kernel::RotaryEmbedding::operator()(X, cos_cache, sin_cache, position_ids,
// attrs) (kernel_rotary_embedding.cc:47-218).
int ref_rotary_embedding(const void *x, const int64_t *xs, int xn, int dt, const void *c,
                         const void *s, const int64_t *cs, int cn, const int64_t *pos,
                         const int64_t *ps, int pn, int interleaved, int64_t rotary_dim,
                         int64_t num_heads, void *y, size_t y_bytes, char *err, size_t errlen) {
  try {
    kernel::RotaryEmbedding k(Ctx());
    kernel::RotaryEmbedding::Attributes attrs;
    attrs.interleaved = interleaved != 0;
    attrs.rotary_embedding_dim = rotary_dim;
    attrs.num_heads = num_heads;
    Tensor tp;
    if (pos) tp = MakeTensor(pos, 7, ps, pn);
    // FLOAT16 / BFLOAT16 mirror the kernel's own half path (:65-88): promote,
    // run in float32, demote (its scratch RuntimeContext is not carried here).
    const bool half = dt != 1;
    auto up = [&](Tensor t) { return half ? PromoteToFloat32(t) : t; };
    Tensor r = k(up(MakeTensor(x, dt, xs, xn)), up(MakeTensor(c, dt, cs, cn)),
                 up(MakeTensor(s, dt, cs, cn)), tp, attrs);
    CopyOut(half ? DemoteFromFloat32(r, dt) : r, y, y_bytes, nullptr, nullptr);
    return 0;
  } catch (const std::exception &e) {
    Fail(e, err, errlen);
    return -1;
  }
}

// kernel::SwiGLU::operator()(a, b, alpha) (kernel_swiglu.cc:58-85).
int ref_swiglu(const void *a, const void *b, const int64_t *shp, int nd, int dt, float alpha, void *y,
               size_t y_bytes, char *err, size_t errlen) {
  try {
    kernel::SwiGLU k(Ctx());
    Tensor r = k(MakeTensor(a, dt, shp, nd), MakeTensor(b, dt, shp, nd), alpha);
    CopyOut(r, y, y_bytes, nullptr, nullptr);
    return 0;
  } catch (const std::exception &e) {
    Fail(e, err, errlen);
    return -1;
  }
}

// FloatToFloat8E4M3FNBits (cast_float8.cc:27-80), exposed so that the
// restatement's encoder can be compared against it.
uint8_t ref_f32_to_f8e4m3fn(float v) { return onnx_light::core::runtime::FloatToFloat8E4M3FNBits(v); }

} // extern "C"
