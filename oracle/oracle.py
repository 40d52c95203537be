"""CPU oracle — test infrastructure only.

numpy front end for two shared libraries built by ``oracle/Makefile``:

* ``liboracle.so`` — the C restatement of onnx-light's CPU kernels
  (``oracle/oracle.c``; each function there cites the reference file:line it
  follows);
* ``_ref/libref.so`` — onnx-light's own kernels compiled from the reference
  sources (``oracle/ref_shim.cc``), used to pin the restatement and, in
  ``bench.py --impl reference``, as the timed CPU baseline.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg import this module.  The shipped library never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

# ONNX TensorProto.DataType codes (onnx_proto/include/onnx_proto/onnx.h:300-330).
FLOAT, UINT8, INT8, UINT16, INT16, INT32, INT64, BOOL = 1, 2, 3, 4, 5, 6, 7, 9
FLOAT16, DOUBLE, BFLOAT16 = 10, 11, 16
F8E4M3FN, F8E4M3FNUZ, F8E5M2, F8E5M2FNUZ = 17, 18, 19, 20
UINT4, INT4, F4E2M1, F8E8M0, UINT2, INT2, F6E2M3, F6E3M2 = 21, 22, 23, 24, 25, 26, 27, 28

SUB_BYTE_BITS = {UINT4: 4, INT4: 4, F4E2M1: 4, UINT2: 2, INT2: 2, F6E2M3: 6, F6E3M2: 6}
ELEM_BYTES = {FLOAT: 4, UINT8: 1, INT8: 1, UINT16: 2, INT16: 2, INT32: 4, INT64: 8, BOOL: 1,
              FLOAT16: 2, DOUBLE: 8, BFLOAT16: 2, F8E4M3FN: 1, F8E4M3FNUZ: 1, F8E5M2: 1,
              F8E5M2FNUZ: 1}


def packed_nbytes(dtype: int, n: int) -> int:
    """Storage bytes of n elements (simple_tensor.cc:205-231)."""
    if dtype in (UINT4, INT4, F4E2M1):
        return n // 2 + (n % 2)
    if dtype in (UINT2, INT2):
        return n // 4 + (1 if n % 4 else 0)
    if dtype in (F6E2M3, F6E3M2):
        return n // 4 * 3 + (n % 4 * 6 + 7) // 8
    return n * ELEM_BYTES[dtype]


def pack_bits(values: np.ndarray, bits: int) -> np.ndarray:
    """Packs small integer codes low-order-first (cast_sub_byte.h:48-60)."""
    v = np.asarray(values, dtype=np.int64).ravel() & ((1 << bits) - 1)
    per = 8 // bits
    pad = (-len(v)) % per
    v = np.concatenate([v, np.zeros(pad, np.int64)]).reshape(-1, per)
    out = np.zeros(v.shape[0], np.int64)
    for k in range(per):
        out |= v[:, k] << (k * bits)
    return out.astype(np.uint8)


def _build(target: str) -> None:
    subprocess.run(["make", "-s", "-C", HERE, target], check=True)


def _load(path: str, target: str):
    if not os.path.exists(path):
        _build(target)
    return C.CDLL(path)


_lib = None
_ref = None


def lib():
    global _lib
    if _lib is None:
        _lib = _load(os.path.join(HERE, "liboracle.so"), "liboracle")
        _declare_oracle(_lib)
    return _lib


def ref_available() -> bool:
    return os.path.exists(os.path.join(HERE, "_ref", "libref.so"))


def ref():
    """onnx-light's own kernels (oracle/_ref).  Raises when not built."""
    global _ref
    if _ref is None:
        path = os.path.join(HERE, "_ref", "libref.so")
        if not os.path.exists(path):
            raise FileNotFoundError("oracle/_ref/libref.so is not built (make -C oracle ref)")
        _ref = C.CDLL(path)
        _ref.ref_f32_to_f8e4m3fn.restype = C.c_uint8
        _ref.ref_f32_to_f8e4m3fn.argtypes = [C.c_float]
    return _ref


P = C.c_void_p
I64P = C.POINTER(C.c_int64)


def _declare_oracle(L):
    L.orc_f32_to_f16.restype = C.c_uint16
    L.orc_f32_to_f16.argtypes = [C.c_float]
    L.orc_f16_to_f32.restype = C.c_float
    L.orc_f16_to_f32.argtypes = [C.c_uint16]
    L.orc_f32_to_f8e4m3fn.restype = C.c_uint8
    L.orc_f32_to_f8e4m3fn.argtypes = [C.c_float]
    L.orc_rand_uniform_f32.argtypes = [C.c_uint64, C.c_int64, C.c_double, C.c_double, P]
    L.orc_randn_f32.argtypes = [C.c_uint64, C.c_int64, C.c_double, C.c_double, P]
    L.orc_randint.argtypes = [C.c_uint64, C.c_int64, C.c_int64, C.c_int64, P]
    L.orc_dequantize_linear.argtypes = [P, C.c_int, I64P, C.c_int, P, C.c_int, I64P, C.c_int,
                                        P, C.c_int, I64P, C.c_int, C.c_int64, P]
    L.orc_matmul_shape.argtypes = [I64P, C.c_int, I64P, C.c_int, I64P, C.POINTER(C.c_int)]
    L.orc_matmul.argtypes = [P, I64P, C.c_int, P, I64P, C.c_int, C.c_int, P]
    L.orc_matmul_integer.argtypes = [P, C.c_int, I64P, C.c_int, P, C.c_int, I64P, C.c_int,
                                     P, C.c_int64, P, C.c_int64, P]
    L.orc_qlinear_matmul.argtypes = [P, C.c_int, I64P, C.c_int, C.c_float, C.c_int32,
                                     P, C.c_int, I64P, C.c_int, C.c_float, C.c_int32,
                                     C.c_float, C.c_int32, C.c_int, P]
    L.orc_attention_f32.argtypes = [P, P, P] + [C.c_int64] * 7 + [C.c_float, C.c_int, C.c_int64,
                                                                   C.c_float, P, I64P, C.c_int64,
                                                                   C.c_int64, P, P, C.c_int, P]
    L.orc_rms_norm_f32.argtypes = [P, P, C.c_int64, C.c_int64, C.c_float, C.c_int, P]
    L.orc_rotary_f32.argtypes = [P, P, P, P] + [C.c_int64] * 5 + [C.c_int, C.c_int, C.c_int64, P]
    L.orc_swiglu_f32.argtypes = [P, P, C.c_int64, C.c_float, P]
    for fn in ("orc_f16_to_f32_n", "orc_f32_to_f16_n", "orc_bf16_to_f32_n", "orc_f32_to_bf16_n",
               "orc_f32_to_f8e4m3fn_n"):
        getattr(L, fn).argtypes = [P, P, C.c_int64]
    L.orc_decode_n.argtypes = [C.c_int, P, P, C.c_int64]


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(P) if a is not None else None


def _shape(s):
    arr = (C.c_int64 * max(1, len(s)))(*[int(d) for d in s])
    return arr, len(s)


class OracleError(ValueError):
    pass


def _check(rc: int, what: str):
    if rc != 0:
        raise OracleError(f"oracle {what} rejected its inputs (code {rc})")


# ---------------------------------------------------------------------------
# Conversions
# ---------------------------------------------------------------------------

def f16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    b = np.ascontiguousarray(bits, np.uint16)
    out = np.empty(b.shape, np.float32)
    lib().orc_f16_to_f32_n(_ptr(b), _ptr(out), b.size)
    return out


def f32_to_f16_bits(x: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(x, np.float32)
    out = np.empty(a.shape, np.uint16)
    lib().orc_f32_to_f16_n(_ptr(a), _ptr(out), a.size)
    return out


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    b = np.ascontiguousarray(bits, np.uint16)
    out = np.empty(b.shape, np.float32)
    lib().orc_bf16_to_f32_n(_ptr(b), _ptr(out), b.size)
    return out


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(x, np.float32)
    out = np.empty(a.shape, np.uint16)
    lib().orc_f32_to_bf16_n(_ptr(a), _ptr(out), a.size)
    return out


def f32_to_f8e4m3fn(x: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(x, np.float32)
    out = np.empty(a.shape, np.uint8)
    lib().orc_f32_to_f8e4m3fn_n(_ptr(a), _ptr(out), a.size)
    return out


def decode(dtype: int, raw: np.ndarray, n: int) -> np.ndarray:
    """Element values of a quantized tensor as float32 (no scale, no zero point)."""
    r = np.ascontiguousarray(raw, np.uint8)
    out = np.empty(n, np.float32)
    lib().orc_decode_n(dtype, _ptr(r), _ptr(out), n)
    return out


# ---------------------------------------------------------------------------
# SplitMix64 generators (random.cc:38-176)
# ---------------------------------------------------------------------------

def rand_uniform(seed: int, shape, lo: float, hi: float) -> np.ndarray:
    out = np.empty(shape, np.float32)
    lib().orc_rand_uniform_f32(seed, out.size, lo, hi, _ptr(out))
    return out


def randn(seed: int, shape, mean: float = 0.0, scale: float = 1.0) -> np.ndarray:
    out = np.empty(shape, np.float32)
    lib().orc_randn_f32(seed, out.size, mean, scale, _ptr(out))
    return out


def randint(seed: int, shape, lo: int, hi_inclusive: int) -> np.ndarray:
    out = np.empty(shape, np.int64)
    lib().orc_randint(seed, out.size, lo, hi_inclusive + 1, _ptr(out))
    return out


# ---------------------------------------------------------------------------
# Kernels
# ---------------------------------------------------------------------------

def dequantize_linear(x_raw: np.ndarray, x_dt: int, x_shape, scale_raw: np.ndarray, s_dt: int,
                      s_shape, zp_raw=None, zp_shape=None, axis: int = 1) -> np.ndarray:
    """Returns the output's raw storage: float32 values or float16 bit patterns."""
    n = int(np.prod(x_shape)) if len(x_shape) else 1
    out = np.empty(n, np.float32 if s_dt == FLOAT else np.uint16)
    xs, xn = _shape(x_shape)
    ss, sn = _shape(s_shape)
    zs, zn = _shape(zp_shape if zp_shape is not None else [])
    x_raw = np.ascontiguousarray(x_raw, np.uint8)
    scale_raw = np.ascontiguousarray(scale_raw).view(np.uint8)
    zp = None if zp_raw is None else np.ascontiguousarray(zp_raw, np.uint8)
    rc = lib().orc_dequantize_linear(_ptr(x_raw), x_dt, xs, xn, _ptr(scale_raw), s_dt, ss, sn,
                                     _ptr(zp), x_dt, zs, zn, axis, _ptr(out))
    _check(rc, "DequantizeLinear")
    return out.reshape(tuple(x_shape))


def matmul_shape(a_shape, b_shape):
    a, an = _shape(a_shape)
    b, bn = _shape(b_shape)
    out = (C.c_int64 * 16)()
    nd = C.c_int()
    _check(lib().orc_matmul_shape(a, an, b, bn, out, C.byref(nd)), "MatMul shape")
    return tuple(out[i] for i in range(nd.value))


def matmul(a: np.ndarray, b: np.ndarray, dt: int) -> np.ndarray:
    """a, b: float32 arrays (FLOAT) or uint16 bit patterns (FLOAT16 / BFLOAT16)."""
    shape = matmul_shape(a.shape, b.shape)
    out = np.empty(shape, np.float32 if dt == FLOAT else np.uint16)
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b)
    asz, an = _shape(a.shape)
    bsz, bn = _shape(b.shape)
    _check(lib().orc_matmul(_ptr(a), asz, an, _ptr(b), bsz, bn, dt, _ptr(out)), "MatMul")
    return out


def matmul_integer(a: np.ndarray, a_dt: int, b: np.ndarray, b_dt: int, a_zp=None, b_zp=None):
    shape = matmul_shape(a.shape, b.shape)
    out = np.empty(shape, np.int32)
    a = np.ascontiguousarray(a).view(np.uint8)
    b = np.ascontiguousarray(b).view(np.uint8)
    az = None if a_zp is None else np.ascontiguousarray(a_zp).view(np.uint8).ravel()
    bz = None if b_zp is None else np.ascontiguousarray(b_zp).view(np.uint8).ravel()
    asz, an = _shape(a.shape)
    bsz, bn = _shape(b.shape)
    rc = lib().orc_matmul_integer(_ptr(a), a_dt, asz, an, _ptr(b), b_dt, bsz, bn,
                                  _ptr(az), 0 if az is None else az.size,
                                  _ptr(bz), 0 if bz is None else bz.size, _ptr(out))
    _check(rc, "MatMulInteger")
    return out


def qlinear_matmul(a, a_dt, a_scale: float, a_zp: int, b, b_dt, b_scale: float, b_zp: int,
                   y_scale: float, y_zp: int, y_dt: int):
    shape = matmul_shape(a.shape, b.shape)
    out = np.empty(shape, np.uint8)
    a = np.ascontiguousarray(a).view(np.uint8)
    b = np.ascontiguousarray(b).view(np.uint8)
    asz, an = _shape(a.shape)
    bsz, bn = _shape(b.shape)
    rc = lib().orc_qlinear_matmul(_ptr(a), a_dt, asz, an, a_scale, a_zp, _ptr(b), b_dt, bsz, bn,
                                  b_scale, b_zp, y_scale, y_zp, y_dt, _ptr(out))
    _check(rc, "QLinearMatMul")
    return out.view(np.int8) if y_dt == INT8 else out


def mask_to_float(mask):
    """A FLOAT, BOOL (numpy bool) or half-precision (float16 / bfloat16 bits
    given as ('bf16', uint16 array)) attention mask as the float32 bias the
    reference kernel adds: BOOL true -> 0, false -> -inf
    (kernel_attention.cc:391-392); half masks promoted to float32 (:797-801)."""
    if isinstance(mask, tuple) and mask[0] == "bf16":
        return bf16_bits_to_f32(mask[1])
    m = np.asarray(mask)
    if m.dtype == np.bool_:
        return np.where(m, np.float32(0.0), np.float32(-np.inf)).astype(np.float32)
    if m.dtype == np.float16:
        return m.astype(np.float32)
    return np.ascontiguousarray(m, np.float32)


def attention_f32(q, k, v, scale=None, is_causal=False, past_len=0, softcap=0.0, mask=None,
                  left_window=-1, right_window=-1, nonpad=None, qk_mode=None):
    """Rank-4 float32 attention over an already-concatenated KV (B,Hkv,L,D).

    Returns Y, or (Y, qk) when qk_mode (0..3) asks for qk_matmul_output."""
    q = np.ascontiguousarray(q, np.float32)
    k = np.ascontiguousarray(k, np.float32)
    v = np.ascontiguousarray(v, np.float32)
    B, Hq, Sq, D = q.shape
    _, Hkv, L, _ = k.shape
    Dv = v.shape[3]
    if scale is None:
        scale = float(np.float32(1.0) / np.sqrt(np.float32(D)))
    y = np.empty((B, Hq, Sq, Dv), np.float32)
    m = None
    ms = (C.c_int64 * 4)(1, 1, 1, 1)
    if mask is not None:
        m = np.ascontiguousarray(mask_to_float(mask), np.float32)
        shp = [1] * (4 - m.ndim) + list(m.shape)
        ms = (C.c_int64 * 4)(*shp)
    npd = None if nonpad is None else np.ascontiguousarray(nonpad, np.int64)
    qk = None if qk_mode is None else np.zeros((B, Hq, Sq, L), np.float32)
    rc = lib().orc_attention_f32(_ptr(q), _ptr(k), _ptr(v), B, Hq, Hkv, Sq, L, D, Dv, scale,
                                 int(is_causal), past_len, softcap, _ptr(m), ms, left_window,
                                 right_window, _ptr(npd), _ptr(qk), int(qk_mode or 0), _ptr(y))
    _check(rc, "Attention")
    return y if qk_mode is None else (y, qk)


def _up(raw, dt):
    if dt == FLOAT16:
        return f16_bits_to_f32(raw)
    if dt == BFLOAT16:
        return bf16_bits_to_f32(raw)
    return np.ascontiguousarray(raw, np.float32)


def _down(v, dt):
    if dt == FLOAT16:
        return f32_to_f16_bits(v)
    if dt == BFLOAT16:
        return f32_to_bf16_bits(v)
    return v.astype(np.float32)


def rms_normalization(x, scale, dt=FLOAT, axis=-1, epsilon=1e-5):
    """RMSNormalization of x (float32, or uint16 bits of dt) with the scale
    broadcast against the normalized axes; returns the output in x's storage."""
    xf, sf = _up(x, dt), _up(scale, dt)
    if axis < 0:
        axis += xf.ndim
    norm_shape = xf.shape[axis:]
    outer = int(np.prod(xf.shape[:axis])) if axis else 1
    norm = int(np.prod(norm_shape)) if norm_shape else 1
    s_full = np.ascontiguousarray(np.broadcast_to(sf, norm_shape), np.float32).ravel()
    y = np.empty(xf.size, np.float32)
    lib().orc_rms_norm_f32(_ptr(np.ascontiguousarray(xf).ravel()), _ptr(s_full), outer, norm,
                           C.c_float(epsilon), int(dt if dt != FLOAT else 0), _ptr(y))
    return _down(y.reshape(xf.shape), dt)


def rotary_embedding(x, cos, sin, dt=FLOAT, position_ids=None, interleaved=False,
                     rotary_embedding_dim=0, num_heads=0):
    xf, cf, sf = _up(x, dt), _up(cos, dt), _up(sin, dt)
    rank3 = xf.ndim == 3
    if rank3:
        B, S, hid = xf.shape
        H, D = num_heads, hid // num_heads
    else:
        B, H, S, D = xf.shape
    rot = rotary_embedding_dim or D
    pos = None if position_ids is None else np.ascontiguousarray(position_ids, np.int64)
    y = np.empty_like(np.ascontiguousarray(xf))
    rc = lib().orc_rotary_f32(_ptr(np.ascontiguousarray(xf)), _ptr(np.ascontiguousarray(cf)),
                              _ptr(np.ascontiguousarray(sf)), _ptr(pos), B, H, S, D, rot // 2,
                              int(rank3), int(bool(interleaved)),
                              cf.shape[0] if pos is not None else 0, _ptr(y))
    _check(rc, "RotaryEmbedding")
    return _down(y, dt)


def swiglu(a, b, dt=FLOAT, alpha=1.0):
    af, bf = _up(a, dt), _up(b, dt)
    y = np.empty(af.size, np.float32)
    lib().orc_swiglu_f32(_ptr(np.ascontiguousarray(af).ravel()), _ptr(np.ascontiguousarray(bf).ravel()),
                         af.size, C.c_float(alpha), _ptr(y))
    return _down(y.reshape(af.shape), dt)


# ---------------------------------------------------------------------------
# onnx-light's own kernels (oracle/_ref)
# ---------------------------------------------------------------------------

class ReferenceError_(ValueError):
    pass


def _ref_call(fn, *args):
    err = C.create_string_buffer(1024)
    rc = fn(*args, err, C.c_size_t(1024))
    if rc != 0:
        raise ReferenceError_(err.value.decode(errors="replace"))


def ref_dequantize_linear(x_raw, x_dt, x_shape, scale_raw, s_dt, s_shape, zp_raw=None,
                          zp_shape=None, axis=1):
    n = int(np.prod(x_shape)) if len(x_shape) else 1
    out = np.empty(n, np.float32 if s_dt == FLOAT else np.uint16)
    xs, xn = _shape(x_shape)
    ss, sn = _shape(s_shape)
    zs, zn = _shape(zp_shape if zp_shape is not None else [])
    x_raw = np.ascontiguousarray(x_raw, np.uint8)
    scale_raw = np.ascontiguousarray(scale_raw).view(np.uint8)
    zp = None if zp_raw is None else np.ascontiguousarray(zp_raw, np.uint8)
    _ref_call(ref().ref_dequantize_linear, _ptr(x_raw), x_dt, xs, xn, _ptr(scale_raw), s_dt, ss,
              sn, _ptr(zp), zs, zn, C.c_int64(axis), _ptr(out), C.c_size_t(out.nbytes))
    return out.reshape(tuple(x_shape))


def ref_matmul(a, b, dt):
    shape = matmul_shape(a.shape, b.shape)
    out = np.empty(shape, np.float32 if dt == FLOAT else np.uint16)
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b)
    asz, an = _shape(a.shape)
    bsz, bn = _shape(b.shape)
    ys = (C.c_int64 * 16)()
    yn = C.c_int()
    _ref_call(ref().ref_matmul, _ptr(a), asz, an, _ptr(b), bsz, bn, dt, _ptr(out),
              C.c_size_t(out.nbytes), ys, C.byref(yn))
    return out


def ref_matmul_integer(a, a_dt, b, b_dt, a_zp=None, b_zp=None, a_zp_shape=None, b_zp_shape=None):
    shape = matmul_shape(a.shape, b.shape)
    out = np.empty(shape, np.int32)
    a = np.ascontiguousarray(a).view(np.uint8)
    b = np.ascontiguousarray(b).view(np.uint8)
    asz, an = _shape(a.shape)
    bsz, bn = _shape(b.shape)
    az = None if a_zp is None else np.ascontiguousarray(a_zp).view(np.uint8)
    bz = None if b_zp is None else np.ascontiguousarray(b_zp).view(np.uint8)
    azs, azn = _shape(a_zp_shape if a_zp_shape is not None else ([] if az is None else az.shape))
    bzs, bzn = _shape(b_zp_shape if b_zp_shape is not None else ([] if bz is None else bz.shape))
    ys = (C.c_int64 * 16)()
    yn = C.c_int()
    _ref_call(ref().ref_matmul_integer, _ptr(a), a_dt, asz, an, _ptr(b), b_dt, bsz, bn, _ptr(az),
              azs, azn, _ptr(bz), bzs, bzn, _ptr(out), C.c_size_t(out.nbytes), ys, C.byref(yn))
    return out


def ref_qlinear_matmul(a, a_dt, a_scale, a_zp, b, b_dt, b_scale, b_zp, y_scale, y_zp, y_dt,
                       scale_dt=FLOAT):
    """Scales are python floats; with scale_dt=FLOAT16 they are first rounded to fp16 bits."""
    shape = matmul_shape(a.shape, b.shape)
    out = np.empty(shape, np.uint8)
    a = np.ascontiguousarray(a).view(np.uint8)
    b = np.ascontiguousarray(b).view(np.uint8)
    asz, an = _shape(a.shape)
    bsz, bn = _shape(b.shape)

    def sc(x):
        return (np.array([x], np.float32) if scale_dt == FLOAT
                else f32_to_f16_bits(np.array([x], np.float32)))

    def zp(x, dt):
        return np.array([x], np.int8 if dt == INT8 else np.uint8)

    sa, sb, sy = sc(a_scale), sc(b_scale), sc(y_scale)
    za, zb, zy = zp(a_zp, a_dt), zp(b_zp, b_dt), zp(y_zp, y_dt)
    ys = (C.c_int64 * 16)()
    yn = C.c_int()
    _ref_call(ref().ref_qlinear_matmul, _ptr(a), a_dt, asz, an, _ptr(sa), _ptr(za), _ptr(b), b_dt,
              bsz, bn, _ptr(sb), _ptr(zb), _ptr(sy), _ptr(zy), y_dt, scale_dt, _ptr(out),
              C.c_size_t(out.nbytes), ys, C.byref(yn))
    return out.view(np.int8) if y_dt == INT8 else out


def ref_attention(q, k, v, dt=FLOAT, scale=None, is_causal=False, softcap=0.0, mask=None,
                  past_k=None, past_v=None, q_num_heads=0, kv_num_heads=0, mask_dt=None,
                  nonpad=None, left_window=-1, right_window=-1, qk_mode=None):
    """q,k,v: float32 (dt=FLOAT) or uint16 bit patterns (FLOAT16/BFLOAT16), rank 3 or 4.

    mask: float32 (mask_dt FLOAT, the default), numpy bool (BOOL) or uint16
    bits with mask_dt FLOAT16 / BFLOAT16.  Returns (Y, present_key,
    present_value), plus qk_matmul_output when qk_mode is given, in the
    storage type of dt."""
    rank = q.ndim
    q = np.ascontiguousarray(q)
    k = np.ascontiguousarray(k)
    v = np.ascontiguousarray(v)
    qs, _ = _shape(q.shape)
    ks, _ = _shape(k.shape)
    vs, _ = _shape(v.shape)
    store = np.float32 if dt == FLOAT else np.uint16
    if rank == 4:
        ysh = (q.shape[0], q.shape[1], q.shape[2], v.shape[3])
        sq, hq = q.shape[2], q.shape[1]
        snew = k.shape[2]
    else:
        ysh = (q.shape[0], q.shape[1], q_num_heads * (v.shape[2] // kv_num_heads))
        sq, hq = q.shape[1], q_num_heads
        snew = k.shape[1]
    y = np.empty(ysh, store)
    m = None
    ms, mn = _shape([])
    mdt = FLOAT
    if mask is not None:
        m = np.ascontiguousarray(mask)
        if m.dtype == np.bool_:
            m, mdt = m.astype(np.uint8), BOOL
        elif mask_dt in (FLOAT16, BFLOAT16):
            m, mdt = m.astype(np.uint16), mask_dt
        else:
            m = m.astype(np.float32)
        ms, mn = _shape(m.shape)
    pk = pv = None
    ps, _ = _shape([])
    pvs, _ = _shape([])
    present_k = present_v = None
    past = 0
    if past_k is not None:
        pk = np.ascontiguousarray(past_k)
        pv = np.ascontiguousarray(past_v)
        ps, _ = _shape(pk.shape)
        pvs, _ = _shape(pv.shape)
        past = pk.shape[2]
        L = past + snew
        present_k = np.empty((pk.shape[0], pk.shape[1], L, pk.shape[3]), store)
        present_v = np.empty((pv.shape[0], pv.shape[1], L, pv.shape[3]), store)
    npd = None if nonpad is None else np.ascontiguousarray(nonpad, np.int64)
    qk = None
    if qk_mode is not None:
        qk = np.zeros((q.shape[0], hq, sq, past + snew), store)
    _ref_call(ref().ref_attention, _ptr(q), qs, _ptr(k), ks, _ptr(v), vs, rank, dt, _ptr(m),
              int(mdt), ms, mn, _ptr(pk), _ptr(pv), ps, pvs, _ptr(npd),
              C.c_int64(0 if npd is None else npd.size), int(scale is not None),
              C.c_float(0.0 if scale is None else scale), int(is_causal), C.c_float(softcap),
              C.c_int64(q_num_heads), C.c_int64(kv_num_heads), C.c_int64(left_window),
              C.c_int64(right_window), int(qk_mode or 0), _ptr(y), C.c_size_t(y.nbytes),
              _ptr(present_k), _ptr(present_v),
              C.c_size_t(0 if present_k is None else present_k.nbytes),
              C.c_size_t(0 if present_v is None else present_v.nbytes), _ptr(qk),
              C.c_size_t(0 if qk is None else qk.nbytes))
    if qk_mode is not None:
        return y, present_k, present_v, qk
    return y, present_k, present_v


def ref_rms_normalization(x, scale, dt=FLOAT, axis=-1, epsilon=1e-5):
    x, scale = np.ascontiguousarray(x), np.ascontiguousarray(scale)
    xs, xn = _shape(x.shape)
    ss, sn = _shape(scale.shape)
    y = np.empty_like(x)
    _ref_call(ref().ref_rms_normalization, _ptr(x), xs, xn, dt, _ptr(scale), ss, sn,
              C.c_int64(axis), C.c_float(epsilon), _ptr(y), C.c_size_t(y.nbytes))
    return y


def ref_rotary_embedding(x, cos, sin, dt=FLOAT, position_ids=None, interleaved=False,
                         rotary_embedding_dim=0, num_heads=0):
    x, cos, sin = np.ascontiguousarray(x), np.ascontiguousarray(cos), np.ascontiguousarray(sin)
    xs, xn = _shape(x.shape)
    cs, cn = _shape(cos.shape)
    pos = None if position_ids is None else np.ascontiguousarray(position_ids, np.int64)
    ps, pn = _shape([] if pos is None else pos.shape)
    y = np.empty_like(x)
    _ref_call(ref().ref_rotary_embedding, _ptr(x), xs, xn, dt, _ptr(cos), _ptr(sin), cs, cn,
              _ptr(pos), ps, pn, int(bool(interleaved)), C.c_int64(rotary_embedding_dim),
              C.c_int64(num_heads), _ptr(y), C.c_size_t(y.nbytes))
    return y


def ref_swiglu(a, b, dt=FLOAT, alpha=1.0):
    a, b = np.ascontiguousarray(a), np.ascontiguousarray(b)
    sh, nd = _shape(a.shape)
    y = np.empty_like(a)
    _ref_call(ref().ref_swiglu, _ptr(a), _ptr(b), sh, nd, dt, C.c_float(alpha), _ptr(y),
              C.c_size_t(y.nbytes))
    return y


def ref_thread_count() -> int:
    return int(ref().ref_thread_count())
