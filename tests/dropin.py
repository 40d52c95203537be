"""ctypes access to oracle/_ref/libref_harness.so: one ONNX node run through
onnx-light's own RunNode on a GPU device, resolved to the drop-in kernels of
onnx-light_b200/binding (test infrastructure)."""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
HARNESS = os.path.join(os.path.dirname(HERE), "oracle", "_ref", "libref_harness.so")


class T(C.Structure):
    _fields_ = [("data", C.c_void_p), ("dtype", C.c_int32), ("ndim", C.c_int32),
                ("shape", C.POINTER(C.c_int64))]


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(HARNESS):
            raise FileNotFoundError(f"{HARNESS} is not built (make -C oracle runtime)")
        L = C.CDLL(HARNESS)
        P = C.c_void_p
        L.h_register.argtypes = [C.c_int]
        L.h_dispatch_key.argtypes = [C.c_char_p, C.c_char_p, C.c_int, C.c_char_p, C.c_size_t]
        L.h_run_node.argtypes = [C.c_char_p, C.c_char_p, C.c_int, C.c_int, C.POINTER(T), C.c_int, P,
                                 P, P, P, C.c_int, C.POINTER(T), P, P, C.c_char_p, C.c_size_t]
        _lib = L
    return _lib


class NodeError(RuntimeError):
    pass


def run_node(domain, op_type, inputs, n_out, attrs=None, device=0, out_bytes=None):
    """inputs: list of (data_ptr, onnx_dtype, shape) or None (omitted input);
    attrs: {name: int | float}; out_bytes: capacity of each output buffer,
    list of (torch uint8 device tensors).  Returns [(dtype, shape)] per output."""
    import torch
    keep = []
    ins = (T * max(1, len(inputs)))()
    for i, x in enumerate(inputs):
        if x is None:
            ins[i] = T(None, 0, -1, None)
            continue
        ptr, dt, shape = x
        s = (C.c_int64 * max(1, len(shape)))(*[int(d) for d in shape])
        keep.append(s)
        ins[i] = T(C.c_void_p(ptr), dt, len(shape), s)
    attrs = attrs or {}
    names = (C.c_char_p * max(1, len(attrs)))(*[k.encode() for k in attrs])
    kinds = (C.c_int * max(1, len(attrs)))(*[0 if isinstance(v, (bool, int)) else 1
                                             for v in attrs.values()])
    ivals = (C.c_int64 * max(1, len(attrs)))(*[int(v) if isinstance(v, (bool, int)) else 0
                                               for v in attrs.values()])
    fvals = (C.c_float * max(1, len(attrs)))(*[float(v) for v in attrs.values()])
    outs = (T * max(1, n_out))()
    caps = (C.c_size_t * max(1, n_out))()
    bufs = []
    for i in range(n_out):
        if out_bytes[i] is None:
            outs[i] = T(None, 0, 0, None)
            bufs.append(None)
            continue
        b = torch.empty(max(1, out_bytes[i]), dtype=torch.uint8, device="cuda")
        bufs.append(b)
        outs[i] = T(C.c_void_p(b.data_ptr()), 0, 0, None)
        caps[i] = b.numel()
    shapes = (C.c_int64 * (8 * max(1, n_out)))()
    err = C.create_string_buffer(2048)
    rc = lib().h_run_node(domain.encode(), op_type.encode(), device, len(inputs), ins, len(attrs),
                          C.cast(names, C.c_void_p), C.cast(kinds, C.c_void_p),
                          C.cast(ivals, C.c_void_p), C.cast(fvals, C.c_void_p), n_out, outs,
                          C.cast(caps, C.c_void_p), C.cast(shapes, C.c_void_p), err, 2048)
    if rc != 0:
        raise NodeError(err.value.decode(errors="replace"))
    res = []
    for i in range(n_out):
        if bufs[i] is None:
            res.append(None)
            continue
        res.append((outs[i].dtype, tuple(shapes[8 * i + d] for d in range(outs[i].ndim)), bufs[i]))
    return res
