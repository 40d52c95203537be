"""ctypes binding of the onnxl_b200 C ABI (include/onnxl_b200.h).

This is the Python analogue of the binding an onnx-light maintainer adds on
the C++ side (a KernelBase subclass calling the same entry points): tensors
are described by (device pointer, ONNX dtype, shape), calls are stream-ordered
on torch's current stream, and a negative status is raised as the exception
the reference kernel would throw (std::invalid_argument -> ValueError).
"""
from __future__ import annotations

import ctypes as C
import os
import threading

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libonnxl_b200.so")

# ONNX TensorProto.DataType codes.
FLOAT, UINT8, INT8, UINT16, INT16, INT32, INT64, BOOL = 1, 2, 3, 4, 5, 6, 7, 9
FLOAT16, DOUBLE, BFLOAT16 = 10, 11, 16
FLOAT8E4M3FN, FLOAT8E4M3FNUZ, FLOAT8E5M2, FLOAT8E5M2FNUZ = 17, 18, 19, 20
UINT4, INT4, FLOAT4E2M1, FLOAT8E8M0, UINT2, INT2, FLOAT6E2M3, FLOAT6E3M2 = 21, 22, 23, 24, 25, 26, 27, 28

B2_OK = 0
B2_ERR_INVALID_ARGUMENT = -1
B2_ERR_UNSUPPORTED_DTYPE = -2
B2_ERR_CUDA = -3
B2_ERR_WORKSPACE = -4
B2_ERR_TIMEOUT = -5
B2_ERR_UNSUPPORTED = -6

TORCH_TO_ONNX = {
    torch.float32: FLOAT, torch.float16: FLOAT16, torch.bfloat16: BFLOAT16, torch.uint8: UINT8,
    torch.int8: INT8, torch.int16: INT16, torch.int32: INT32, torch.int64: INT64,
    torch.uint16: UINT16, torch.bool: BOOL, torch.float64: DOUBLE,
}
ONNX_TO_TORCH = {FLOAT: torch.float32, FLOAT16: torch.float16, BFLOAT16: torch.bfloat16,
                 UINT8: torch.uint8, INT8: torch.int8, INT16: torch.int16, INT32: torch.int32,
                 INT64: torch.int64, UINT16: torch.uint16}

# Every symbol the header declares (checked by the CPU tests).
EXPORTS = ("b2_version", "b2_last_error", "b2_dequantize_linear", "b2_dequantize_matmul",
           "b2_dequantize_matmul_noalloc", "b2_matmul_integer", "b2_qlinear_matmul", "b2_attention", "b2_attention_ex", "b2_synth_fill",
           "b2_convert", "b2_kernel_status", "b2_selftest_bounded_wait", "b2_selftest_gemm_timeout",
           "b2_rms_normalization", "b2_rotary_embedding", "b2_swiglu", "b2_ipc_alloc",
           "b2_ipc_free", "b2_ipc_open", "b2_ipc_close", "b2_allgather_cols",
           "b2_dequantize_matmul_peer", "b2_peer_wait", "b2_dequantize_matmul_group",
           "b2_dequantize_matmul_group_peer")


class B2Tensor(C.Structure):
    _fields_ = [("data", C.c_void_p), ("dtype", C.c_int32), ("ndim", C.c_int32),
                ("shape", C.POINTER(C.c_int64))]


class B2PeerOut(C.Structure):
    """b2_peer_out: a column-sharded output over a multi-GPU group."""
    _fields_ = [("full", C.c_void_p * 8), ("flags", C.c_void_p * 8), ("counters", C.c_void_p),
                ("world", C.c_int32), ("rank", C.c_int32), ("n_full", C.c_int64),
                ("wait_input", C.c_int32)]


class B2AttentionAttrs(C.Structure):
    _fields_ = [("has_scale", C.c_int32), ("scale", C.c_float), ("is_causal", C.c_int32),
                ("softcap", C.c_float), ("qk_matmul_output_mode", C.c_int32),
                ("q_num_heads", C.c_int64), ("kv_num_heads", C.c_int64),
                ("left_window_size", C.c_int64), ("right_window_size", C.c_int64),
                ("kv_capacity", C.c_int64)]


class B2Error(RuntimeError):
    """A CUDA, workspace or timeout failure inside the library."""

    def __init__(self, status: int, message: str):
        super().__init__(f"[{status}] {message}")
        self.status = status


class UnsupportedOnGpu(B2Error):
    """Valid for the reference, not handled by the GPU path (no CPU fallback)."""


_lib = None
_lock = threading.Lock()


def lib() -> C.CDLL:
    """Loads libonnxl_b200.so; raises if the CUDA library has not been built."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise ImportError(
                        f"{LIB_PATH} is missing: build the CUDA library first "
                        "(python onnx-light_b200/build.py).  There is no CPU fallback.")
                L = C.CDLL(LIB_PATH)
                P = C.c_void_p
                T = C.POINTER(B2Tensor)
                SZ = C.POINTER(C.c_size_t)
                L.b2_version.restype = C.c_char_p
                L.b2_last_error.argtypes = [C.c_char_p, C.c_size_t]
                L.b2_dequantize_linear.argtypes = [T, T, T, C.c_int64, T, P]
                L.b2_dequantize_matmul.argtypes = [T, T, T, T, C.c_int64, C.c_int32, T, P, SZ, P]
                L.b2_matmul_integer.argtypes = [T, T, T, T, T, P, SZ, P]
                L.b2_qlinear_matmul.argtypes = [T] * 9 + [P, SZ, P]
                L.b2_attention.argtypes = [T, T, T, T, T, T, C.POINTER(B2AttentionAttrs), T, T, T,
                                           P, SZ, P]
                L.b2_attention_ex.argtypes = [T, T, T, T, T, T, T, C.POINTER(B2AttentionAttrs), T,
                                              T, T, T, P, SZ, P]
                L.b2_rms_normalization.argtypes = [T, T, C.c_int64, C.c_float, T, P]
                L.b2_rotary_embedding.argtypes = [T, T, T, T, C.c_int32, C.c_int64, C.c_int64, T, P]
                L.b2_swiglu.argtypes = [T, T, C.c_float, T, P]
                L.b2_ipc_alloc.argtypes = [C.c_size_t, C.POINTER(C.c_void_p), P]
                L.b2_ipc_free.argtypes = [P]
                L.b2_ipc_open.argtypes = [P, C.POINTER(C.c_void_p)]
                L.b2_ipc_close.argtypes = [P]
                L.b2_allgather_cols.argtypes = [T, C.POINTER(C.c_void_p), C.POINTER(C.c_void_p), P,
                                                C.c_int, C.c_int, C.c_int64, P]
                L.b2_dequantize_matmul_peer.argtypes = [T, T, T, T, C.c_int64, C.c_int32, T,
                                                        C.POINTER(B2PeerOut), P, SZ, P]
                L.b2_peer_wait.argtypes = [C.POINTER(B2PeerOut), P]
                L.b2_dequantize_matmul_group.argtypes = [C.c_int32, T, T, T, C.c_int64, T, P, SZ, P]
                L.b2_dequantize_matmul_group_peer.argtypes = [C.c_int32, T, T, T, C.c_int64, T,
                                                              C.POINTER(B2PeerOut), P, SZ, P]
                L.b2_synth_fill.argtypes = [C.c_int32, C.c_uint64, C.c_int64, C.c_double,
                                            C.c_double, P, P]
                L.b2_convert.argtypes = [P, C.c_int32, P, C.c_int32, C.c_int64, P]
                L.b2_kernel_status.argtypes = [C.c_int]
                L.b2_selftest_bounded_wait.argtypes = [C.c_int64, P]
                L.b2_selftest_gemm_timeout.argtypes = [T, T, T, T, P, C.c_size_t, C.c_int64, P]
                L.b2_dequantize_matmul_noalloc.argtypes = [T, T, T, T, C.c_int64, C.c_int32, T, P]
                _lib = L
    return _lib


def version() -> str:
    return lib().b2_version().decode()


def check(rc: int) -> None:
    if rc == B2_OK:
        return
    buf = C.create_string_buffer(1024)
    lib().b2_last_error(buf, 1024)
    msg = buf.value.decode(errors="replace")
    if rc in (B2_ERR_INVALID_ARGUMENT, B2_ERR_UNSUPPORTED_DTYPE):
        raise ValueError(msg)
    if rc == B2_ERR_UNSUPPORTED:
        raise UnsupportedOnGpu(rc, msg)
    raise B2Error(rc, msg)


class Desc:
    """Keeps a B2Tensor and its shape array alive for the duration of a call."""

    __slots__ = ("t", "_shape")

    def __init__(self, data_ptr: int, dtype: int, shape):
        shape = [int(d) for d in shape]
        self._shape = (C.c_int64 * max(1, len(shape)))(*shape)
        self.t = B2Tensor(C.c_void_p(data_ptr or None), dtype, len(shape), self._shape)

    @property
    def ref(self):
        return C.byref(self.t)


class DescArray:
    """A contiguous array of B2Tensor (one per member of a group call), kept
    alive with its shape arrays for the duration of the call."""

    __slots__ = ("arr", "_descs")

    def __init__(self, descs):
        self._descs = list(descs)
        self.arr = (B2Tensor * len(self._descs))(*[d.t for d in self._descs])

    @property
    def ref(self):
        return C.cast(self.arr, C.POINTER(B2Tensor))


def stream_ptr(device=None) -> C.c_void_p:
    return C.c_void_p(torch.cuda.current_stream(device).cuda_stream)
