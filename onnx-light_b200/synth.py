"""Seeded synthetic inputs generated on the device.

The same SplitMix64 streams as onnx-light's generators
(onnx_light/onnx_core/runtime/kernels/random.cc:38-176), evaluated on the GPU
by b2_synth_fill, so benchmark inputs of hundreds of MB never cross PCIe and
tests can generate identical bytes on the host with the oracle.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _capi as capi
from ._capi import check, lib, stream_ptr
from .kernels import QTensor


def _numel(shape) -> int:
    n = 1
    for d in shape:
        n *= int(d)
    return n


def uniform(seed: int, shape, lo: float, hi: float, device="cuda") -> torch.Tensor:
    """RandUniformInto<float>: lo + u * (hi - lo), float32."""
    out = torch.empty(tuple(shape), dtype=torch.float32, device=device)
    check(lib().b2_synth_fill(0, seed, out.numel(), lo, hi, C.c_void_p(out.data_ptr()),
                              stream_ptr(out.device)))
    return out


def randn(seed: int, shape, mean: float = 0.0, scale: float = 1.0, device="cuda") -> torch.Tensor:
    """RandNormalInto<float>: mean + (sum of 12 uniforms - 6) * scale, float32."""
    out = torch.empty(tuple(shape), dtype=torch.float32, device=device)
    check(lib().b2_synth_fill(1, seed, out.numel(), mean, scale, C.c_void_p(out.data_ptr()),
                              stream_ptr(out.device)))
    return out


def randint(seed: int, shape, lo: int, hi_inclusive: int, device="cuda") -> torch.Tensor:
    """RandInt(lo, hi + 1) as int64."""
    out = torch.empty(tuple(shape), dtype=torch.int64, device=device)
    check(lib().b2_synth_fill(2, seed, out.numel(), float(lo), float(hi_inclusive),
                              C.c_void_p(out.data_ptr()), stream_ptr(out.device)))
    return out


def convert(src: torch.Tensor, onnx_dtype: int, shape=None) -> "torch.Tensor | QTensor":
    """FLOAT -> FLOAT16/BFLOAT16/FLOAT8E4M3FN, INT64 -> packed integer codes."""
    n = src.numel()
    shape = tuple(src.shape) if shape is None else tuple(shape)
    src_dt = capi.TORCH_TO_ONNX[src.dtype]
    if onnx_dtype in (capi.FLOAT16, capi.BFLOAT16):
        out = torch.empty(shape, dtype=capi.ONNX_TO_TORCH[onnx_dtype], device=src.device)
    elif onnx_dtype in (capi.INT8, capi.UINT8):
        out = torch.empty(shape, dtype=capi.ONNX_TO_TORCH[onnx_dtype], device=src.device)
    else:
        per = {capi.INT4: 2, capi.UINT4: 2, capi.FLOAT4E2M1: 2, capi.INT2: 4, capi.UINT2: 4,
               capi.FLOAT8E4M3FN: 1}[onnx_dtype]
        out = torch.empty(((n + per - 1) // per,), dtype=torch.uint8, device=src.device)
    check(lib().b2_convert(C.c_void_p(src.data_ptr()), src_dt, C.c_void_p(out.data_ptr()),
                           onnx_dtype, n, stream_ptr(src.device)))
    if out.dtype == torch.uint8 and onnx_dtype not in (capi.UINT8,):
        return QTensor(out, onnx_dtype, shape)
    return out


def packed_randint(seed: int, shape, lo: int, hi: int, onnx_dtype: int, device="cuda") -> QTensor:
    """Uniform integer codes in [lo, hi], packed as INT4/UINT4/INT2/UINT2/FLOAT4E2M1."""
    codes = randint(seed, (_numel(shape),), lo, hi, device)
    return convert(codes, onnx_dtype, shape)
