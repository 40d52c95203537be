"""Host-side mirror of onnx-light's kernel classes for the quantized-inference path.

Each class keeps the reference's name, call signature, argument meaning and
error behaviour (std::invalid_argument -> ValueError), and runs on the GPU
through the C ABI in include/onnxl_b200.h.  Inputs and outputs are CUDA
tensors; sub-byte and 8-bit float tensors travel as :class:`QTensor` (packed
uint8 storage + ONNX dtype + logical shape), exactly like onnx-light's Tensor
storage.  There is no CPU fallback: a missing library or a CPU tensor raises.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field
from typing import Optional

import torch

from . import _capi as capi
from ._capi import Desc, check, lib, stream_ptr


@dataclass
class QTensor:
    """Quantized tensor: packed storage bytes, ONNX dtype, logical shape."""

    data: torch.Tensor  # uint8 storage on the device (packed low-order-first)
    dtype: int
    shape: tuple

    @property
    def device(self):
        return self.data.device


def _desc(t, dtype: Optional[int] = None) -> Desc:
    if isinstance(t, QTensor):
        if not t.data.is_cuda:
            raise ValueError("onnxl_b200 tensors must live on a CUDA device")
        return Desc(t.data.data_ptr(), t.dtype, t.shape)
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"expected a torch.Tensor or QTensor, got {type(t).__name__}")
    if not t.is_cuda:
        raise ValueError("onnxl_b200 tensors must live on a CUDA device (no CPU fallback)")
    if not t.is_contiguous():
        raise ValueError("onnxl_b200 tensors must be contiguous")
    dt = dtype if dtype is not None else capi.TORCH_TO_ONNX[t.dtype]
    return Desc(t.data_ptr(), dt, tuple(t.shape))


def _ref(d: Optional[Desc]):
    return d.ref if d is not None else None


# ---------------------------------------------------------------------------
# Workspace: one zero-initialised buffer per (device, stream), grown on
# demand.  The kernels return their split-K counters to zero, so a buffer
# stays valid from call to call.  Keying by stream keeps the header's rule
# that calls sharing a workspace must not overlap on the GPU: calls on one
# stream are ordered, calls on two streams get two buffers.  A buffer is
# allocated with its stream current, so when a larger one replaces it, torch's
# caching allocator hands the old memory out again only to later work on that
# same stream, never while a kernel queued before the swap still reads it.
# ---------------------------------------------------------------------------

_workspaces: dict = {}


def workspace(device: torch.device, nbytes: int, stream=None) -> torch.Tensor:
    index = device.index if device.index is not None else torch.cuda.current_device()
    if stream is None:
        stream = torch.cuda.current_stream(index)
    key = (index, stream.cuda_stream)
    buf = _workspaces.get(key)
    if buf is None or buf.numel() < nbytes:
        with torch.cuda.stream(stream):
            buf = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _workspaces[key] = buf
    return buf


def _call_with_workspace(fn, args_before, args_after, device):
    """Queries the workspace size (workspace=NULL), then runs."""
    need = C.c_size_t(0)
    check(fn(*args_before, None, C.byref(need), *args_after))
    if need.value == 0:
        check(fn(*args_before, None, None, *args_after))
        return
    ws = workspace(device, need.value)
    cap = C.c_size_t(ws.numel())
    check(fn(*args_before, C.c_void_p(ws.data_ptr()), C.byref(cap), *args_after))


# ---------------------------------------------------------------------------
# Kernels
# ---------------------------------------------------------------------------


class DequantizeLinear:
    """kernel::DequantizeLinear (kernel_dequantizelinear.cc:332-712).

    ``y = (x - x_zero_point) * x_scale``; per-tensor, per-axis or blocked along
    ``axis`` (the block is x.shape[axis] / x_scale.shape[axis]); the output
    dtype is x_scale's (FLOAT or FLOAT16).  Bit-exact with the reference.
    """

    name = "onnx_kernels:GPU:ai.onnx:DequantizeLinear"

    def __call__(self, x, x_scale: torch.Tensor, x_zero_point=None, axis: int = 1,
                 out: Optional[torch.Tensor] = None) -> torch.Tensor:
        xd = _desc(x)
        sd = _desc(x_scale)
        zd = _desc(x_zero_point) if x_zero_point is not None else None
        shape = tuple(x.shape)
        if out is None:
            if x_scale.dtype not in (torch.float32, torch.float16):
                raise ValueError("kernel::DequantizeLinear: x_scale must be FLOAT or FLOAT16.")
            out = torch.empty(shape, dtype=x_scale.dtype, device=x_scale.device)
        yd = _desc(out)
        check(lib().b2_dequantize_linear(xd.ref, sd.ref, _ref(zd), int(axis), yd.ref,
                                         stream_ptr(out.device)))
        return out


class DequantizeMatMul:
    """The DequantizeLinear -> [Cast] -> MatMul weight-only pattern as one kernel.

    Equivalent to ``MatMul(a, Cast(DequantizeLinear(w, w_scale, w_zero_point, axis)))``
    with kernel::DequantizeLinear (kernel_dequantizelinear.cc:522-693) and
    kernel::MatMul (kernel_matmul.cc:181-223): the weight is dequantized with the
    reference's rounding and never written to HBM.
    """

    name = "onnx_kernels:GPU:b200:DequantizeMatMul"

    def __call__(self, a: torch.Tensor, w, w_scale: torch.Tensor, w_zero_point=None,
                 axis: int = 0, cast_dtype: Optional[torch.dtype] = None,
                 out: Optional[torch.Tensor] = None) -> torch.Tensor:
        ad, wd, sd = _desc(a), _desc(w), _desc(w_scale)
        zd = _desc(w_zero_point) if w_zero_point is not None else None
        cast = capi.TORCH_TO_ONNX[cast_dtype] if cast_dtype is not None else 0
        if out is None:
            n = int(w.shape[-1])
            out = torch.empty(tuple(a.shape[:-1]) + (n,), dtype=a.dtype, device=a.device)
        yd = _desc(out)
        _call_with_workspace(lib().b2_dequantize_matmul,
                             (ad.ref, wd.ref, sd.ref, _ref(zd), int(axis), cast, yd.ref),
                             (stream_ptr(a.device),), a.device)
        return out


class DequantizeMatMulGroup:
    """Several DequantizeLinear -> MatMul nodes on the same activations (q / k / v,
    gate / up) as one call: ``[a @ DequantizeLinear(w_i, s_i) for i]``.

    Each member is the two-node pattern of DequantizeMatMul (kernel_dequantizelinear.cc
    :522-693 then kernel_matmul.cc:181-223) with the same ``a`` and ``axis``, no zero
    point and no cast; members with one K, weight type and scale layout that the
    int4 / fp16 decode kernel takes run as one launch (b2_dequantize_matmul_group).
    """

    name = "onnx_kernels:GPU:b200:DequantizeMatMulGroup"

    def __call__(self, a: torch.Tensor, ws, scales, axis: int = 0, outs=None):
        if len(ws) != len(scales) or not 1 <= len(ws) <= 4:
            raise ValueError("DequantizeMatMulGroup: 1 to 4 weights, one scale each")
        if outs is None:
            outs = [torch.empty(tuple(a.shape[:-1]) + (int(w.shape[-1]),), dtype=a.dtype,
                                device=a.device) for w in ws]
        ad = _desc(a)
        wd = capi.DescArray([_desc(w) for w in ws])
        sd = capi.DescArray([_desc(s) for s in scales])
        yd = capi.DescArray([_desc(y) for y in outs])
        _call_with_workspace(lib().b2_dequantize_matmul_group,
                             (len(ws), ad.ref, wd.ref, sd.ref, int(axis), yd.ref),
                             (stream_ptr(a.device),), a.device)
        return outs


def _matmul_shape(a_shape, b_shape):
    a2 = list(a_shape) if len(a_shape) > 1 else [1, a_shape[0]]
    b2 = list(b_shape) if len(b_shape) > 1 else [b_shape[0], 1]
    ap, bp = a2[:-2], b2[:-2]
    r = max(len(ap), len(bp))
    ap = [1] * (r - len(ap)) + ap
    bp = [1] * (r - len(bp)) + bp
    out = [max(x, y) if 1 in (x, y) else x for x, y in zip(ap, bp)]
    if len(a_shape) != 1:
        out.append(a2[-2])
    if len(b_shape) != 1:
        out.append(b2[-1])
    return tuple(out)


class MatMulInteger:
    """kernel::MatMulInteger (kernel_matmul_integer.cc:178-250): int32 output, bit-exact."""

    name = "onnx_kernels:GPU:ai.onnx:MatMulInteger"

    def __call__(self, a: torch.Tensor, b: torch.Tensor, a_zero_point=None, b_zero_point=None,
                 out: Optional[torch.Tensor] = None) -> torch.Tensor:
        ad, bd = _desc(a), _desc(b)
        azd = _desc(a_zero_point) if a_zero_point is not None else None
        bzd = _desc(b_zero_point) if b_zero_point is not None else None
        if out is None:
            out = torch.empty(_matmul_shape(a.shape, b.shape), dtype=torch.int32, device=a.device)
        yd = _desc(out)
        _call_with_workspace(lib().b2_matmul_integer, (ad.ref, bd.ref, _ref(azd), _ref(bzd), yd.ref),
                             (stream_ptr(a.device),), a.device)
        return out


class QLinearMatMul:
    """kernel::QLinearMatMul (kernel_qlinearmatmul.cc:221-284): int8/uint8 output, bit-exact."""

    name = "onnx_kernels:GPU:ai.onnx:QLinearMatMul"

    def __call__(self, a, a_scale, a_zero_point, b, b_scale, b_zero_point, y_scale, y_zero_point,
                 out: Optional[torch.Tensor] = None) -> torch.Tensor:
        ds = [_desc(t) for t in (a, a_scale, a_zero_point, b, b_scale, b_zero_point, y_scale,
                                 y_zero_point)]
        if out is None:
            out = torch.empty(_matmul_shape(a.shape, b.shape), dtype=y_zero_point.dtype,
                              device=a.device)
        yd = _desc(out)
        _call_with_workspace(lib().b2_qlinear_matmul, tuple(d.ref for d in ds) + (yd.ref,),
                             (stream_ptr(a.device),), a.device)
        return out


@dataclass
class Attributes:
    """kernel::Attention::Attributes (include_nn_kernels.h:1027-1040)."""

    has_scale: bool = False
    scale: float = 0.0
    is_causal: bool = False
    softcap: float = 0.0
    qk_matmul_output_mode: int = 0
    q_num_heads: int = 0
    kv_num_heads: int = 0
    left_window_size: int = -1
    right_window_size: int = -1


@dataclass
class Result:
    Y: torch.Tensor
    present_key: Optional[torch.Tensor] = None
    present_value: Optional[torch.Tensor] = None
    qk_matmul_output: Optional[torch.Tensor] = None


class KVCache:
    """Contiguous, capacity-reserved KV cache [B, Hkv, capacity, D] per K and V.

    The device counterpart of onnx-light's persistent KV storage
    (RuntimeSessionOptions::persistent_tensor_initial_capacity,
    runtime_context.h:763-768): past and present share one buffer and each
    Attention call appends its new tokens in place.
    """

    def __init__(self, batch: int, kv_heads: int, capacity: int, head_size: int,
                 dtype=torch.float16, device="cuda"):
        self.k = torch.zeros((batch, kv_heads, capacity, head_size), dtype=dtype, device=device)
        self.v = torch.zeros_like(self.k)
        self.capacity = capacity
        self.length = 0

    def view(self, length: int):
        """past/present views: the buffer with a logical sequence length."""
        return self.k, self.v, length


class Attention:
    """kernel::Attention, opset 23 (kernel_attention.cc:767-902), GQA + contiguous KV cache.

    ``attn_mask`` may be FLOAT or BOOL (or FLOAT16 / BFLOAT16 with half
    inputs); ``nonpad_kv_seqlen`` is an INT64 [B] tensor; with
    ``qk_matmul_output=True`` the result also carries the [B, Hq, Sq, L]
    scores selected by ``attrs.qk_matmul_output_mode``.
    """

    name = "onnx_kernels:GPU:ai.onnx:Attention"

    def __call__(self, Q, K, V, attrs: Optional[Attributes] = None, attn_mask=None,
                 past_key=None, past_value=None, nonpad_kv_seqlen=None,
                 cache: Optional[KVCache] = None, present_key=None, present_value=None,
                 qk_matmul_output: bool = False, out=None) -> Result:
        attrs = attrs or Attributes()
        a = capi.B2AttentionAttrs(int(attrs.has_scale), float(attrs.scale), int(attrs.is_causal),
                                  float(attrs.softcap), int(attrs.qk_matmul_output_mode),
                                  int(attrs.q_num_heads), int(attrs.kv_num_heads),
                                  int(attrs.left_window_size), int(attrs.right_window_size), 0)
        qd, kd, vd = _desc(Q), _desc(K), _desc(V)
        md = _desc(attn_mask) if attn_mask is not None else None
        nd = _desc(nonpad_kv_seqlen) if nonpad_kv_seqlen is not None else None
        rank3 = Q.dim() == 3
        new = K.shape[1] if rank3 else K.shape[2]
        B = Q.shape[0]
        if rank3:
            hkv = attrs.kv_num_heads
            D = K.shape[2] // hkv if hkv > 0 else 0
            Dv = V.shape[2] // hkv if hkv > 0 else 0
        else:
            hkv, D, Dv = K.shape[1], K.shape[3], V.shape[3]
        Hq = attrs.q_num_heads if rank3 else Q.shape[1]
        Sq = Q.shape[1] if rank3 else Q.shape[2]
        pkd = pvd = None
        if cache is not None:
            past = cache.length
            a.kv_capacity = cache.capacity
            if past:
                pkd = Desc(cache.k.data_ptr(), capi.TORCH_TO_ONNX[cache.k.dtype], (B, hkv, past, D))
                pvd = Desc(cache.v.data_ptr(), capi.TORCH_TO_ONNX[cache.v.dtype], (B, hkv, past, Dv))
            total = past + new
            prk = Desc(cache.k.data_ptr(), capi.TORCH_TO_ONNX[cache.k.dtype], (B, hkv, total, D))
            prv = Desc(cache.v.data_ptr(), capi.TORCH_TO_ONNX[cache.v.dtype], (B, hkv, total, Dv))
        else:
            if past_key is not None:
                pkd, pvd = _desc(past_key), _desc(past_value)
                total = past_key.shape[2] + new
            else:
                total = new
            if present_key is None and (past_key is not None):
                present_key = torch.empty((B, hkv, total, D), dtype=Q.dtype, device=Q.device)
                present_value = torch.empty((B, hkv, total, Dv), dtype=Q.dtype, device=Q.device)
            prk = _desc(present_key) if present_key is not None else None
            prv = _desc(present_value) if present_value is not None else None
        if out is None:
            shape = (B, Sq, Hq * Dv) if rank3 else (B, Hq, Sq, Dv)
            out = torch.empty(shape, dtype=Q.dtype, device=Q.device)
        yd = _desc(out)
        qk = None
        if qk_matmul_output:
            qk = torch.empty((B, Hq, Sq, total), dtype=Q.dtype, device=Q.device)
        qkd = _desc(qk) if qk is not None else None
        _call_with_workspace(lib().b2_attention_ex,
                             (qd.ref, kd.ref, vd.ref, _ref(md), _ref(pkd), _ref(pvd), _ref(nd),
                              C.byref(a), yd.ref, _ref(prk), _ref(prv), _ref(qkd)),
                             (stream_ptr(Q.device),), Q.device)
        if cache is not None:
            cache.length = total
            return Result(out, cache.k[:, :, :total], cache.v[:, :, :total], qk)
        return Result(out, present_key, present_value, qk)


class RMSNormalization:
    """kernel::RMSNormalization, opset 23 (kernel_rmsnormalization.cc:83-228)."""

    name = "onnx_kernels:GPU:ai.onnx:RMSNormalization"

    def __call__(self, x: torch.Tensor, scale: torch.Tensor, axis: int = -1,
                 epsilon: float = 1e-5, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        if out is None:
            out = torch.empty_like(x)
        xd, sd, yd = _desc(x), _desc(scale), _desc(out)
        check(lib().b2_rms_normalization(xd.ref, sd.ref, int(axis), float(epsilon), yd.ref,
                                         stream_ptr(x.device)))
        return out


class RotaryEmbedding:
    """kernel::RotaryEmbedding, opset 23 (kernel_rotary_embedding.cc:47-242)."""

    name = "onnx_kernels:GPU:ai.onnx:RotaryEmbedding"

    def __call__(self, x: torch.Tensor, cos_cache: torch.Tensor, sin_cache: torch.Tensor,
                 position_ids: Optional[torch.Tensor] = None, interleaved: bool = False,
                 rotary_embedding_dim: int = 0, num_heads: int = 0,
                 out: Optional[torch.Tensor] = None) -> torch.Tensor:
        if out is None:
            out = torch.empty_like(x)
        xd, cd, sd, yd = _desc(x), _desc(cos_cache), _desc(sin_cache), _desc(out)
        pd = _desc(position_ids) if position_ids is not None else None
        check(lib().b2_rotary_embedding(xd.ref, cd.ref, sd.ref, _ref(pd), int(bool(interleaved)),
                                        int(rotary_embedding_dim), int(num_heads), yd.ref,
                                        stream_ptr(x.device)))
        return out


class SwiGLU:
    """kernel::SwiGLU (kernel_swiglu.cc:58-129): a * sigmoid(alpha a) * b."""

    name = "onnx_kernels:GPU:ai.onnx:SwiGLU"

    def __call__(self, a: torch.Tensor, b: torch.Tensor, alpha: float = 1.0,
                 out: Optional[torch.Tensor] = None) -> torch.Tensor:
        if out is None:
            out = torch.empty_like(a)
        ad, bd, yd = _desc(a), _desc(b), _desc(out)
        check(lib().b2_swiglu(ad.ref, bd.ref, float(alpha), yd.ref, stream_ptr(a.device)))
        return out
