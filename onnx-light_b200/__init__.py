"""onnxl_b200 — B200 (sm_100a) kernels for onnx-light's quantized-inference path.

Drop-in GPU implementations of onnx-light's DequantizeLinear, MatMulInteger,
QLinearMatMul, the fused DequantizeLinear -> MatMul weight-only pattern and
opset-23 Attention (GQA, contiguous KV cache), plus the decoder-layer operators
around them (RMSNormalization, RotaryEmbedding, SwiGLU), exposed through the C ABI in
include/onnxl_b200.h and mirrored here with the reference's class names.
"""
from ._capi import version  # noqa: F401
from .dispatch import (KernelDispatchTable, RegisterB200KernelFunctions,  # noqa: F401
                       default_table)
from .kernels import (Attention, Attributes, DequantizeLinear, DequantizeMatMul,  # noqa: F401
                      DequantizeMatMulGroup, KVCache, MatMulInteger, QLinearMatMul, QTensor, Result, RMSNormalization,
                      RotaryEmbedding, SwiGLU)
