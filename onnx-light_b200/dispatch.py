"""Device-keyed kernel registration, mirroring onnx-light's dispatch table.

onnx-light resolves a node to a kernel through a process-wide table keyed
``"<domain>:<op_type>"`` plus ``":<device-int>"`` for any device other than
the CPU (onnx_light/onnx_core/runtime/kernels/kernel_dispatch_table.cc:45-58,
onnx_light/onnx_core/symbolic/sym_tensor.cc:107-112).  ``RegisterKernelFn``
stores a factory, replacing an existing one unless ``overwrite`` is false, in
which case the existing entry wins and the call returns False (:97-109).

``RegisterB200KernelFunctions`` is the GPU counterpart of
``onnx_kernels::RegisterKernelFunctions``
(onnx_light/onnx_extensions/kernels/kernel_dispatch_table.cc:374-488): it
registers the B200 kernels for ``Device::kGPU0 + i`` with overwrite=False, so an
override installed earlier by another library keeps precedence.

This module is the registry of the Python host API (a Python program that
drives the kernels by name) and of the CPU tests of the resolution rules.
onnx-light sessions do not read it: they resolve through the compiled
registration of onnx-light_b200/binding (``onnxl_b200::binding::
RegisterB200KernelFunctions``, KernelBase subclasses over the C ABI), which
registers the same operators under the same keys.
"""
from __future__ import annotations

from typing import Callable, Dict, Optional

from .kernels import (Attention, DequantizeLinear, DequantizeMatMul, MatMulInteger,
                      QLinearMatMul, RMSNormalization, RotaryEmbedding, SwiGLU)

K_DEFAULT_ONNX_DOMAIN = "ai.onnx"
DEVICE_CPU = -1
DEVICE_UNDEFINED = -2
DEVICE_GPU0 = 0
MAX_GPU_INDEX = 8191
FUSED_DOMAIN = "b200"  # custom domain of the fused DequantizeLinear -> MatMul node


def normalise_domain(domain: str) -> str:
    return K_DEFAULT_ONNX_DOMAIN if domain in ("", K_DEFAULT_ONNX_DOMAIN) else domain


def device_key_suffix(device: int) -> str:
    if device in (DEVICE_CPU, DEVICE_UNDEFINED):
        return ""
    return f":{int(device)}"


def dispatch_key(domain: str, op_type: str, device: int = DEVICE_CPU) -> str:
    return f"{normalise_domain(domain)}:{op_type}{device_key_suffix(device)}"


class KernelDispatchTable:
    def __init__(self):
        self._table: Dict[str, Callable] = {}

    def register(self, domain: str, op_type: str, device: int, factory: Callable,
                 overwrite: bool = True) -> bool:
        key = dispatch_key(domain, op_type, device)
        if not overwrite and key in self._table:
            return False
        self._table[key] = factory
        return True

    def resolve(self, domain: str, op_type: str, device: int) -> Callable:
        """Factory for the node, or ValueError naming the device (run_nodes.cc:1597-1600).

        No fallback to the CPU entry: a GPU session resolves GPU kernels only.
        """
        key = dispatch_key(domain, op_type, device)
        try:
            return self._table[key]
        except KeyError:
            raise ValueError(f"no kernel registered for {normalise_domain(domain)}:{op_type} "
                             f"on device {device}") from None

    def __contains__(self, key: str) -> bool:
        return key in self._table

    def keys(self):
        return self._table.keys()


_default: Optional[KernelDispatchTable] = None


def default_table() -> KernelDispatchTable:
    global _default
    if _default is None:
        _default = KernelDispatchTable()
    return _default


def RegisterB200KernelFunctions(table: Optional[KernelDispatchTable] = None,
                                num_gpus: int = 8) -> KernelDispatchTable:
    """Registers the B200 kernels for kGPU0 .. kGPU0+num_gpus-1 (overwrite=False)."""
    table = table or default_table()
    entries = {
        ("", "DequantizeLinear"): DequantizeLinear,
        ("", "MatMulInteger"): MatMulInteger,
        ("", "QLinearMatMul"): QLinearMatMul,
        ("", "Attention"): Attention,
        ("", "RMSNormalization"): RMSNormalization,
        ("", "RotaryEmbedding"): RotaryEmbedding,
        ("", "SwiGLU"): SwiGLU,
        (FUSED_DOMAIN, "DequantizeMatMul"): DequantizeMatMul,
    }
    for i in range(num_gpus):
        for (domain, op), cls in entries.items():
            table.register(domain, op, DEVICE_GPU0 + i, cls, overwrite=False)
    return table
