"""Host-side checks that need no GPU: the C-ABI library loads, exports every
entry point include/onnxl_b200.h declares, and the dispatch-table mirror keeps
onnx-light's registration rules."""
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_symbols():
    text = open(os.path.join(ROOT, "include", "onnxl_b200.h")).read()
    return sorted(set(re.findall(r"\b(b2_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol(b2):
    from onnx_light_b200 import _capi
    lib_path = _capi.LIB_PATH
    assert os.path.exists(lib_path), "build the library first (python onnx-light_b200/build.py)"
    out = subprocess.run(["nm", "-D", "--defined-only", lib_path], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\bT (b2_[a-z0-9_]+)", out))
    declared = header_symbols()
    assert declared, "no declarations parsed"
    missing = [s for s in declared if s not in exported]
    assert not missing, f"declared but not exported: {missing}"
    assert set(_capi.EXPORTS) <= set(declared)


def test_library_loads_without_gpu(b2):
    from onnx_light_b200 import _capi
    lib = _capi.lib()
    for s in header_symbols():
        assert hasattr(lib, s)
    assert _capi.version().startswith("onnxl_b200")


def test_null_tensor_is_invalid_argument(b2):
    from onnx_light_b200 import _capi
    rc = _capi.lib().b2_dequantize_linear(None, None, None, 0, None, None)
    assert rc == _capi.B2_ERR_INVALID_ARGUMENT


def test_dtype_validation_runs_on_host(b2):
    """Validation mirrors the reference and fails before touching the device."""
    from onnx_light_b200 import _capi
    x = _capi.Desc(0, _capi.UINT8, (3,))
    bad_scale = _capi.Desc(0, _capi.INT32, ())
    y = _capi.Desc(0, _capi.FLOAT, (3,))
    with pytest.raises(ValueError, match="x_scale must be FLOAT or FLOAT16"):
        _capi.check(_capi.lib().b2_dequantize_linear(x.ref, bad_scale.ref, None, 0, y.ref, None))
    fx = _capi.Desc(0, _capi.FLOAT, (3,))
    scale = _capi.Desc(0, _capi.FLOAT, ())
    with pytest.raises(ValueError, match="unsupported data type"):
        _capi.check(_capi.lib().b2_dequantize_linear(fx.ref, scale.ref, None, 0, y.ref, None))
    a = _capi.Desc(0, _capi.INT32, (2, 3))
    b = _capi.Desc(0, _capi.UINT8, (3, 2))
    yy = _capi.Desc(0, _capi.INT32, (2, 2))
    with pytest.raises(ValueError, match="A must be INT8 or UINT8"):
        _capi.check(_capi.lib().b2_matmul_integer(a.ref, b.ref, None, None, yy.ref, None, None, None))


def test_workspace_query_protocol(b2):
    """workspace == NULL returns the required size without launching anything."""
    import ctypes as C
    from onnx_light_b200 import _capi
    a = _capi.Desc(0, _capi.FLOAT16, (1, 4096))
    w = _capi.Desc(0, _capi.INT4, (4096, 4096))
    s = _capi.Desc(0, _capi.FLOAT16, (32, 4096))
    y = _capi.Desc(0, _capi.FLOAT16, (1, 4096))
    need = C.c_size_t(0)
    # Querying consults the device's SM count, which needs a GPU; on a CPU-only
    # host the library must fail cleanly rather than crash.
    rc = _capi.lib().b2_dequantize_matmul(a.ref, w.ref, s.ref, None, 0, 0, y.ref, None,
                                          C.byref(need), None)
    assert rc in (_capi.B2_OK, _capi.B2_ERR_CUDA)


def test_group_call_validates_on_host(b2):
    """The group entry points check the member count, the arrays and each
    member's types before touching the device."""
    from onnx_light_b200 import _capi
    lib = _capi.lib()
    a = _capi.Desc(0, _capi.FLOAT16, (1, 256))
    ws = _capi.DescArray([_capi.Desc(0, _capi.INT4, (256, 64)) for _ in range(2)])
    ss = _capi.DescArray([_capi.Desc(0, _capi.FLOAT16, (2, 64)) for _ in range(2)])
    ys = _capi.DescArray([_capi.Desc(0, _capi.FLOAT16, (1, 64)) for _ in range(2)])
    for count in (0, 5):
        assert lib.b2_dequantize_matmul_group(count, a.ref, ws.ref, ss.ref, 0, ys.ref, None, None,
                                              None) == _capi.B2_ERR_INVALID_ARGUMENT
    assert lib.b2_dequantize_matmul_group(2, a.ref, None, ss.ref, 0, ys.ref, None, None,
                                          None) == _capi.B2_ERR_INVALID_ARGUMENT
    # a member whose scale is not FLOAT / FLOAT16 fails like b2_dequantize_matmul
    bad = _capi.DescArray([_capi.Desc(0, _capi.FLOAT16, (2, 64)), _capi.Desc(0, _capi.INT32, (2, 64))])
    with pytest.raises(ValueError):
        _capi.check(lib.b2_dequantize_matmul_group(2, a.ref, ws.ref, bad.ref, 0, ys.ref, None, None,
                                                   None))
    assert lib.b2_dequantize_matmul_group_peer(2, a.ref, ws.ref, ss.ref, 0, ys.ref, None, None, None,
                                               None) == _capi.B2_ERR_INVALID_ARGUMENT


def test_dispatch_table_rules(b2):
    t = b2.KernelDispatchTable()
    from onnx_light_b200 import dispatch as d
    assert d.dispatch_key("", "Attention", d.DEVICE_CPU) == "ai.onnx:Attention"
    assert d.dispatch_key("ai.onnx", "Attention", d.DEVICE_GPU0 + 3) == "ai.onnx:Attention:3"
    # device is part of the identifier (test_dispatch_table_registration.cc:286)
    assert t.register("", "Attention", d.DEVICE_CPU, "cpu")
    assert t.register("", "Attention", d.DEVICE_GPU0, "gpu")
    assert t.resolve("", "Attention", d.DEVICE_CPU) == "cpu"
    assert t.resolve("", "Attention", d.DEVICE_GPU0) == "gpu"
    # overwrite=False keeps an existing entry (test_dispatch_table_registration.cc:307)
    assert not t.register("", "Attention", d.DEVICE_GPU0, "other", overwrite=False)
    assert t.resolve("", "Attention", d.DEVICE_GPU0) == "gpu"
    b2.RegisterB200KernelFunctions(t, num_gpus=8)
    assert t.resolve("", "Attention", d.DEVICE_GPU0) == "gpu"  # earlier override wins
    assert t.resolve("", "DequantizeLinear", d.DEVICE_GPU0 + 7) is b2.DequantizeLinear
    assert t.resolve("b200", "DequantizeMatMul", 2) is b2.DequantizeMatMul
    with pytest.raises(ValueError, match="on device 8"):
        t.resolve("", "MatMulInteger", 8)  # no silent CPU fallback
