"""The no-allocation entry point b2_dequantize_matmul_noalloc.

Callers that cannot allocate device memory (a sealed session memory plan, a
real-time loop, a plugin that only gets its input and output buffers) use this
entry point; it takes its split-K scratch from a fixed array inside the
library instead of a caller workspace.  It must give the same results as
b2_dequantize_matmul, call after call, because the fixed scratch is reused.
Collected last on purpose (file name), so a failure here stops a -x run only
after every other test has run."""
import ctypes as C

import numpy as np
import pytest
import torch

import oracle as O
from util import random_q, rel_l2, scale_raw, to_dev

pytestmark = pytest.mark.gpu


def _inputs(seed, K, N, M):
    """Device tensors (w, s, a) and the oracle's result of the same chain:
    DequantizeLinear (int4, fp16 scales, block 128 along K) then fp16 MatMul."""
    w = random_q(seed, (K, N), O.INT4)
    s = scale_raw(O.rand_uniform(seed + 1, (K // 128 * N,), 0.002, 0.02), O.FLOAT16)
    a = O.f32_to_f16_bits(O.randn(seed + 2, (M, K)))
    wq = O.dequantize_linear(w, O.INT4, (K, N), s, O.FLOAT16, (K // 128, N), None, None, 0)
    ref = O.f16_bits_to_f32(O.matmul(a, wq, O.FLOAT16))
    return (to_dev(w), to_dev(s, torch.float16).reshape(K // 128, N),
            to_dev(a, torch.float16).reshape(M, K), ref)


def _desc(capi, t, dtype, shape):
    return capi.Desc(t.data_ptr(), dtype, shape)


def _call(b2, fn_name, w, s, a, K, N, M):
    from onnx_light_b200 import _capi as capi, kernels
    lib = capi.lib()
    y = torch.empty((M, N), dtype=torch.float16, device="cuda")
    dw = _desc(capi, w, capi.INT4, (K, N))
    ds = _desc(capi, s, capi.FLOAT16, (K // 128, N))
    da = _desc(capi, a, capi.FLOAT16, (M, K))
    dy = _desc(capi, y, capi.FLOAT16, (M, N))
    stream = capi.stream_ptr()
    if fn_name == "noalloc":
        f = lib.b2_dequantize_matmul_noalloc
        f.argtypes = [C.POINTER(capi.B2Tensor)] * 4 + [C.c_int64, C.c_int32, C.POINTER(capi.B2Tensor), C.c_void_p]
        capi.check(f(da.ref, dw.ref, ds.ref, None, 0, 0, dy.ref, stream))
    else:
        kernels.DequantizeMatMul()(a, kernels.QTensor(w, capi.INT4, (K, N)), s, None, axis=0, out=y)
    torch.cuda.synchronize()
    return y.float().cpu().numpy()


@pytest.mark.parametrize("M", [1, 32])
def test_noalloc_matches_oracle_twice_in_a_row(b2, cuda, M):
    # Two different shapes back to back: the second call reuses the fixed
    # scratch the first one left behind (both M = 1, stream-K decode GEMV, and
    # M = 32, tensor-core split-K, sum partial results through it).  Each
    # result is checked against the oracle and against the workspace entry
    # point, within the fp16 MatMul tolerance (rel-L2 1e-3).
    for seed, (K, N) in ((11, (4096, 4096)), (12, (11008, 4096))):
        w, s, a, ref = _inputs(seed + M, K, N, M)
        got = _call(b2, "noalloc", w, s, a, K, N, M)
        assert rel_l2(got, ref) <= 1e-3, rel_l2(got, ref)
        ws = _call(b2, "workspace", w, s, a, K, N, M)
        assert rel_l2(got, ws) <= 1e-3


def test_noalloc_rejects_plans_beyond_the_fixed_scratch(b2, cuda, monkeypatch):
    # FLOAT activations on the generic CUDA-core GEMM, 64 x 16384 outputs split
    # in two along K: the split-K partials alone are 2 x 64 x 16384 x 4 bytes =
    # 8 MiB, beyond the fixed scratch.
    monkeypatch.setenv("ONNXL_B200_DQ_KERNEL", "simt")
    from onnx_light_b200 import _capi as capi
    K, N, M = 4096, 16384, 64
    w = torch.zeros((K * N // 2,), dtype=torch.uint8, device="cuda")
    s = torch.ones((K // 128, N), dtype=torch.float32, device="cuda")
    a = torch.ones((M, K), dtype=torch.float32, device="cuda")
    y = torch.empty((M, N), dtype=torch.float32, device="cuda")
    lib = capi.lib()
    f = lib.b2_dequantize_matmul_noalloc
    f.argtypes = [C.POINTER(capi.B2Tensor)] * 4 + [C.c_int64, C.c_int32, C.POINTER(capi.B2Tensor), C.c_void_p]
    da = capi.Desc(a.data_ptr(), capi.FLOAT, (M, K))
    dw = capi.Desc(w.data_ptr(), capi.INT4, (K, N))
    ds = capi.Desc(s.data_ptr(), capi.FLOAT, (K // 128, N))
    dy = capi.Desc(y.data_ptr(), capi.FLOAT, (M, N))
    rc = f(da.ref, dw.ref, ds.ref, None, 0, 0, dy.ref, capi.stream_ptr())
    assert rc == capi.B2_ERR_WORKSPACE
    buf = C.create_string_buffer(512)
    lib.b2_last_error(buf, 512)
    assert b"fixed scratch" in buf.value
