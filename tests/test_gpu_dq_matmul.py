"""Fused DequantizeLinear -> [Cast] -> MatMul on the GPU against the oracle's
two-node chain (DequantizeLinear then MatMul), with the tolerance of the
rel-L2 <= 1e-3 for FLOAT16/BFLOAT16, <= 1e-5 for FLOAT."""
import numpy as np
import pytest
import torch

import oracle as O
from util import random_q, rel_l2, scale_raw, to_dev

pytestmark = pytest.mark.gpu
TOL = {O.FLOAT: 1e-5, O.FLOAT16: 1e-3, O.BFLOAT16: 1e-3}
TORCH = {O.FLOAT: torch.float32, O.FLOAT16: torch.float16, O.BFLOAT16: torch.bfloat16}


def finite_q(seed, shape, dt):
    """Random weight codes without the NaN/Inf encodings of the float8 types."""
    if dt == O.F8E4M3FN:
        return O.f32_to_f8e4m3fn(O.randn(seed, shape))
    if dt in (O.F8E5M2, O.F8E4M3FNUZ, O.F8E5M2FNUZ):
        n = int(np.prod(shape))
        mag = O.randint(seed, (n,), 0, 100)
        sign = O.randint(seed + 1000, (n,), 0, 1) * 128
        return (mag + sign).astype(np.uint8) if dt == O.F8E5M2 else mag.astype(np.uint8)
    return random_q(seed, shape, dt)


def run_case(b2, M, K, N, wdt, s_dt, act_dt, axis=0, block=None, zp=False, cast=0, seed=1,
             lead=None):
    """Returns (gpu, oracle) outputs as float32 arrays."""
    # weight + scales in the requested layout
    w = finite_q(seed, (K, N), wdt)
    if block is None:               # per-axis
        s_shape = (K,) if axis == 0 else (N,)
    elif block == 0:                # per-tensor
        s_shape = ()
    else:                           # blocked
        s_shape = (K // block, N) if axis == 0 else (K, N // block)
    sn = int(np.prod(s_shape)) if s_shape else 1
    s = scale_raw(O.rand_uniform(seed + 1, (sn,), 0.002, 0.02), s_dt)
    z = random_q(seed + 2, s_shape if s_shape else (1,), wdt, -2, 2) if zp else None
    a32 = O.randn(seed + 3, (M, K))
    a_raw = {O.FLOAT: a32, O.FLOAT16: O.f32_to_f16_bits(a32), O.BFLOAT16: O.f32_to_bf16_bits(a32)}[act_dt]
    # oracle: DequantizeLinear, optional Cast, MatMul in the activation dtype
    wq = O.dequantize_linear(w, wdt, (K, N), s, s_dt, s_shape, z, s_shape if zp else None, axis)
    wf = wq if s_dt == O.FLOAT else O.f16_bits_to_f32(wq)
    if cast == O.FLOAT16:
        wb = O.f32_to_f16_bits(wf)
    elif cast == O.BFLOAT16:
        wb = O.f32_to_bf16_bits(wf)
    elif cast == O.FLOAT:
        wb = wf
    else:
        wb = wq
    ref = O.matmul(a_raw, wb, act_dt)
    # GPU
    tw = b2.QTensor(to_dev(w), wdt, (K, N))
    ts = to_dev(s, torch.float16 if s_dt == O.FLOAT16 else None)
    ts = ts.reshape(s_shape) if s_shape else ts.reshape(())
    tz = b2.QTensor(to_dev(z), wdt, s_shape if s_shape else ()) if zp else None
    ta = to_dev(a_raw).view(TORCH[act_dt]).reshape(M, K)
    if lead:
        ta = ta.reshape(*lead, K)
    cast_t = {0: None, O.FLOAT: torch.float32, O.FLOAT16: torch.float16, O.BFLOAT16: torch.bfloat16}[cast]
    y = b2.DequantizeMatMul()(ta, tw, ts, tz, axis=axis, cast_dtype=cast_t)
    torch.cuda.synchronize()
    y = y.float().cpu().numpy().reshape(M, N)
    up = {O.FLOAT: lambda t: t, O.FLOAT16: O.f16_bits_to_f32, O.BFLOAT16: O.bf16_bits_to_f32}[act_dt]
    return y, up(ref)


@pytest.mark.parametrize("M", [1, 2, 3, 4])
def test_decode_gemv_int4_fp16_config3(b2, cuda, M):
    # int4 blocked along K (block 128), FLOAT16 scales, no zero point.
    y, ref = run_case(b2, M, 4096, 4096, O.INT4, O.FLOAT16, O.FLOAT16, block=128)
    assert rel_l2(y, ref) <= TOL[O.FLOAT16]


def test_decode_gemv_down_proj_shape(b2, cuda):
    y, ref = run_case(b2, 1, 11008, 4096, O.INT4, O.FLOAT16, O.FLOAT16, block=128, seed=7)
    assert rel_l2(y, ref) <= TOL[O.FLOAT16]


def test_config1_int4_zero_point_fp32(b2, cuda):
    # int4 [4096,4096], block 32 along K, fp32 scales, int4 zero points,
    # fp32 activations [1, 32, 4096].
    y, ref = run_case(b2, 32, 4096, 4096, O.INT4, O.FLOAT, O.FLOAT, block=32, zp=True, lead=(1, 32))
    assert rel_l2(y, ref) <= TOL[O.FLOAT]


@pytest.mark.parametrize("wdt", [O.F8E4M3FN, O.F4E2M1])
def test_prefill_style_fp8_fp4_cast_bf16(b2, cuda, wdt):
    # BASELINE config 5 weight path: fp8/fp4 blocked along K (block 32), fp32 scales,
    # DequantizeLinear -> Cast(BFLOAT16) -> MatMul with bf16 activations.
    y, ref = run_case(b2, 64, 512, 384, wdt, O.FLOAT, O.BFLOAT16, block=32, cast=O.BFLOAT16)
    assert rel_l2(y, ref) <= TOL[O.BFLOAT16]


@pytest.mark.parametrize("wdt,s_dt,act,axis,block,zp,cast", [
    (O.UINT4, O.FLOAT16, O.FLOAT16, 0, 64, False, 0),
    (O.INT4, O.FLOAT, O.FLOAT, 1, None, True, 0),        # per-axis along N
    (O.INT8, O.FLOAT, O.FLOAT16, 0, None, True, O.FLOAT16),  # per-axis along K
    (O.UINT8, O.FLOAT16, O.FLOAT16, 1, 16, True, 0),      # blocked along N
    (O.INT4, O.FLOAT, O.FLOAT, 0, 0, True, 0),            # per-tensor
    (O.F8E5M2, O.FLOAT16, O.BFLOAT16, 0, 32, False, O.BFLOAT16),
    (O.INT2, O.FLOAT, O.FLOAT, 0, 16, True, 0),
])
def test_layouts_and_types(b2, cuda, wdt, s_dt, act, axis, block, zp, cast):
    for M in (1, 5, 40):
        y, ref = run_case(b2, M, 256, 192, wdt, s_dt, act, axis, block, zp, cast, seed=M)
        assert rel_l2(y, ref) <= TOL[act], (M, rel_l2(y, ref))


def test_repeated_calls_reuse_workspace(b2, cuda):
    # split-K counters must return to zero: many calls on one workspace agree.
    outs = [run_case(b2, 1, 4096, 4096, O.INT4, O.FLOAT16, O.FLOAT16, block=128, seed=3)[0]
            for _ in range(3)]
    assert np.array_equal(outs[0], outs[1]) and np.array_equal(outs[1], outs[2])


def test_dtype_mismatch_errors(b2, cuda):
    w = b2.QTensor(to_dev(random_q(1, (64, 32), O.INT4)), O.INT4, (64, 32))
    s = torch.ones((2, 32), device="cuda", dtype=torch.float16)
    a = torch.ones((1, 64), device="cuda", dtype=torch.float32)
    with pytest.raises(ValueError, match="must share the same dtype"):
        b2.DequantizeMatMul()(a, w, s, axis=0)
    a16 = torch.ones((1, 63), device="cuda", dtype=torch.float16)
    with pytest.raises(ValueError, match="incompatible inner dimensions"):
        b2.DequantizeMatMul()(a16, w, s, axis=0)


# ---------------------------------------------------------------------------
# Every kernel family on the same shapes (ONNXL_B200_DQ_KERNEL forces one).
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("M", [1, 3, 5, 8, 32, 64, 100, 300])
def test_tensor_core_int4_fp16(b2, cuda, monkeypatch, M):
    monkeypatch.setenv("ONNXL_B200_DQ_KERNEL", "tc")
    y, ref = run_case(b2, M, 1024, 512, O.INT4, O.FLOAT16, O.FLOAT16, block=128, seed=M)
    assert rel_l2(y, ref) <= TOL[O.FLOAT16]


@pytest.mark.parametrize("wdt,axis,block,K,N", [
    (O.INT4, 1, None, 512, 200),    # per-column fp16 scales, N not a multiple of 128
    (O.UINT4, 0, 96, 384, 256),     # blocks that do not divide the 64-row stage
    (O.INT4, 0, 32, 256, 136),      # two scale blocks per stage
])
def test_tensor_core_int4_scale_layouts(b2, cuda, monkeypatch, wdt, axis, block, K, N):
    monkeypatch.setenv("ONNXL_B200_DQ_KERNEL", "tc")
    for M in (5, 40):
        y, ref = run_case(b2, M, K, N, wdt, O.FLOAT16, O.FLOAT16, axis=axis, block=block, seed=M + 9)
        assert rel_l2(y, ref) <= TOL[O.FLOAT16], (M, rel_l2(y, ref))


def test_tensor_core_config3_shape_batch32(b2, cuda, monkeypatch):
    monkeypatch.setenv("ONNXL_B200_DQ_KERNEL", "tc")
    y, ref = run_case(b2, 32, 4096, 4096, O.INT4, O.FLOAT16, O.FLOAT16, block=128, seed=11)
    assert rel_l2(y, ref) <= TOL[O.FLOAT16]


@pytest.mark.parametrize("wdt", [O.F8E4M3FN, O.F4E2M1])
@pytest.mark.parametrize("M", [8, 64, 300])
def test_tensor_core_fp8_fp4_bf16(b2, cuda, monkeypatch, wdt, M):
    monkeypatch.setenv("ONNXL_B200_DQ_KERNEL", "tc")
    y, ref = run_case(b2, M, 512, 384, wdt, O.FLOAT, O.BFLOAT16, block=32, cast=O.BFLOAT16, seed=M)
    assert rel_l2(y, ref) <= TOL[O.BFLOAT16]


@pytest.mark.parametrize("wdt,s_dt,act,axis,block,zp,cast", [
    (O.UINT8, O.FLOAT16, O.FLOAT16, 0, 64, True, 0),
    (O.INT4, O.FLOAT16, O.FLOAT16, 0, 32, True, 0),
    (O.INT4, O.FLOAT, O.BFLOAT16, 1, None, True, O.BFLOAT16),
    (O.UINT4, O.FLOAT16, O.FLOAT16, 0, 0, False, 0),
])
def test_tensor_core_generic_layouts(b2, cuda, monkeypatch, wdt, s_dt, act, axis, block, zp, cast):
    monkeypatch.setenv("ONNXL_B200_DQ_KERNEL", "tc")
    for M in (6, 40):
        y, ref = run_case(b2, M, 256, 192, wdt, s_dt, act, axis, block, zp, cast, seed=M + 3)
        assert rel_l2(y, ref) <= TOL[act], (M, rel_l2(y, ref))


@pytest.mark.parametrize("path", ["simt", "gemv"])
def test_cuda_core_paths_config3_decode(b2, cuda, monkeypatch, path):
    monkeypatch.setenv("ONNXL_B200_DQ_KERNEL", path)
    y, ref = run_case(b2, 2, 4096, 4096, O.INT4, O.FLOAT16, O.FLOAT16, block=128, seed=21)
    assert rel_l2(y, ref) <= TOL[O.FLOAT16]


# ---------------------------------------------------------------------------
# Decode path on register-level MMA (M <= 16, INT4/UINT4, FLOAT16 chain): the
# default for these shapes.  Stream-K splits, whole-tile CTAs, partial last
# stages, every supported scale layout.
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("M", [1, 2, 3, 5, 8, 9, 12, 16])
def test_mma_decode_config3_batches(b2, cuda, M):
    y, ref = run_case(b2, M, 4096, 4096, O.INT4, O.FLOAT16, O.FLOAT16, block=128, seed=40 + M)
    assert rel_l2(y, ref) <= TOL[O.FLOAT16]


@pytest.mark.parametrize("K,N", [(4096, 11008), (11008, 4096), (128, 256), (128, 76800),
                                 (256, 1024), (4096, 1024),
                                 # column shards of 11008 over 2 / 4 / 8 ranks: ragged last tile
                                 (4096, 5504), (4096, 2752), (4096, 1376), (512, 32)])
def test_mma_decode_llama_and_edge_shapes(b2, cuda, K, N):
    for M in (1, 4):
        y, ref = run_case(b2, M, K, N, O.INT4, O.FLOAT16, O.FLOAT16, block=128, seed=K + N + M)
        assert rel_l2(y, ref) <= TOL[O.FLOAT16], (M, rel_l2(y, ref))


@pytest.mark.parametrize("wdt,block,axis", [
    (O.INT4, 32, 0), (O.UINT4, 64, 0), (O.UINT4, 128, 0), (O.INT4, 256, 0),
    (O.INT4, None, 1),   # per-column scales
    (O.UINT4, 0, 0),     # per-tensor scale
])
def test_mma_decode_scale_layouts(b2, cuda, wdt, block, axis):
    for M in (1, 6):
        y, ref = run_case(b2, M, 1024, 768, wdt, O.FLOAT16, O.FLOAT16, axis=axis, block=block,
                          seed=M + 7)
        assert rel_l2(y, ref) <= TOL[O.FLOAT16], (M, rel_l2(y, ref))


def test_mma_decode_partial_last_stage_and_cast(b2, cuda):
    # K = 200: the last 128-row stage is partly outside the weight (TMA zero fill);
    # per-column scales; an explicit Cast(FLOAT16) between the nodes.
    for M in (1, 11):
        y, ref = run_case(b2, M, 200, 512, O.INT4, O.FLOAT16, O.FLOAT16, axis=1, block=None,
                          cast=O.FLOAT16, seed=M)
        assert rel_l2(y, ref) <= TOL[O.FLOAT16], (M, rel_l2(y, ref))


def test_mma_decode_unaligned_activations_fall_back(b2, cuda):
    # Activations at an address that is not 16-byte aligned cannot be read by
    # TMA; the call still succeeds (CUDA-core kernel) and agrees.
    M, K, N = 2, 512, 512
    w = random_q(5, (K, N), O.INT4)
    s = to_dev(scale_raw(O.rand_uniform(6, (K // 128 * N,), 0.002, 0.02), O.FLOAT16),
               torch.float16).reshape(K // 128, N)
    a = torch.randn(M * K + 1, device="cuda").half()
    tw = b2.QTensor(to_dev(w), O.INT4, (K, N))
    y_off = b2.DequantizeMatMul()(a[1:].view(M, K), tw, s, None, axis=0)
    y_al = b2.DequantizeMatMul()(a[1:].clone().view(M, K), tw, s, None, axis=0)
    torch.cuda.synchronize()
    assert rel_l2(y_off.float().cpu().numpy(), y_al.float().cpu().numpy()) <= TOL[O.FLOAT16]


# ---------------------------------------------------------------------------
# Large M (prefill): the weight is dequantized once into the workspace and the
# tcgen05 GEMM streams both operands by TMA.
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("wdt,s_dt,act,block,zp,cast", [
    (O.F8E4M3FN, O.FLOAT, O.BFLOAT16, 32, False, O.BFLOAT16),
    (O.F4E2M1, O.FLOAT, O.BFLOAT16, 32, False, O.BFLOAT16),
    (O.INT4, O.FLOAT16, O.FLOAT16, 64, False, 0),
    (O.UINT8, O.FLOAT16, O.FLOAT16, 32, True, 0),
])
def test_prefill_predequantized_gemm(b2, cuda, wdt, s_dt, act, block, zp, cast):
    y, ref = run_case(b2, 2304, 320, 200, wdt, s_dt, act, axis=0, block=block, zp=zp, cast=cast,
                      seed=17)
    assert rel_l2(y, ref) <= TOL[act], rel_l2(y, ref)


# ---------------------------------------------------------------------------
# Failure detection: a tensor-core GEMM whose bounded wait runs out reports
# it, and leaves the caller's workspace valid for the next call.
# ---------------------------------------------------------------------------

def test_gemm_timeout_is_reported_and_workspace_stays_valid(b2, cuda, monkeypatch):
    import ctypes as C
    from onnx_light_b200 import _capi as capi
    lib = capi.lib()
    # the tensor-core plan (forced: the default for 32 rows is the narrow-tile
    # GEMV), K split across CTAs
    monkeypatch.setenv("ONNXL_B200_DQ_KERNEL", "tc")
    M, K, N = 32, 4096, 4096
    w = random_q(41, (K, N), O.INT4)
    s = scale_raw(O.rand_uniform(42, (K // 128 * N,), 0.002, 0.02), O.FLOAT16)
    a = O.f32_to_f16_bits(O.randn(43, (M, K)))
    wq = O.dequantize_linear(w, O.INT4, (K, N), s, O.FLOAT16, (K // 128, N), None, None, 0)
    ref = O.f16_bits_to_f32(O.matmul(a, wq, O.FLOAT16))
    tw, ts, ta = to_dev(w), to_dev(s), to_dev(a)
    y = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
    da = capi.Desc(ta.data_ptr(), capi.FLOAT16, (M, K))
    dw = capi.Desc(tw.data_ptr(), capi.INT4, (K, N))
    ds = capi.Desc(ts.data_ptr(), capi.FLOAT16, (K // 128, N))
    dy = capi.Desc(y.data_ptr(), capi.FLOAT16, (M, N))
    stream = capi.stream_ptr()
    need = C.c_size_t(0)
    capi.check(lib.b2_dequantize_matmul(da.ref, dw.ref, ds.ref, None, 0, 0, dy.ref, None,
                                        C.byref(need), stream))
    ws = torch.zeros(need.value, dtype=torch.uint8, device="cuda")
    assert lib.b2_kernel_status(1) == 0
    # every CTA's first data wait runs out after 10 ms: code 1 comes back
    code = lib.b2_selftest_gemm_timeout(da.ref, dw.ref, ds.ref, dy.ref, C.c_void_p(ws.data_ptr()),
                                        need.value, 10_000_000, stream)
    assert code == 1
    assert lib.b2_kernel_status(0) == 1
    buf = C.create_string_buffer(256)
    lib.b2_last_error(buf, 256)
    assert b"dq_gemm_tc" in buf.value
    assert lib.b2_kernel_status(1) == 1 and lib.b2_kernel_status(0) == 0
    # the give-up arrivals returned every split-K counter to zero
    assert int(ws[:65536].count_nonzero()) == 0
    # so a real call on the same workspace computes the right result
    cap = C.c_size_t(need.value)
    capi.check(lib.b2_dequantize_matmul(da.ref, dw.ref, ds.ref, None, 0, 0, dy.ref,
                                        C.c_void_p(ws.data_ptr()), C.byref(cap), stream))
    torch.cuda.synchronize()
    assert rel_l2(y.float().cpu().numpy(), ref) <= TOL[O.FLOAT16]
    assert lib.b2_kernel_status(0) == 0


def test_workspace_is_per_stream(b2, cuda):
    """Calls on two streams get two workspaces (no shared split-K counters)."""
    from onnx_light_b200 import kernels
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    w1 = kernels.workspace(torch.device("cuda", 0), 1 << 20, s1)
    w2 = kernels.workspace(torch.device("cuda", 0), 1 << 20, s2)
    assert w1.data_ptr() != w2.data_ptr()
    assert kernels.workspace(torch.device("cuda", 0), 1 << 20, s1).data_ptr() == w1.data_ptr()


# ---------------------------------------------------------------------------
# FLOAT activations with integer weights (dq_gemm_f32, the default for them
# from 3 rows): every weight type, scale type and layout it takes, ragged
# rows / columns / K, one and several row tiles and split-K.
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("wdt,s_dt,cast,axis,block,zp", [
    (O.INT4, O.FLOAT, 0, 0, 32, True),        # config 1's layout
    (O.UINT4, O.FLOAT, 0, 0, 64, False),
    (O.INT8, O.FLOAT, 0, 0, 96, True),        # blocks that straddle the warps' K slices
    (O.UINT8, O.FLOAT, O.FLOAT, 1, None, True),  # per-column scales
    (O.INT4, O.FLOAT16, O.FLOAT, 0, 32, True),   # FLOAT16 DequantizeLinear output + Cast
    (O.UINT4, O.FLOAT16, O.FLOAT, 0, 0, True),   # per-tensor
])
@pytest.mark.parametrize("M,K,N", [(3, 1000, 196), (16, 512, 384), (33, 2048, 260), (70, 256, 4100)])
def test_fp32_chain_kernel(b2, cuda, monkeypatch, wdt, s_dt, cast, axis, block, zp, M, K, N):
    monkeypatch.setenv("ONNXL_B200_DQ_KERNEL", "f32")
    if block and K % block:
        K = (K // block + 1) * block
    y, ref = run_case(b2, M, K, N, wdt, s_dt, O.FLOAT, axis, block, zp, cast, seed=M + K)
    assert rel_l2(y, ref) <= TOL[O.FLOAT], rel_l2(y, ref)


def test_fp32_chain_config1_split_k_is_deterministic(b2, cuda):
    # config 1 takes dq_gemm_f32 with split-K; repeated calls are bit-identical
    # and agree with the generic CUDA-core GEMM within the contract
    outs = [run_case(b2, 32, 4096, 4096, O.INT4, O.FLOAT, O.FLOAT, block=32, zp=True, seed=5,
                     lead=(1, 32)) for _ in range(3)]
    assert np.array_equal(outs[0][0], outs[1][0]) and np.array_equal(outs[1][0], outs[2][0])
    assert rel_l2(outs[0][0], outs[0][1]) <= TOL[O.FLOAT]


def test_fp32_chain_unaligned_activations_fall_back(b2, cuda):
    # activations one float past a 16-byte boundary: the generic kernel runs
    K, N, M = 256, 192, 9
    w = b2.QTensor(to_dev(random_q(3, (K, N), O.INT4)), O.INT4, (K, N))
    s = to_dev(O.rand_uniform(4, (K // 32 * N,), 0.002, 0.02)).reshape(K // 32, N)
    base = torch.from_numpy(O.randn(5, (M * K + 1,))).cuda()
    a_off = base[1:].view(M, K)
    a_al = a_off.clone()
    y_off = b2.DequantizeMatMul()(a_off, w, s, axis=0)
    y_al = b2.DequantizeMatMul()(a_al, w, s, axis=0)
    torch.cuda.synchronize()
    assert rel_l2(y_off.cpu().numpy(), y_al.cpu().numpy()) <= TOL[O.FLOAT]


# ---------------------------------------------------------------------------
# Decode path with the reference's exact fp16 weights (dq_gemv_x, forced with
# ONNXL_B200_DQ_KERNEL=x): one to eight activation tiles, two row passes,
# stream-K splits, every scale layout it takes, ragged shapes.
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("M", [1, 2, 5, 8, 9, 16, 17, 32, 33, 64])
def test_exact_decode_config3_batches(b2, cuda, monkeypatch, M):
    monkeypatch.setenv("ONNXL_B200_DQ_KERNEL", "x")
    y, ref = run_case(b2, M, 4096, 4096, O.INT4, O.FLOAT16, O.FLOAT16, block=128, seed=60 + M)
    assert rel_l2(y, ref) <= TOL[O.FLOAT16], rel_l2(y, ref)


@pytest.mark.parametrize("K,N", [(11008, 4096), (4096, 11008), (1000, 4128), (200, 96)])
def test_exact_decode_shapes(b2, cuda, monkeypatch, K, N):
    monkeypatch.setenv("ONNXL_B200_DQ_KERNEL", "x")
    for M in (1, 12, 40):
        y, ref = run_case(b2, M, K, N, O.INT4, O.FLOAT16, O.FLOAT16, block=None, axis=1, seed=K + M)
        assert rel_l2(y, ref) <= TOL[O.FLOAT16], (M, rel_l2(y, ref))


@pytest.mark.parametrize("wdt,block,axis", [(O.INT4, 32, 0), (O.UINT4, 64, 0), (O.INT4, 256, 0),
                                            (O.UINT4, 0, 0), (O.INT4, None, 1)])
def test_exact_decode_scale_layouts(b2, cuda, monkeypatch, wdt, block, axis):
    monkeypatch.setenv("ONNXL_B200_DQ_KERNEL", "x")
    K = 512 if block != 256 else 768
    for M in (3, 24):
        y, ref = run_case(b2, M, K, 512, wdt, O.FLOAT16, O.FLOAT16, axis=axis, block=block, seed=M + 71)
        assert rel_l2(y, ref) <= TOL[O.FLOAT16], (M, rel_l2(y, ref))


def test_exact_decode_weights_match_the_reference_rounding(b2, cuda, monkeypatch):
    # a single activation row that is one-hot at k selects row k of the
    # dequantized weight: the kernel's weights equal the reference's fp16
    # DequantizeLinear output bit for bit (scales spanning normal and
    # subnormal products)
    monkeypatch.setenv("ONNXL_B200_DQ_KERNEL", "x")
    K, N = 256, 256
    w = random_q(5, (K, N), O.INT4)
    s = scale_raw(np.concatenate([O.rand_uniform(6, (N,), 1e-6, 1e-4),
                                  O.rand_uniform(7, (N,), 0.002, 300.0)]), O.FLOAT16)
    s_shape = (K // 128, N)
    wq = O.dequantize_linear(w, O.INT4, (K, N), s, O.FLOAT16, s_shape, None, None, 0)
    tw = b2.QTensor(to_dev(w), O.INT4, (K, N))
    ts = to_dev(s, torch.float16).reshape(s_shape)
    for k in (0, 77, 200):
        a = torch.zeros((1, K), dtype=torch.float16, device="cuda")
        a[0, k] = 1.0
        y = b2.DequantizeMatMul()(a, tw, ts, None, axis=0)
        torch.cuda.synchronize()
        got = y.view(torch.int16).cpu().numpy().reshape(N).view(np.uint16)
        assert np.array_equal(got, wq.reshape(K, N)[k]), k


def test_exact_decode_repeated_calls_are_identical(b2, cuda, monkeypatch):
    monkeypatch.setenv("ONNXL_B200_DQ_KERNEL", "x")
    outs = [run_case(b2, 33, 4096, 4096, O.INT4, O.FLOAT16, O.FLOAT16, block=128, seed=3)[0]
            for _ in range(3)]
    assert np.array_equal(outs[0], outs[1]) and np.array_equal(outs[1], outs[2])


# ---------------------------------------------------------------------------
# Decode path on narrow column tiles (dq_gemv_n, forced with
# ONNXL_B200_DQ_KERNEL=n): whole K per CTA, several tiles per CTA, chunks of
# 256 / 128 / 64 rows, one to eight activation tiles, every scale layout it
# takes.
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("M", [1, 3, 8, 9, 16, 17, 32, 33, 40, 63, 64])
def test_narrow_decode_config3_batches(b2, cuda, monkeypatch, M):
    monkeypatch.setenv("ONNXL_B200_DQ_KERNEL", "n")
    y, ref = run_case(b2, M, 4096, 4096, O.INT4, O.FLOAT16, O.FLOAT16, block=128, seed=80 + M)
    assert rel_l2(y, ref) <= TOL[O.FLOAT16], rel_l2(y, ref)


@pytest.mark.parametrize("K,N", [(11008, 4096), (4096, 11008), (1000, 4128), (200, 96), (4096, 32)])
def test_narrow_decode_shapes(b2, cuda, monkeypatch, K, N):
    monkeypatch.setenv("ONNXL_B200_DQ_KERNEL", "n")
    for M in (1, 12, 30, 50):
        y, ref = run_case(b2, M, K, N, O.INT4, O.FLOAT16, O.FLOAT16, block=None, axis=1, seed=K + M + 1)
        assert rel_l2(y, ref) <= TOL[O.FLOAT16], (M, rel_l2(y, ref))


@pytest.mark.parametrize("wdt,block,axis", [(O.INT4, 16, 0), (O.UINT4, 64, 0), (O.INT4, 512, 0),
                                            (O.UINT4, 0, 0), (O.INT4, None, 1)])
def test_narrow_decode_scale_layouts(b2, cuda, monkeypatch, wdt, block, axis):
    monkeypatch.setenv("ONNXL_B200_DQ_KERNEL", "n")
    K = 1024
    for M in (2, 20, 64):
        y, ref = run_case(b2, M, K, 512, wdt, O.FLOAT16, O.FLOAT16, axis=axis, block=block, seed=M + 91)
        assert rel_l2(y, ref) <= TOL[O.FLOAT16], (M, rel_l2(y, ref))


def test_narrow_decode_weights_match_the_reference_rounding(b2, cuda, monkeypatch):
    monkeypatch.setenv("ONNXL_B200_DQ_KERNEL", "n")
    K, N = 512, 64
    w = random_q(15, (K, N), O.INT4)
    s = scale_raw(np.concatenate([O.rand_uniform(16, (2 * N,), 1e-6, 1e-4),
                                  O.rand_uniform(17, (2 * N,), 0.002, 300.0)]), O.FLOAT16)
    s_shape = (K // 128, N)
    wq = O.dequantize_linear(w, O.INT4, (K, N), s, O.FLOAT16, s_shape, None, None, 0)
    tw = b2.QTensor(to_dev(w), O.INT4, (K, N))
    ts = to_dev(s, torch.float16).reshape(s_shape)
    for k in (0, 130, 300, 511):
        a = torch.zeros((1, K), dtype=torch.float16, device="cuda")
        a[0, k] = 1.0
        y = b2.DequantizeMatMul()(a, tw, ts, None, axis=0)
        torch.cuda.synchronize()
        got = y.view(torch.int16).cpu().numpy().reshape(N).view(np.uint16)
        assert np.array_equal(got, wq.reshape(K, N)[k]), k


# ---------------------------------------------------------------------------
# Decode path split along K inside clusters (dq_gemv_c, forced with
# ONNXL_B200_DQ_KERNEL=c for the magic-number form, cx for the exact fp16
# weights): clusters of 8 / 4 / 2 / 1, more tiles than clusters, ragged
# shapes, every scale layout it takes.
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("form", ["c", "cx"])
@pytest.mark.parametrize("M", [1, 3, 8, 9, 16, 17, 32])
def test_cluster_decode_config3_batches(b2, cuda, monkeypatch, M, form):
    monkeypatch.setenv("ONNXL_B200_DQ_KERNEL", form)
    y, ref = run_case(b2, M, 4096, 4096, O.INT4, O.FLOAT16, O.FLOAT16, block=128, seed=100 + M)
    assert rel_l2(y, ref) <= TOL[O.FLOAT16], rel_l2(y, ref)


@pytest.mark.parametrize("form", ["c", "cx"])
@pytest.mark.parametrize("K,N", [(11008, 4096), (4096, 11008), (1000, 4128), (200, 96), (384, 64),
                                 (128, 8192)])
def test_cluster_decode_shapes(b2, cuda, monkeypatch, K, N, form):
    monkeypatch.setenv("ONNXL_B200_DQ_KERNEL", form)
    for M in (1, 12, 30):
        y, ref = run_case(b2, M, K, N, O.INT4, O.FLOAT16, O.FLOAT16, block=None, axis=1, seed=K + M + 2)
        assert rel_l2(y, ref) <= TOL[O.FLOAT16], (M, rel_l2(y, ref))


@pytest.mark.parametrize("form", ["c", "cx"])
@pytest.mark.parametrize("wdt,block,axis", [(O.INT4, 32, 0), (O.UINT4, 64, 0), (O.INT4, 256, 0),
                                            (O.UINT4, 0, 0), (O.INT4, None, 1)])
def test_cluster_decode_scale_layouts(b2, cuda, monkeypatch, wdt, block, axis, form):
    monkeypatch.setenv("ONNXL_B200_DQ_KERNEL", form)
    K = 1024
    for M in (2, 20):
        y, ref = run_case(b2, M, K, 512, wdt, O.FLOAT16, O.FLOAT16, axis=axis, block=block, seed=M + 93)
        assert rel_l2(y, ref) <= TOL[O.FLOAT16], (M, rel_l2(y, ref))


def test_cluster_decode_weights_match_the_reference_rounding(b2, cuda, monkeypatch):
    monkeypatch.setenv("ONNXL_B200_DQ_KERNEL", "cx")
    K, N = 1024, 256
    w = random_q(25, (K, N), O.INT4)
    s = scale_raw(np.concatenate([O.rand_uniform(26, (4 * N,), 1e-6, 1e-4),
                                  O.rand_uniform(27, (4 * N,), 0.002, 300.0)]), O.FLOAT16)
    s_shape = (K // 128, N)
    wq = O.dequantize_linear(w, O.INT4, (K, N), s, O.FLOAT16, s_shape, None, None, 0)
    tw = b2.QTensor(to_dev(w), O.INT4, (K, N))
    ts = to_dev(s, torch.float16).reshape(s_shape)
    for k in (0, 130, 700, 1023):
        a = torch.zeros((1, K), dtype=torch.float16, device="cuda")
        a[0, k] = 1.0
        y = b2.DequantizeMatMul()(a, tw, ts, None, axis=0)
        torch.cuda.synchronize()
        got = y.view(torch.int16).cpu().numpy().reshape(N).view(np.uint16)
        assert np.array_equal(got, wq.reshape(K, N)[k]), k


@pytest.mark.parametrize("form", ["c", "cx"])
def test_cluster_decode_repeated_calls_are_identical(b2, cuda, monkeypatch, form):
    monkeypatch.setenv("ONNXL_B200_DQ_KERNEL", form)
    outs = [run_case(b2, 5, 4096, 11008, O.INT4, O.FLOAT16, O.FLOAT16, block=128, seed=4)[0]
            for _ in range(3)]
    assert np.array_equal(outs[0], outs[1]) and np.array_equal(outs[1], outs[2])


@pytest.mark.parametrize("K,N", [(4096, 4096), (11008, 4096), (4096, 11008)])
def test_mma_decode_stream_k_partition(b2, cuda, monkeypatch, K, N):
    # the stream-K unit partition (ONNXL_B200_GEMV_STREAMK) that shapes with
    # more tiles than SMs take; the default splits each tile among whole CTAs
    monkeypatch.setenv("ONNXL_B200_GEMV_STREAMK", "1")
    for M in (1, 9):
        y, ref = run_case(b2, M, K, N, O.INT4, O.FLOAT16, O.FLOAT16, block=128, seed=K + N + M)
        assert rel_l2(y, ref) <= TOL[O.FLOAT16], (M, rel_l2(y, ref))


# ---------------------------------------------------------------------------
# Projections that share their activations in one call (b2_dequantize_matmul_group):
# the members' weight tiles split among the CTAs of one decode launch, or one
# call per member when they do not fit it.
# ---------------------------------------------------------------------------

def group_case(b2, M, K, Ns, block, seed, axis=0):
    """Runs DequantizeMatMulGroup on len(Ns) int4 members; returns (gpu, oracle) lists."""
    a32 = O.randn(seed, (M, K))
    a_raw = O.f32_to_f16_bits(a32)
    ta = to_dev(a_raw).view(torch.float16).reshape(M, K)
    ws, ss, refs = [], [], []
    for j, N in enumerate(Ns):
        w = finite_q(seed + 10 * j + 1, (K, N), O.INT4)
        s_shape = (K // block, N) if block else ((K,) if axis == 0 else (N,))
        s = scale_raw(O.rand_uniform(seed + 10 * j + 2, (int(np.prod(s_shape)),), 0.002, 0.02), O.FLOAT16)
        wq = O.dequantize_linear(w, O.INT4, (K, N), s, O.FLOAT16, s_shape, None, None, axis)
        refs.append(O.f16_bits_to_f32(O.matmul(a_raw, wq, O.FLOAT16)))
        ws.append(b2.QTensor(to_dev(w), O.INT4, (K, N)))
        ss.append(to_dev(s, torch.float16).reshape(s_shape))
    ys = b2.DequantizeMatMulGroup()(ta, ws, ss, axis=axis)
    torch.cuda.synchronize()
    return [y.float().cpu().numpy().reshape(M, N) for y, N in zip(ys, Ns)], refs, (ta, ws, ss)


@pytest.mark.parametrize("M,K,Ns,block,axis", [(1, 4096, (4096, 4096, 4096), 128, 0),
                                               (8, 4096, (11008, 11008), 128, 0),
                                               (16, 4096, (4096, 1024, 1024), 128, 0),
                                               (5, 11008, (4096, 256, 512, 768), 64, 0),
                                               (3, 1000, (4128, 96), None, 1),
                                               (2, 512, (64, 4096), None, 0)])
def test_group_projections_match_the_oracle(b2, cuda, M, K, Ns, block, axis):
    # the last case (per-row scales) is not the decode kernel's: one call per member
    ys, refs, _ = group_case(b2, M, K, Ns, block, seed=500 + M + len(Ns), axis=axis)
    for y, ref in zip(ys, refs):
        assert rel_l2(y, ref) <= TOL[O.FLOAT16], rel_l2(y, ref)


def test_group_of_one_is_the_single_call(b2, cuda):
    # one member: the same decode plan and launch as DequantizeMatMul, bit for bit
    ys, refs, (ta, ws, ss) = group_case(b2, 1, 4096, (11008,), 128, seed=611)
    y1 = b2.DequantizeMatMul()(ta, ws[0], ss[0], None, axis=0)
    torch.cuda.synchronize()
    assert np.array_equal(ys[0], y1.float().cpu().numpy().reshape(1, 11008))


@pytest.mark.parametrize("M", [24, 64])
def test_group_beyond_the_decode_kernel_runs_each_member(b2, cuda, M):
    ys, refs, _ = group_case(b2, M, 4096, (4096, 1024), 128, seed=700 + M)
    for y, ref in zip(ys, refs):
        assert rel_l2(y, ref) <= TOL[O.FLOAT16], rel_l2(y, ref)


def test_group_rejects_a_bad_member_count(b2, cuda):
    from onnx_light_b200 import _capi as capi
    a = torch.zeros((1, 64), dtype=torch.float16, device="cuda")
    ad = capi.Desc(a.data_ptr(), O.FLOAT16, (1, 64))
    for count in (0, 5):
        rc = capi.lib().b2_dequantize_matmul_group(count, ad.ref, ad.ref, ad.ref, 0, ad.ref, None,
                                                   None, capi.stream_ptr())
        assert rc == capi.B2_ERR_INVALID_ARGUMENT
