"""DequantizeLinear on the GPU through the C ABI: bit-exact against onnx-light's
own outputs (fixtures), the known answers of its tests, and the oracle on
larger seeded inputs."""
import json
import os

import numpy as np
import pytest
import torch

import oracle as O
from util import encode_codes, fixture_dq_inputs, load_fixtures, random_q, scale_raw, to_dev

pytestmark = pytest.mark.gpu
META, Z = load_fixtures()
HERE = os.path.dirname(os.path.abspath(__file__))
KAT = json.load(open(os.path.join(HERE, "golden", "kat_reference_tests.json")))


def gpu_dq(b2, x_raw, x_dt, x_shape, s_raw, s_dt, s_shape, zp_raw=None, axis=1):
    x = b2.QTensor(to_dev(x_raw), x_dt, tuple(x_shape))
    s = to_dev(s_raw, torch.float16 if s_dt == O.FLOAT16 else None)
    s = s.reshape(tuple(s_shape)) if len(s_shape) else s.reshape(())
    zp = b2.QTensor(to_dev(zp_raw), x_dt, tuple(s_shape)) if zp_raw is not None else None
    y = b2.DequantizeLinear()(x, s, zp, axis=axis)
    torch.cuda.synchronize()
    return y.cpu().numpy()


def bits(a):
    a = np.ascontiguousarray(a)
    return a.view(np.uint32) if a.dtype == np.float32 else a.view(np.uint16)


@pytest.mark.parametrize("m", META["dq"], ids=lambda m: m["key"])
def test_matches_reference_fixture(b2, cuda, m):
    x, s, zp, y = fixture_dq_inputs(m, Z)
    got = gpu_dq(b2, x, m["x_dt"], m["x_shape"], s, m["s_dt"], m["s_shape"], zp, m["axis"])
    np.testing.assert_array_equal(bits(got).ravel(), bits(y).ravel())


@pytest.mark.parametrize("case", KAT["dequantize_linear"], ids=lambda c: c["src"].split("/")[-1])
def test_known_answers(b2, cuda, case):
    from test_oracle_kat import dq_inputs
    x, s_raw, zp = dq_inputs(case)
    got = gpu_dq(b2, x, case["x_dtype"], case["x_shape"], s_raw, case["scale_dtype"],
                 case["scale_shape"], zp, case["axis"])
    ref = O.dequantize_linear(x, case["x_dtype"], case["x_shape"], s_raw, case["scale_dtype"],
                              case["scale_shape"], zp, case.get("zp_shape"), case["axis"])
    np.testing.assert_array_equal(bits(got), bits(ref))


@pytest.mark.parametrize("dt,s_dt", [(O.INT4, O.FLOAT), (O.INT4, O.FLOAT16), (O.F8E4M3FN, O.FLOAT),
                                     (O.F4E2M1, O.FLOAT), (O.UINT8, O.FLOAT16), (O.INT8, O.FLOAT)])
def test_blocked_weight_sizes_match_oracle(b2, cuda, dt, s_dt):
    # BASELINE config 1 / 5 weight layouts: [K, N] blocked along K.
    K, N, bs = (4096, 4096, 32) if dt == O.INT4 else (1024, 11008, 32)
    x = random_q(1, (K, N), dt)
    s = scale_raw(O.rand_uniform(2, (K // bs * N,), 0.005, 0.02), s_dt)
    zp = random_q(3, (K // bs, N), dt, -2, 2) if dt in (O.INT4, O.INT8) else None
    got = gpu_dq(b2, x, dt, (K, N), s, s_dt, (K // bs, N), zp, 0)
    ref = O.dequantize_linear(x, dt, (K, N), s, s_dt, (K // bs, N), zp,
                              (K // bs, N) if zp is not None else None, 0)
    np.testing.assert_array_equal(bits(got), bits(ref))


@pytest.mark.parametrize("dt", [O.F8E4M3FN, O.F8E4M3FNUZ, O.F8E5M2, O.F8E5M2FNUZ])
@pytest.mark.parametrize("s_dt", [O.FLOAT, O.FLOAT16])
def test_all_float8_codes_including_nan_and_inf(b2, cuda, dt, s_dt):
    x = np.arange(256, dtype=np.uint8)
    s = scale_raw(np.array([0.37], np.float32), s_dt)
    got = gpu_dq(b2, x, dt, (256,), s, s_dt, ())
    ref = O.dequantize_linear(x, dt, (256,), s, s_dt, ())
    np.testing.assert_array_equal(bits(got), bits(ref))


def test_fp16_output_rounding_exhaustive(b2, cuda):
    """Every int8 value times scales that force fp16 subnormals, ties and overflow."""
    x = np.tile(np.arange(-128, 128, dtype=np.int8), 64).view(np.uint8)
    scales = np.concatenate([np.float32(2.0) ** np.arange(-30, 16, dtype=np.float32)[:46],
                             O.rand_uniform(9, (18,), 1e-6, 600.0)])
    s = O.f32_to_f16_bits(scales)  # FLOAT16 scale -> FLOAT16 output
    got = gpu_dq(b2, x, O.INT8, (64, 256), s, O.FLOAT16, (64,), None, 0)
    ref = O.dequantize_linear(x, O.INT8, (64, 256), s, O.FLOAT16, (64,), None, None, 0)
    np.testing.assert_array_equal(bits(got), bits(ref))


def test_empty_and_ragged(b2, cuda):
    for n in (0, 1, 7, 9, 1023):
        x = random_q(n + 5, (n,), O.INT4)
        s = np.array([0.5], np.float32)
        got = gpu_dq(b2, x, O.INT4, (n,), s, O.FLOAT, ())
        ref = O.dequantize_linear(x, O.INT4, (n,), s, O.FLOAT, ())
        np.testing.assert_array_equal(bits(got), bits(ref))


def test_errors_mirror_reference(b2, cuda):
    x = b2.QTensor(to_dev(random_q(1, (4, 6), O.UINT8)), O.UINT8, (4, 6))
    with pytest.raises(ValueError, match="axis out of range"):
        b2.DequantizeLinear()(x, torch.ones(6, device="cuda"), axis=2)
    with pytest.raises(ValueError, match="element count must equal axis dimension"):
        b2.DequantizeLinear()(x, torch.ones(5, device="cuda"), axis=1)
    with pytest.raises(ValueError, match="blocked x_scale dimension must divide"):
        b2.DequantizeLinear()(x, torch.ones((4, 4), device="cuda"), axis=1)
    with pytest.raises(ValueError, match="may only differ from x along the quantization axis"):
        b2.DequantizeLinear()(x, torch.ones((2, 3), device="cuda"), axis=1)
    zp_bad = b2.QTensor(to_dev(np.zeros(6, np.uint8)), O.INT8, (6,))
    with pytest.raises(ValueError, match="x_zero_point data_type must match x"):
        b2.DequantizeLinear()(x, torch.ones(6, device="cuda"), zp_bad, axis=1)
    with pytest.raises(ValueError, match="x_scale must be FLOAT or FLOAT16"):
        b2.DequantizeLinear()(x, torch.ones(6, device="cuda", dtype=torch.float64), axis=1)


def test_cpu_tensor_is_rejected(b2, cuda):
    with pytest.raises(ValueError, match="CUDA"):
        b2.DequantizeLinear()(torch.zeros(4, dtype=torch.uint8), torch.ones(()))
