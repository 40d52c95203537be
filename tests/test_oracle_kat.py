"""The CPU oracle against the known answers written in onnx-light's own tests
(tests/golden/kat_reference_tests.json, each case citing its source lines)."""
import json
import os

import numpy as np
import pytest

import oracle as O
from util import encode_codes

HERE = os.path.dirname(os.path.abspath(__file__))
KAT = json.load(open(os.path.join(HERE, "golden", "kat_reference_tests.json")))


def _x_raw(case, key="x", dtype_key="x_dtype"):
    dt = case[dtype_key]
    vals = case[key]
    if dt == O.F8E4M3FN:
        return O.f32_to_f8e4m3fn(np.array(vals, np.float32))
    if dt == O.F4E2M1:
        table = [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0]
        codes = [next(i for i, t in enumerate(table) if t == v and np.signbit(t) == np.signbit(v)) for v in vals]
        return encode_codes(codes, dt)
    return encode_codes(vals, dt)


def dq_inputs(case):
    x = _x_raw(case)
    s = np.array(case["scale"], np.float32)
    s_raw = s if case["scale_dtype"] == O.FLOAT else O.f32_to_f16_bits(s)
    zp = None
    if case.get("zp") is not None:
        zc = dict(case, x=case["zp"])
        zp = _x_raw(zc)
    return x, s_raw, zp


@pytest.mark.parametrize("case", KAT["dequantize_linear"], ids=lambda c: c["src"].split("/")[-1])
def test_dequantize_linear_kat(case):
    x, s_raw, zp = dq_inputs(case)
    y = O.dequantize_linear(x, case["x_dtype"], case["x_shape"], s_raw, case["scale_dtype"],
                            case["scale_shape"], zp, case.get("zp_shape"), case["axis"])
    if case.get("y_bits") is not None:
        assert y.ravel().tolist() == case["y_bits"]
    elif case.get("y") is not None:
        if case["scale_dtype"] == O.FLOAT16:
            y = O.f16_bits_to_f32(y)
        np.testing.assert_array_equal(y.ravel(), np.array(case["y"], np.float32))
    else:
        # No literal expectation in the source: the case is checked against the
        # reference build in test_oracle_vs_reference.py.
        assert y.shape == tuple(case["x_shape"])


@pytest.mark.parametrize("case", KAT["matmul_integer"], ids=lambda c: c["src"].split("/")[-1])
def test_matmul_integer_kat(case):
    def arr(v, dt):
        return np.array(v, np.int8 if dt == O.INT8 else np.uint8)
    a = arr(case["a"], case["a_dtype"]).reshape(case["a_shape"])
    b = arr(case["b"], case["b_dtype"]).reshape(case["b_shape"])
    azp = arr(case["a_zp"], case["a_dtype"]) if case.get("a_zp") is not None else None
    bzp = arr(case["b_zp"], case["b_dtype"]) if case.get("b_zp") is not None else None
    y = O.matmul_integer(a, case["a_dtype"], b, case["b_dtype"], azp, bzp)
    assert y.ravel().tolist() == case["y"]


def test_f16_conversion_exhaustive_roundtrip():
    bits = np.arange(1 << 16, dtype=np.uint16)
    f = O.f16_bits_to_f32(bits)
    back = O.f32_to_f16_bits(f)
    nan = np.isnan(f)
    np.testing.assert_array_equal(back[~nan], bits[~nan])
    # NaN collapses to sign | 0x7e00 (cast_helper.cc:51-60)
    np.testing.assert_array_equal(back[nan], (bits[nan] & 0x8000) | 0x7e00)
