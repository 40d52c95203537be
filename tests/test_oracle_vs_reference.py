"""Pins the CPU oracle (oracle/oracle.c) to onnx-light's own kernels.

Always: against tests/golden/ref_fixtures.npz, which the reference kernels
produced (tests/golden/make_golden.py).  When oracle/_ref/libref.so is built
(only where the reference tree exists), also against the live reference on
fresh seeds."""
import numpy as np
import pytest

import oracle as O
from util import (CODE_RANGE, attention_fixture, encode_codes, fixture_dq_inputs, load_fixtures,
                  np_int, rel_l2, scale_raw)

META, Z = load_fixtures()


def _bits(a):
    a = np.ascontiguousarray(a)
    return a.view(np.uint32) if a.dtype == np.float32 else a.view(np.uint16)


@pytest.mark.parametrize("m", META["dq"], ids=lambda m: m["key"])
def test_dequantize_linear_matches_reference_fixture(m):
    x, s, zp, y = fixture_dq_inputs(m, Z)
    got = O.dequantize_linear(x, m["x_dt"], m["x_shape"], s, m["s_dt"], m["s_shape"], zp,
                              m["s_shape"] if m["zp"] else None, m["axis"])
    np.testing.assert_array_equal(_bits(got).ravel(), _bits(y).ravel())


@pytest.mark.parametrize("m", META["mmi"], ids=lambda m: m["key"])
def test_matmul_integer_matches_reference_fixture(m):
    k = m["key"]
    a = np_int(Z[k + "_a"], m["a_dt"]).reshape(m["a_shape"])
    b = np_int(Z[k + "_b"], m["b_dt"]).reshape(m["b_shape"])
    az = np_int(Z[k + "_az"], m["a_dt"]) if m["az"] else None
    bz = np_int(Z[k + "_bz"], m["b_dt"]) if m["bz"] else None
    got = O.matmul_integer(a, m["a_dt"], b, m["b_dt"], az, bz)
    np.testing.assert_array_equal(got, Z[k + "_y"])


@pytest.mark.parametrize("m", META["qlm"], ids=lambda m: m["key"])
def test_qlinear_matmul_matches_reference_fixture(m):
    k = m["key"]
    a = np_int(Z[k + "_a"], m["dt"]).reshape(m["a_shape"])
    b = np_int(Z[k + "_b"], m["dt"]).reshape(m["b_shape"])
    sc = [float(v) for v in m["sc"]]
    if m["s_dt"] == O.FLOAT16:  # the reference reads FLOAT16 scales as fp16 values
        sc = [float(O.f16_bits_to_f32(O.f32_to_f16_bits(np.array([v], np.float32)))[0]) for v in sc]
    sc = [float(np.float32(v)) for v in sc]
    got = O.qlinear_matmul(a, m["dt"], sc[0], m["zp"][0], b, m["dt"], sc[1], m["zp"][1], sc[2],
                           m["zp"][2], m["ydt"])
    np.testing.assert_array_equal(got.view(np.uint8).ravel(), Z[k + "_y"].ravel())


@pytest.mark.parametrize("m", META["mm"], ids=lambda m: m["key"])
def test_matmul_matches_reference_fixture(m):
    k = m["key"]
    got = O.matmul(Z[k + "_a"], Z[k + "_b"], m["dt"])
    np.testing.assert_array_equal(got, Z[k + "_y"])


@pytest.mark.parametrize("m", [m for m in META["att"] if not m.get("overflow")],
                         ids=lambda m: m["key"])
def test_attention_matches_reference_fixture(m):
    f = attention_fixture(m, Z)
    up = {O.FLOAT: lambda t: t, O.FLOAT16: O.f16_bits_to_f32, O.BFLOAT16: O.bf16_bits_to_f32}[m["dt"]]
    q, kk, v = up(f["q"]), up(f["k"]), up(f["v"])
    B, Hq, Hkv, Sq, P, D = m["B"], m["Hq"], m["Hkv"], m["Sq"], m["P"], m["D"]
    Sk, Dv = m.get("Sk", Sq), m.get("Dv", D)
    if m["rank"] == 3:
        q = q.reshape(B, Sq, Hq, D).transpose(0, 2, 1, 3)
        kk = kk.reshape(B, Sk, Hkv, D).transpose(0, 2, 1, 3)
        v = v.reshape(B, Sk, Hkv, Dv).transpose(0, 2, 1, 3)
    if P:
        kk = np.concatenate([up(f["pk"]), kk], 2)
        v = np.concatenate([up(f["pv"]), v], 2)
    mask = f["mask"]
    if mask is not None and f["mask_dt"] == O.FLOAT16:
        mask = O.f16_bits_to_f32(mask)
    elif mask is not None and f["mask_dt"] == O.BFLOAT16:
        mask = ("bf16", mask)
    out = O.attention_f32(q, kk, v, is_causal=m["causal"], past_len=P, softcap=m["softcap"],
                          mask=mask, left_window=m.get("lw", -1), right_window=m.get("rw", -1),
                          nonpad=f["nonpad"], qk_mode=m.get("qk"))
    y, qk = (out, None) if m.get("qk") is None else out
    if m["rank"] == 3:
        y = y.transpose(0, 2, 1, 3).reshape(B, Sq, Hq * Dv)
    ref = up(f["y"])
    if m["dt"] == O.FLOAT:
        np.testing.assert_allclose(y, ref, rtol=1e-5, atol=1e-6)
        if qk is not None:
            np.testing.assert_allclose(qk, f["qk"], rtol=1e-5, atol=1e-6)
    else:
        # the reference demotes Y to the input type; round the oracle the same way
        dn = O.f32_to_f16_bits if m["dt"] == O.FLOAT16 else O.f32_to_bf16_bits
        np.testing.assert_allclose(up(dn(y)), ref, rtol=1e-2, atol=2e-3)
        assert rel_l2(up(dn(y)), ref) <= 1e-3
        if qk is not None:
            fin = np.isfinite(up(f["qk"]))
            np.testing.assert_array_equal(fin, np.isfinite(qk))
            np.testing.assert_allclose(up(dn(qk))[fin], up(f["qk"])[fin], rtol=1e-2, atol=2e-3)
    if P:
        np.testing.assert_array_equal(f["prk"][:, :, :P], f["pk"])


def test_attention_overflow_is_the_documented_divergence():
    """Scores that overflow FLOAT: the reference rescues the row (finite
    output, kernel_attention.cc:33-158); the restatement, like the GPU
    kernels, does not (NaN); the other row agrees."""
    m = next(m for m in META["att"] if m.get("overflow"))
    f = attention_fixture(m, Z)
    y = O.attention_f32(f["q"], f["k"], f["v"])
    assert np.all(np.isfinite(f["y"])) and np.all(np.isnan(y[:, :, 0]))
    np.testing.assert_allclose(y[:, :, 1], f["y"][:, :, 1], rtol=1e-5, atol=1e-6)


live = pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built (no reference tree)")


@live
@pytest.mark.parametrize("seed", range(5))
def test_live_dequantize_int4_blocked(seed):
    K, N, bs = 256, 96, 32
    x = encode_codes(O.randint(seed * 7 + 1, (K * N,), -8, 7), O.INT4)
    s = O.rand_uniform(seed * 7 + 2, (K // bs, N), 0.005, 0.02)
    zp = encode_codes(O.randint(seed * 7 + 3, (K // bs * N,), -2, 2), O.INT4)
    a = O.dequantize_linear(x, O.INT4, (K, N), s, O.FLOAT, (K // bs, N), zp, (K // bs, N), 0)
    b = O.ref_dequantize_linear(x, O.INT4, (K, N), s, O.FLOAT, (K // bs, N), zp, (K // bs, N), 0)
    np.testing.assert_array_equal(_bits(a), _bits(b))


@live
def test_live_f8e4m3fn_encoder_matches_reference():
    x = np.concatenate([np.linspace(-500, 500, 20001, dtype=np.float32), O.randn(3, (20000,)),
                        O.randn(4, (20000,)) * np.float32(0.003),
                        np.array([np.inf, -np.inf, np.nan, 0.0, -0.0, 448.0, 464.0, -464.0], np.float32)])
    mine = O.f32_to_f8e4m3fn(x)
    ref = np.array([O.ref().ref_f32_to_f8e4m3fn(float(v)) for v in x], np.uint8)
    np.testing.assert_array_equal(mine, ref)


@live
@pytest.mark.parametrize("dt", [O.FLOAT, O.FLOAT16, O.BFLOAT16])
def test_live_matmul(dt):
    a = O.randn(11, (4, 33, 70))
    b = O.randn(12, (70, 45))
    if dt == O.FLOAT16:
        a, b = O.f32_to_f16_bits(a), O.f32_to_f16_bits(b)
    elif dt == O.BFLOAT16:
        a, b = O.f32_to_bf16_bits(a), O.f32_to_bf16_bits(b)
    np.testing.assert_array_equal(O.matmul(a, b, dt), O.ref_matmul(a, b, dt))


@live
def test_live_matmul_integer_config2_slice():
    # BASELINE config 2 inputs on a K-complete slice: A uint8 zp 128, B int8 per-column zp.
    a = encode_codes(O.randint(2001, (8 * 4096,), 0, 255), O.UINT8).reshape(8, 4096)
    b = encode_codes(O.randint(2002, (4096 * 64,), -127, 127), O.INT8).view(np.int8).reshape(4096, 64)
    bz = encode_codes(O.randint(2003, (64,), -4, 4), O.INT8).view(np.int8)
    az = np.array([128], np.uint8)
    got = O.matmul_integer(a, O.UINT8, b, O.INT8, az, bz)
    ref = O.ref_matmul_integer(a, O.UINT8, b, O.INT8, az, bz, a_zp_shape=[], b_zp_shape=[64])
    np.testing.assert_array_equal(got, ref)


@pytest.mark.parametrize("m", META["dec"], ids=lambda m: m["key"])
def test_decoder_ops_match_reference_fixture(m):
    """RMSNormalization, RotaryEmbedding and SwiGLU: the restatement is
    bit-exact with onnx-light's own output."""
    k, dt = m["key"], m["dt"]
    if m["op"] == "RMSNormalization":
        y = O.rms_normalization(Z[k + "_x"], Z[k + "_s"], dt, m["axis"], m["eps"])
    elif m["op"] == "RotaryEmbedding":
        y = O.rotary_embedding(Z[k + "_x"], Z[k + "_c"], Z[k + "_s"], dt,
                               Z[k + "_p"] if m["pos"] else None, m["interleaved"], m["rdim"],
                               m["num_heads"])
    else:
        y = O.swiglu(Z[k + "_a"], Z[k + "_b"], dt, m["alpha"])
    np.testing.assert_array_equal(np.asarray(y).view(np.uint8), Z[k + "_y"].view(np.uint8))
