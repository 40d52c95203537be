"""MatMulInteger and QLinearMatMul on the GPU: bit-exact against onnx-light's
own outputs, its known answers, and the oracle; BASELINE config 2 at full size
through exact fp64 products on a row slice plus the oracle on a sub-block."""
import json
import os

import numpy as np
import pytest
import torch

import oracle as O
from util import encode_codes, load_fixtures, np_int, to_dev

pytestmark = pytest.mark.gpu
META, Z = load_fixtures()
HERE = os.path.dirname(os.path.abspath(__file__))
KAT = json.load(open(os.path.join(HERE, "golden", "kat_reference_tests.json")))
TD = {O.INT8: torch.int8, O.UINT8: torch.uint8}


def dev(raw, dt, shape):
    return to_dev(np.ascontiguousarray(raw).view(np.uint8)).view(TD[dt]).reshape(tuple(shape))


@pytest.mark.parametrize("m", META["mmi"], ids=lambda m: m["key"])
def test_matmul_integer_fixture(b2, cuda, m):
    k = m["key"]
    a = dev(Z[k + "_a"], m["a_dt"], m["a_shape"])
    b = dev(Z[k + "_b"], m["b_dt"], m["b_shape"])
    az = dev(Z[k + "_az"], m["a_dt"], Z[k + "_az"].shape) if m["az"] else None
    bz = dev(Z[k + "_bz"], m["b_dt"], Z[k + "_bz"].shape) if m["bz"] else None
    y = b2.MatMulInteger()(a, b, az, bz)
    np.testing.assert_array_equal(y.cpu().numpy(), Z[k + "_y"])


@pytest.mark.parametrize("case", KAT["matmul_integer"], ids=lambda c: c["src"].split("/")[-1])
def test_matmul_integer_known_answers(b2, cuda, case):
    npdt = lambda dt: np.int8 if dt == O.INT8 else np.uint8  # noqa: E731
    a = dev(np.array(case["a"], npdt(case["a_dtype"])), case["a_dtype"], case["a_shape"])
    b = dev(np.array(case["b"], npdt(case["b_dtype"])), case["b_dtype"], case["b_shape"])
    az = (dev(np.array(case["a_zp"], npdt(case["a_dtype"])), case["a_dtype"], case.get("a_zp_shape") or [])
          if case.get("a_zp") is not None else None)
    bz = (dev(np.array(case["b_zp"], npdt(case["b_dtype"])), case["b_dtype"], case.get("b_zp_shape") or [])
          if case.get("b_zp") is not None else None)
    y = b2.MatMulInteger()(a, b, az, bz)
    assert y.cpu().numpy().ravel().tolist() == case["y"]


@pytest.mark.parametrize("m", META["qlm"], ids=lambda m: m["key"])
def test_qlinear_matmul_fixture(b2, cuda, m):
    k = m["key"]
    a = dev(Z[k + "_a"], m["dt"], m["a_shape"])
    b = dev(Z[k + "_b"], m["dt"], m["b_shape"])
    sdt = torch.float32 if m["s_dt"] == O.FLOAT else torch.float16
    sc = [torch.tensor(v, dtype=sdt, device="cuda") for v in m["sc"]]
    zp = [torch.tensor(v, dtype=TD[d], device="cuda") for v, d in zip(m["zp"], (m["dt"], m["dt"], m["ydt"]))]
    y = b2.QLinearMatMul()(a, sc[0], zp[0], b, sc[1], zp[1], sc[2], zp[2])
    np.testing.assert_array_equal(y.cpu().numpy().view(np.uint8).ravel(), Z[k + "_y"].ravel())


def test_qlinear_matmul_rejects_zero_y_scale(b2, cuda):
    a = torch.ones((2, 3), dtype=torch.uint8, device="cuda")
    b = torch.ones((3, 2), dtype=torch.uint8, device="cuda")
    one = torch.tensor(1.0, device="cuda")
    z = torch.tensor(0, dtype=torch.uint8, device="cuda")
    with pytest.raises(ValueError, match="y_scale must be non-zero"):
        b2.QLinearMatMul()(a, one, z, b, one, z, torch.tensor(0.0, device="cuda"), z)


@pytest.mark.parametrize("M,K,N", [(512, 4096, 11008), (256, 1024, 768), (130, 4097, 129)])
def test_config2_shapes(b2, cuda, M, K, N):
    # uint8 A zp 128, int8 B with per-column zp in [-4, 4].
    a_np = encode_codes(O.randint(3001, (M * K,), 0, 255), O.UINT8).reshape(M, K)
    b_np = encode_codes(O.randint(3002, (K * N,), -127, 127), O.INT8).view(np.int8).reshape(K, N)
    bz_np = encode_codes(O.randint(3003, (N,), -4, 4), O.INT8).view(np.int8)
    a, b = dev(a_np, O.UINT8, (M, K)), dev(b_np, O.INT8, (K, N))
    az = torch.tensor(128, dtype=torch.uint8, device="cuda")
    bz = dev(bz_np, O.INT8, (N,))
    y = b2.MatMulInteger()(a, b, az, bz)
    # exact reference: fp64 products of int32 values are exact below 2^53
    ref = ((a.double() - 128.0) @ (b.double() - bz.double()[None, :])).round().long()
    assert torch.equal(y.long(), ref)
    # oracle bit-exactness on a sub-block of rows
    rows = slice(0, 4)
    o = O.matmul_integer(a_np[rows], O.UINT8, b_np, O.INT8, np.array([128], np.uint8), bz_np)
    np.testing.assert_array_equal(y[rows].cpu().numpy(), o)


def test_int32_wraparound_matches_reference(b2, cuda):
    # K large enough that the int32 accumulator wraps, as the reference's does.
    M, K, N = 2, 40000, 3
    a_np = np.full((M, K), 255, np.uint8)
    b_np = np.full((K, N), 255, np.uint8)
    y = b2.MatMulInteger()(dev(a_np, O.UINT8, (M, K)), dev(b_np, O.UINT8, (K, N)))
    o = O.matmul_integer(a_np, O.UINT8, b_np, O.UINT8)
    np.testing.assert_array_equal(y.cpu().numpy(), o)


@pytest.mark.parametrize("M,K,N,adt,bdt,az,bz", [
    (128, 256, 256, O.UINT8, O.INT8, "scalar128", "col"),
    (200, 512, 272, O.UINT8, O.UINT8, "row", "scalar"),
    (64, 128, 128, O.INT8, O.INT8, "scalar", "col"),
    (300, 4096, 1024, O.UINT8, O.INT8, "scalar128", "col"),
])
def test_tensor_core_matmul_integer_vs_oracle(b2, cuda, M, K, N, adt, bdt, az, bz):
    a_np = encode_codes(O.randint(4001 + M, (M * K,), *(0, 255) if adt == O.UINT8 else (-128, 127)), adt).reshape(M, K)
    b_np = encode_codes(O.randint(4002 + N, (K * N,), *(0, 255) if bdt == O.UINT8 else (-128, 127)), bdt).reshape(K, N)
    azn = {"scalar128": np.array([128]), "scalar": np.array([-3]), "row": O.randint(7, (M,), 100, 140)}[az]
    bzn = {"col": O.randint(8, (N,), -4, 4) if bdt == O.INT8 else O.randint(8, (N,), 120, 130),
           "scalar": np.array([125])}[bz]
    azr = encode_codes(azn, adt)
    bzr = encode_codes(bzn, bdt)
    a, b = dev(a_np, adt, (M, K)), dev(b_np, bdt, (K, N))
    azt = dev(azr, adt, (azr.size,)) if azr.size > 1 else dev(azr, adt, ())
    bzt = dev(bzr, bdt, (bzr.size,)) if bzr.size > 1 else dev(bzr, bdt, ())
    y = b2.MatMulInteger()(a, b, azt, bzt)
    o = O.matmul_integer(np_int(a_np, adt), adt, np_int(b_np, bdt), bdt, np_int(azr, adt), np_int(bzr, bdt))
    np.testing.assert_array_equal(y.cpu().numpy(), o)


def test_tensor_core_qlinear_matmul_vs_oracle(b2, cuda):
    M, K, N = 256, 1024, 512
    a_np = encode_codes(O.randint(5001, (M * K,), 0, 255), O.UINT8).reshape(M, K)
    b_np = encode_codes(O.randint(5002, (K * N,), 0, 255), O.UINT8).reshape(K, N)
    sc = (0.0066, 0.00705, 0.0107 * 40)
    zp = (113, 114, 118)
    a, b = dev(a_np, O.UINT8, (M, K)), dev(b_np, O.UINT8, (K, N))
    s = [torch.tensor(v, dtype=torch.float32, device="cuda") for v in sc]
    z = [torch.tensor(v, dtype=torch.uint8, device="cuda") for v in zp]
    y = b2.QLinearMatMul()(a, s[0], z[0], b, s[1], z[1], s[2], z[2])
    o = O.qlinear_matmul(a_np, O.UINT8, float(np.float32(sc[0])), zp[0], b_np, O.UINT8,
                         float(np.float32(sc[1])), zp[1], float(np.float32(sc[2])), zp[2], O.UINT8)
    np.testing.assert_array_equal(y.cpu().numpy(), o)
