"""The drop-in end to end on the GPU: ONNX nodes run by onnx-light's own
RunNode (oracle/_ref/libref_runtime.so, compiled from the reference sources)
in a RuntimeContext on Device::kGPU0, resolved through the device-keyed
dispatch table to the KernelBase subclasses of onnx-light_b200/binding, with
device tensors in and out.  Results against the oracle and onnx-light's own
outputs, at the contract's tolerances."""
import numpy as np
import pytest
import torch

import dropin
import oracle as O
from util import load_fixtures, random_q, rel_l2, scale_raw, to_dev

pytestmark = pytest.mark.gpu
META, Z = load_fixtures()


@pytest.fixture(scope="module")
def registered(cuda):
    dropin.lib().h_register(1)
    return True


def dev_in(t, dt, shape):
    return (t.data_ptr(), dt, tuple(shape))


def test_dequantize_linear_node_bit_exact(registered):
    K, N, bs = 256, 96, 32
    x = random_q(7, (K, N), O.INT4)
    s = O.rand_uniform(8, (K // bs, N), 0.005, 0.02)
    z = random_q(9, (K // bs, N), O.INT4, -2, 2)
    ref = O.dequantize_linear(x, O.INT4, (K, N), s, O.FLOAT, (K // bs, N), z, (K // bs, N), 0)
    tx, ts, tz = to_dev(x), to_dev(s), to_dev(z)
    for _ in range(2):  # the kernel object is built once per node; run it twice
        (dt, shape, buf), = dropin.run_node(
            "", "DequantizeLinear",
            [dev_in(tx, O.INT4, (K, N)), dev_in(ts, O.FLOAT, (K // bs, N)),
             dev_in(tz, O.INT4, (K // bs, N))], 1, attrs={"axis": 0}, out_bytes=[K * N * 4])
        assert dt == O.FLOAT and shape == (K, N)
        got = buf[:K * N * 4].cpu().numpy().view(np.uint32)
        assert np.array_equal(got, ref.view(np.uint32).ravel())


def test_matmul_integer_node_bit_exact(registered):
    M, K, N = 64, 256, 192
    a = O.randint(11, (M * K,), 0, 255).astype(np.uint8).reshape(M, K)
    b = O.randint(12, (K * N,), -127, 127).astype(np.int8).reshape(K, N)
    az = np.array([128], np.uint8)
    bz = O.randint(13, (N,), -4, 4).astype(np.int8)
    ref = O.matmul_integer(a, O.UINT8, b, O.INT8, az, bz)
    ta, tb, taz, tbz = to_dev(a), to_dev(b), to_dev(az.reshape(())), to_dev(bz)
    (dt, shape, buf), = dropin.run_node(
        "", "MatMulInteger",
        [dev_in(ta, O.UINT8, (M, K)), dev_in(tb, O.INT8, (K, N)), dev_in(taz, O.UINT8, ()),
         dev_in(tbz, O.INT8, (N,))], 1, out_bytes=[M * N * 4])
    assert dt == O.INT32 and shape == (M, N)
    assert np.array_equal(buf[:M * N * 4].cpu().numpy().view(np.int32).reshape(M, N), ref)


def test_qlinear_matmul_node_matches_reference_fixture(registered):
    m = META["qlm"][-1]
    k = m["key"]
    a, b = Z[k + "_a"], Z[k + "_b"]
    sc, zp = m["sc"], m["zp"]
    dt, ydt = m["dt"], m["ydt"]
    np_t = np.int8 if dt == O.INT8 else np.uint8
    ynp = np.int8 if ydt == O.INT8 else np.uint8
    ins = [to_dev(a), to_dev(np.array(sc[0], np.float32)), to_dev(np.array(zp[0], np_t)),
           to_dev(b), to_dev(np.array(sc[1], np.float32)), to_dev(np.array(zp[1], np_t)),
           to_dev(np.array(sc[2], np.float32)), to_dev(np.array(zp[2], ynp))]
    dts = [dt, O.FLOAT, dt, dt, O.FLOAT, dt, O.FLOAT, ydt]
    shapes = [a.shape, (), (), b.shape, (), (), (), ()]
    n_out = int(np.prod(Z[k + "_y"].shape))
    (odt, shape, buf), = dropin.run_node("", "QLinearMatMul",
                                         [dev_in(t, d, s) for t, d, s in zip(ins, dts, shapes)], 1,
                                         out_bytes=[n_out])
    assert odt == ydt
    assert np.array_equal(buf[:n_out].cpu().numpy(), Z[k + "_y"].ravel())


def test_attention_node_with_past_and_all_outputs(registered):
    m = META["att"][0]  # fp16 GQA decode, past 37, head 64
    k = m["key"]
    B, Hq, Hkv, Sq, P, D = m["B"], m["Hq"], m["Hkv"], m["Sq"], m["P"], m["D"]
    q, kk, v, pk, pv = (to_dev(Z[k + s]) for s in ("_q", "_k", "_v", "_pk", "_pv"))
    L = P + Sq
    outs = dropin.run_node(
        "", "Attention",
        [dev_in(q, O.FLOAT16, (B, Hq, Sq, D)), dev_in(kk, O.FLOAT16, (B, Hkv, Sq, D)),
         dev_in(v, O.FLOAT16, (B, Hkv, Sq, D)), None, dev_in(pk, O.FLOAT16, (B, Hkv, P, D)),
         dev_in(pv, O.FLOAT16, (B, Hkv, P, D))], 4, attrs={"is_causal": 1, "qk_matmul_output_mode": 0},
        out_bytes=[B * Hq * Sq * D * 2, B * Hkv * L * D * 2, B * Hkv * L * D * 2, B * Hq * Sq * L * 2])
    (ydt, ysh, yb), (kdt, ksh, kb), (vdt, vsh, vb), (qdt, qsh, qb) = outs
    assert ysh == (B, Hq, Sq, D) and ksh == (B, Hkv, L, D) and qsh == (B, Hq, Sq, L)
    y = O.f16_bits_to_f32(yb[:B * Hq * Sq * D * 2].cpu().numpy().view(np.uint16))
    assert rel_l2(y, O.f16_bits_to_f32(Z[k + "_y"]).ravel()) <= 1e-3
    assert np.array_equal(kb[:B * Hkv * L * D * 2].cpu().numpy().view(np.uint16), Z[k + "_prk"].ravel())
    assert np.array_equal(vb[:B * Hkv * L * D * 2].cpu().numpy().view(np.uint16), Z[k + "_prv"].ravel())
    # qk_matmul_output mode 0: the scaled scores, against the oracle
    up = O.f16_bits_to_f32
    kc = np.concatenate([up(Z[k + "_pk"]), up(Z[k + "_k"])], 2)
    vc = np.concatenate([up(Z[k + "_pv"]), up(Z[k + "_v"])], 2)
    _, qk_ref = O.attention_f32(up(Z[k + "_q"]), kc, vc, is_causal=True, past_len=P, qk_mode=0)
    qk = up(qb[:B * Hq * Sq * L * 2].cpu().numpy().view(np.uint16))
    assert rel_l2(qk, qk_ref.ravel()) <= 1e-3


def test_fused_dequantize_matmul_node(registered):
    K, N, M = 512, 256, 3
    w = random_q(21, (K, N), O.INT4)
    s = scale_raw(O.rand_uniform(22, (K // 128 * N,), 0.002, 0.02), O.FLOAT16)
    a = O.f32_to_f16_bits(O.randn(23, (M, K)))
    wq = O.dequantize_linear(w, O.INT4, (K, N), s, O.FLOAT16, (K // 128, N), None, None, 0)
    ref = O.f16_bits_to_f32(O.matmul(a, wq, O.FLOAT16))
    tw, ts, ta = to_dev(w), to_dev(s), to_dev(a)
    (dt, shape, buf), = dropin.run_node(
        "b200", "DequantizeMatMul",
        [dev_in(ta, O.FLOAT16, (M, K)), dev_in(tw, O.INT4, (K, N)),
         dev_in(ts, O.FLOAT16, (K // 128, N))], 1, attrs={"axis": 0}, out_bytes=[M * N * 2])
    assert dt == O.FLOAT16 and shape == (M, N)
    got = O.f16_bits_to_f32(buf[:M * N * 2].cpu().numpy().view(np.uint16)).reshape(M, N)
    assert rel_l2(got, ref) <= 1e-3


def test_invalid_node_raises_reference_style_error(registered):
    x = torch.zeros(16, dtype=torch.uint8, device="cuda")
    s = torch.ones(3, dtype=torch.float32, device="cuda")
    with pytest.raises(dropin.NodeError, match="kernel::DequantizeLinear"):
        dropin.run_node("", "DequantizeLinear",
                        [dev_in(x, O.UINT8, (4, 4)), dev_in(s, O.FLOAT, (3,))], 1,
                        attrs={"axis": 0}, out_bytes=[64])


def test_rms_normalization_node_bit_exact(registered):
    m = next(m for m in META["dec"] if m["op"] == "RMSNormalization" and m["dt"] == O.FLOAT16)
    k = m["key"]
    x, s = to_dev(Z[k + "_x"]), to_dev(np.ascontiguousarray(Z[k + "_s"]))
    xs = Z[k + "_x"].shape
    (dt, shape, buf), = dropin.run_node(
        "", "RMSNormalization", [dev_in(x, O.FLOAT16, xs), dev_in(s, O.FLOAT16, Z[k + "_s"].shape)], 1,
        attrs={"axis": m["axis"], "epsilon": float(m["eps"])}, out_bytes=[Z[k + "_y"].nbytes])
    assert dt == O.FLOAT16 and shape == xs
    assert np.array_equal(buf[:Z[k + "_y"].nbytes].cpu().numpy().view(np.uint16), Z[k + "_y"].ravel())
