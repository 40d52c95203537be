"""Config 5 (the prefill block) at its full benchmark shapes, checked on
sampled rows against the oracle.

The block is BFLOAT16 activations [4, 8192, 4096] through causal GQA
Attention (32 query / 8 KV heads, head 128) and the blocked dequant-MatMuls
4096 x 11008 and 11008 x 4096 with FLOAT8E4M3FN or FLOAT4E2M1 weights (block
32 along K, FLOAT scales, Cast to BFLOAT16).  The full oracle product would be
1.5 TFLOP per MatMul on the host, so the GPU computes the whole output and the
oracle recomputes a spread of rows: the first, last and ragged-edge rows of
the 256-row activation tiles and of the grouped rasterization, plus seeded
random rows.  The sampled rows together must meet the contract's rel-L2 1e-3
against the reference semantics (DequantizeLinear, Cast, then MatMul in fp32
with the result rounded to BFLOAT16), and no single row may exceed 4e-3 (a
row of 128 values sees a few BFLOAT16 rounding flips)."""
import numpy as np
import pytest
import torch

import oracle as O
from util import rel_l2, to_dev

pytestmark = pytest.mark.gpu

B, S, HQ, HKV, D = 4, 8192, 32, 8, 128
M, K1, N1 = B * S, 4096, 11008


def sample_rows(n_total, seed, extra=16):
    edges = [0, 1, 255, 256, 257, 8191, 8192, n_total - 257, n_total - 256, n_total - 1]
    rnd = O.randint(seed, (extra,), 0, n_total - 1)
    return np.unique(np.array([r for r in edges if 0 <= r < n_total] + list(rnd), np.int64))


def weights(fmt, K, N, seed):
    """(raw weight bytes, FLOAT scales [K/32, N]) of the benchmark's generators."""
    if fmt == O.F8E4M3FN:
        w = O.f32_to_f8e4m3fn(O.randn(seed, (K * N,), 0.0, 1.0))
        s = O.rand_uniform(seed + 10, (K // 32, N), 0.01, 0.05)
    else:
        w = O.pack_bits(O.randint(seed, (K * N,), 0, 15), 4)
        s = O.rand_uniform(seed + 10, (K // 32, N), 0.05, 0.2)
    return w, s


def oracle_rows(a_rows_bf16, w, fmt, K, N, s):
    wq = O.dequantize_linear(w, fmt, (K, N), s, O.FLOAT, (K // 32, N), None, None, 0)
    wb = O.f32_to_bf16_bits(wq)  # the Cast to BFLOAT16
    return O.bf16_bits_to_f32(O.matmul(a_rows_bf16, wb, O.BFLOAT16))


@pytest.mark.parametrize("fmt", [O.F8E4M3FN, O.F4E2M1], ids=["float8e4m3fn", "float4e2m1"])
def test_config5_dequant_matmuls_full_shape(b2, cuda, fmt):
    a = O.f32_to_bf16_bits(O.randn(5101, (M, K1), 0.0, 0.5))
    w1, s1 = weights(fmt, K1, N1, 5110)
    w2, s2 = weights(fmt, N1, K1, 5120)
    ta = to_dev(a).view(torch.bfloat16)
    mm = b2.DequantizeMatMul()
    h = mm(ta, b2.QTensor(to_dev(w1), fmt, (K1, N1)), to_dev(s1), None, axis=0,
           cast_dtype=torch.bfloat16)
    y = mm(h, b2.QTensor(to_dev(w2), fmt, (N1, K1)), to_dev(s2), None, axis=0,
           cast_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    rows = sample_rows(M, 5130)
    r = torch.from_numpy(rows).cuda()
    h_rows = h.index_select(0, r).view(torch.uint16).cpu().numpy()
    y_rows = y.index_select(0, r).float().cpu().numpy()
    # first MatMul on the sampled rows of A
    ref_h = oracle_rows(a[rows], w1, fmt, K1, N1, s1)
    got_h = O.bf16_bits_to_f32(h_rows)
    assert rel_l2(got_h, ref_h) <= 1e-3, rel_l2(got_h, ref_h)
    # second MatMul on the same rows of the GPU's intermediate
    ref_y = oracle_rows(h_rows, w2, fmt, N1, K1, s2)
    assert rel_l2(y_rows, ref_y) <= 1e-3, rel_l2(y_rows, ref_y)
    # no row may be far off even if the aggregate passes
    per_row = [rel_l2(y_rows[i], ref_y[i]) for i in range(len(rows))]
    assert max(per_row) <= 4e-3, max(per_row)
    assert np.isfinite(y.float().sum().item())


def test_config5_attention_full_shape(b2, cuda):
    """Rank-3 [4, 8192, 4096] causal GQA on the tensor-core prefill kernel;
    sampled (batch, head, position) rows against the oracle, compared after
    rounding to BFLOAT16 as the reference demotes Y."""
    q = O.f32_to_bf16_bits(O.randn(5201, (B, S, HQ * D), 0.0, 0.5))
    k = O.f32_to_bf16_bits(O.randn(5202, (B, S, HKV * D), 0.0, 0.5))
    v = O.f32_to_bf16_bits(O.randn(5203, (B, S, HKV * D), 0.0, 0.5))
    attrs = b2.Attributes(is_causal=True, q_num_heads=HQ, kv_num_heads=HKV)
    r = b2.Attention()(to_dev(q).view(torch.bfloat16), to_dev(k).view(torch.bfloat16),
                       to_dev(v).view(torch.bfloat16), attrs)
    torch.cuda.synchronize()
    y = r.Y
    samples = [(b, h, p) for b in (0, 3) for h in (0, 3, 4, 31)
               for p in (0, 1, 127, 128, 129, 4095, 8190, 8191)]
    rnd = O.randint(5204, (3 * 24,), 0, 1 << 30)
    samples += [(int(rnd[3 * j]) % B, int(rnd[3 * j + 1]) % HQ, int(rnd[3 * j + 2]) % S)
                for j in range(24)]
    up = O.bf16_bits_to_f32
    got_all, ref_all = [], []
    for bb, h, p in samples:
        kvh = h // (HQ // HKV)
        qr = up(q[bb, p, h * D:(h + 1) * D]).reshape(1, 1, 1, D)
        kr = up(k[bb, :p + 1, kvh * D:(kvh + 1) * D]).reshape(1, 1, p + 1, D)
        vr = up(v[bb, :p + 1, kvh * D:(kvh + 1) * D]).reshape(1, 1, p + 1, D)
        ref_all.append(up(O.f32_to_bf16_bits(O.attention_f32(qr, kr, vr).reshape(D))))
        got_all.append(y[bb, p, h * D:(h + 1) * D].float().cpu().numpy())
    got, ref = np.stack(got_all), np.stack(ref_all)
    assert rel_l2(got, ref) <= 1e-3, rel_l2(got, ref)
    worst = max(rel_l2(g, r_) for g, r_ in zip(got_all, ref_all))
    assert worst <= 4e-3, worst
