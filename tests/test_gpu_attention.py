"""Opset-23 Attention on the GPU: against onnx-light's own outputs (fixtures)
and the oracle, GQA, causal, softcap, masks, rank-3 inputs, and the contiguous
KV cache with in-place append.  Tolerance: rel-L2 <= 1e-3 (fp16/bf16)."""
import ctypes as C

import numpy as np
import pytest
import torch

import oracle as O
from util import attention_fixture, load_fixtures, rel_l2, to_dev

pytestmark = pytest.mark.gpu
META, Z = load_fixtures()
TORCH = {O.FLOAT: torch.float32, O.FLOAT16: torch.float16, O.BFLOAT16: torch.bfloat16}
UP = {O.FLOAT: lambda t: t, O.FLOAT16: O.f16_bits_to_f32, O.BFLOAT16: O.bf16_bits_to_f32}
TOL = {O.FLOAT: 1e-5, O.FLOAT16: 1e-3, O.BFLOAT16: 1e-3}


def dev(raw, dt):
    return to_dev(raw).view(TORCH[dt])


def raw(t):
    """A device tensor's storage as numpy (uint16 bits for the half types)."""
    if t.dtype in (torch.float16, torch.bfloat16):
        return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
    return t.contiguous().cpu().numpy()


def as_stored(ref, dt):
    """The oracle's fp32 result rounded to the output type, as the reference
    demotes Y (kernel_attention.cc:819-833): half-precision outputs are compared
    with what onnx-light itself returns, at the contract's rel-L2 1e-3."""
    if dt == O.FLOAT16:
        return O.f16_bits_to_f32(O.f32_to_f16_bits(ref))
    if dt == O.BFLOAT16:
        return O.bf16_bits_to_f32(O.f32_to_bf16_bits(ref))
    return ref


FINITE = [m for m in META["att"] if not m.get("overflow")]


@pytest.mark.parametrize("m", FINITE, ids=lambda m: m["key"])
def test_matches_reference_fixture(b2, cuda, m):
    """Every Attention fixture against onnx-light's own output in its own
    storage type: rel-L2 <= 1e-3 for FLOAT16 / BFLOAT16 Y (both sides rounded
    to the half type), 1e-5 for FLOAT; present bit-exact; qk_matmul_output
    within the same bounds.  Covers BOOL / FLOAT16 / BFLOAT16 masks,
    nonpad_kv_seqlen, v_head_size != head_size, windows, and the tensor-core
    decode and prefill kernels in both half types."""
    f = attention_fixture(m, Z)
    dt = m["dt"]
    q, kk, v = dev(f["q"], dt), dev(f["k"], dt), dev(f["v"], dt)
    attrs = b2.Attributes(is_causal=m["causal"], softcap=m["softcap"], q_num_heads=m["Hq"],
                          kv_num_heads=m["Hkv"], left_window_size=m.get("lw", -1),
                          right_window_size=m.get("rw", -1),
                          qk_matmul_output_mode=m.get("qk") or 0)
    mask = None
    if f["mask"] is not None:
        mask = {O.FLOAT: lambda a: to_dev(a), O.BOOL: lambda a: to_dev(a),
                O.FLOAT16: lambda a: to_dev(a).view(torch.float16),
                O.BFLOAT16: lambda a: to_dev(a).view(torch.bfloat16)}[f["mask_dt"]](f["mask"])
    pk = dev(f["pk"], dt) if m["P"] else None
    pv = dev(f["pv"], dt) if m["P"] else None
    nonpad = to_dev(f["nonpad"]) if f["nonpad"] is not None else None
    r = b2.Attention()(q, kk, v, attrs, mask, pk, pv, nonpad_kv_seqlen=nonpad,
                       qk_matmul_output=f["qk"] is not None)
    torch.cuda.synchronize()
    y = r.Y.float().cpu().numpy()
    ref = UP[dt](f["y"])
    assert rel_l2(y, ref) <= TOL[dt], rel_l2(y, ref)
    if f["qk"] is not None:
        got = r.qk_matmul_output.float().cpu().numpy()
        want = UP[dt](f["qk"])
        fin = np.isfinite(want)
        assert np.array_equal(np.isfinite(got), fin)
        assert np.array_equal(got[~fin], want[~fin])  # -inf where masked
        assert rel_l2(got[fin], want[fin]) <= TOL[dt], rel_l2(got[fin], want[fin])
    if m["P"]:
        assert np.array_equal(raw(r.present_key), f["prk"])
        assert np.array_equal(raw(r.present_value), f["prv"])


def test_overflowing_scores_follow_the_oracle_not_the_rescue(b2, cuda):
    """The documented divergence: onnx-light recomputes a row whose scores
    overflow FLOAT with an extended exponent (RecomputeCenteredAttentionScores,
    kernel_attention.cc:33-158) and returns finite values; the GPU kernels do
    not, and return what the oracle's restatement without the rescue returns
    (NaN for that row).  Rows without overflow agree with both at 1e-5."""
    m = next(m for m in META["att"] if m.get("overflow"))
    f = attention_fixture(m, Z)
    r = b2.Attention()(dev(f["q"], O.FLOAT), dev(f["k"], O.FLOAT), dev(f["v"], O.FLOAT))
    torch.cuda.synchronize()
    y = r.Y.cpu().numpy()
    ora = O.attention_f32(f["q"], f["k"], f["v"])
    ref = f["y"]
    assert np.all(np.isfinite(ref))                     # the reference rescues row 0
    assert np.all(np.isnan(ora[:, :, 0])) and np.all(np.isnan(y[:, :, 0]))
    assert rel_l2(y[:, :, 1], ref[:, :, 1]) <= 1e-5
    assert rel_l2(y[:, :, 1], ora[:, :, 1]) <= 1e-5


def oracle_attention(q16, k16, v16, causal, past_len):
    q, k, v = O.f16_bits_to_f32(q16), O.f16_bits_to_f32(k16), O.f16_bits_to_f32(v16)
    return O.attention_f32(q, k, v, is_causal=causal, past_len=past_len)


@pytest.mark.parametrize("B,Hq,Hkv,P,D", [(4, 32, 8, 511, 128), (3, 8, 8, 100, 64), (2, 16, 2, 2000, 128)])
def test_decode_kv_cache_in_place(b2, cuda, B, Hq, Hkv, P, D):
    rng_q = O.randn(51, (B, Hq, 1, D), 0, 0.5)
    rng_k = O.randn(52, (B, Hkv, P + 2, D), 0, 0.5)
    rng_v = O.randn(53, (B, Hkv, P + 2, D), 0, 0.5)
    q16 = O.f32_to_f16_bits(rng_q)
    k16, v16 = O.f32_to_f16_bits(rng_k), O.f32_to_f16_bits(rng_v)
    cache = b2.KVCache(B, Hkv, P + 8, D, dtype=torch.float16)
    cache.k[:, :, :P] = dev(k16[:, :, :P].copy(), O.FLOAT16)
    cache.v[:, :, :P] = dev(v16[:, :, :P].copy(), O.FLOAT16)
    cache.length = P
    att = b2.Attention()
    attrs = b2.Attributes(is_causal=True)
    for step in range(2):  # two decode steps append in place
        pos = P + step
        r = att(dev(q16, O.FLOAT16), dev(k16[:, :, pos:pos + 1].copy(), O.FLOAT16),
                dev(v16[:, :, pos:pos + 1].copy(), O.FLOAT16), attrs, cache=cache)
        torch.cuda.synchronize()
        ref = oracle_attention(q16, k16[:, :, :pos + 1], v16[:, :, :pos + 1], True, pos)
        assert rel_l2(r.Y.float().cpu().numpy(), ref) <= 1e-3
        assert cache.length == pos + 1
        assert np.array_equal(cache.k[:, :, :pos + 1].cpu().numpy().view(np.uint16), k16[:, :, :pos + 1])


def test_prefill_causal_gqa_rank3(b2, cuda):
    B, S, Hq, Hkv, D = 2, 77, 8, 2, 64
    q = O.f32_to_bf16_bits(O.randn(61, (B, S, Hq * D), 0, 0.5))
    k = O.f32_to_bf16_bits(O.randn(62, (B, S, Hkv * D), 0, 0.5))
    v = O.f32_to_bf16_bits(O.randn(63, (B, S, Hkv * D), 0, 0.5))
    r = b2.Attention()(dev(q, O.BFLOAT16), dev(k, O.BFLOAT16), dev(v, O.BFLOAT16),
                       b2.Attributes(is_causal=True, q_num_heads=Hq, kv_num_heads=Hkv))
    torch.cuda.synchronize()
    up = O.bf16_bits_to_f32
    q4 = up(q).reshape(B, S, Hq, D).transpose(0, 2, 1, 3)
    k4 = up(k).reshape(B, S, Hkv, D).transpose(0, 2, 1, 3)
    v4 = up(v).reshape(B, S, Hkv, D).transpose(0, 2, 1, 3)
    ref = O.attention_f32(q4, k4, v4, is_causal=True).transpose(0, 2, 1, 3).reshape(B, S, Hq * D)
    assert rel_l2(r.Y.float().cpu().numpy(), as_stored(ref, O.BFLOAT16)) <= 1e-3


def test_fully_masked_rows_are_zero(b2, cuda):
    B, H, S, D = 1, 2, 4, 16
    q = dev(O.f32_to_f16_bits(O.randn(71, (B, H, S, D))), O.FLOAT16)
    k = dev(O.f32_to_f16_bits(O.randn(72, (B, H, S, D))), O.FLOAT16)
    v = dev(O.f32_to_f16_bits(O.randn(73, (B, H, S, D))), O.FLOAT16)
    mask = torch.full((S, S), float("-inf"), device="cuda")
    mask[0] = 0.0
    r = b2.Attention()(q, k, v, b2.Attributes(), mask)
    y = r.Y.float().cpu().numpy()
    assert np.all(y[:, :, 1:] == 0.0) and np.any(y[:, :, 0] != 0.0)


def test_errors(b2, cuda):
    q = torch.zeros((1, 6, 1, 16), dtype=torch.float16, device="cuda")
    k = torch.zeros((1, 4, 1, 16), dtype=torch.float16, device="cuda")
    with pytest.raises(ValueError, match="positive multiple of kv_num_heads"):
        b2.Attention()(q, k, k)
    with pytest.raises(ValueError, match="same dtype"):
        b2.Attention()(q, k.float(), k.float())


# ---------------------------------------------------------------------------
# Tensor-core decode kernel (FLOAT16, head 128, one new token, GQA group <= 16).
# ---------------------------------------------------------------------------

def _decode_case(b2, B, Hq, Hkv, P, seed, causal=True, softcap=0.0, cache_extra=8):
    D = 128
    q16 = O.f32_to_f16_bits(O.randn(seed, (B, Hq, 1, D), 0, 0.5))
    k16 = O.f32_to_f16_bits(O.randn(seed + 1, (B, Hkv, P + 1, D), 0, 0.5))
    v16 = O.f32_to_f16_bits(O.randn(seed + 2, (B, Hkv, P + 1, D), 0, 0.5))
    cache = b2.KVCache(B, Hkv, P + 1 + cache_extra, D, dtype=torch.float16)
    # garbage past the valid length must not leak into the result
    cache.k.fill_(float("nan"))
    cache.v.fill_(float("nan"))
    cache.k[:, :, :P] = dev(k16[:, :, :P].copy(), O.FLOAT16)
    cache.v[:, :, :P] = dev(v16[:, :, :P].copy(), O.FLOAT16)
    cache.length = P
    attrs = b2.Attributes(is_causal=causal, softcap=softcap)
    r = b2.Attention()(dev(q16, O.FLOAT16), dev(k16[:, :, P:].copy(), O.FLOAT16),
                       dev(v16[:, :, P:].copy(), O.FLOAT16), attrs, cache=cache)
    torch.cuda.synchronize()
    q, k, v = O.f16_bits_to_f32(q16), O.f16_bits_to_f32(k16), O.f16_bits_to_f32(v16)
    ref = O.attention_f32(q, k, v, is_causal=causal, past_len=P, softcap=softcap)
    return r.Y.float().cpu().numpy(), ref


@pytest.mark.parametrize("B,Hq,Hkv,P", [(32, 32, 8, 4096), (2, 16, 1, 1000), (3, 4, 4, 33),
                                        (1, 8, 2, 0), (5, 12, 3, 31), (2, 8, 8, 700)])
def test_decode_tensor_core_gqa(b2, cuda, B, Hq, Hkv, P):
    y, ref = _decode_case(b2, B, Hq, Hkv, P, seed=70 + P % 7)
    assert rel_l2(y, ref) <= 1e-3, rel_l2(y, ref)


def test_decode_tensor_core_softcap_not_causal(b2, cuda):
    y, ref = _decode_case(b2, 4, 8, 2, 300, seed=81, causal=False, softcap=2.0)
    assert rel_l2(y, ref) <= 1e-3, rel_l2(y, ref)


def test_decode_tensor_core_matches_cuda_core_kernel_and_is_deterministic(b2, cuda, monkeypatch):
    B, Hq, Hkv, P, D = 6, 32, 8, 1500, 128
    q = torch.randn(B, Hq, 1, D, device="cuda").half() * 0.5
    kk = torch.randn(B, Hkv, 1, D, device="cuda").half() * 0.5
    vv = torch.randn(B, Hkv, 1, D, device="cuda").half() * 0.5
    pk = torch.randn(B, Hkv, P, D, device="cuda").half() * 0.5
    pv = torch.randn(B, Hkv, P, D, device="cuda").half() * 0.5
    attrs = b2.Attributes(is_causal=True)
    y1 = b2.Attention()(q, kk, vv, attrs, None, pk, pv).Y.float().cpu().numpy()
    y2 = b2.Attention()(q, kk, vv, attrs, None, pk, pv).Y.float().cpu().numpy()
    monkeypatch.setenv("ONNXL_B200_ATTN_KERNEL", "cuda")
    y3 = b2.Attention()(q, kk, vv, attrs, None, pk, pv).Y.float().cpu().numpy()
    torch.cuda.synchronize()
    assert np.array_equal(y1, y2)
    assert rel_l2(y1, y3) <= 1e-3


# ---------------------------------------------------------------------------
# Tensor-core prefill kernel (FLOAT16 / BFLOAT16, head 128, Sq >= 2, no mask).
# ---------------------------------------------------------------------------

def _prefill_case(b2, dt, B, Hq, Hkv, S, P, causal, rank3, softcap=0.0, seed=90):
    D = 128
    enc = O.f32_to_f16_bits if dt == O.FLOAT16 else O.f32_to_bf16_bits
    q16 = enc(O.randn(seed, (B, Hq, S, D), 0, 0.5))
    k16 = enc(O.randn(seed + 1, (B, Hkv, P + S, D), 0, 0.5))
    v16 = enc(O.randn(seed + 2, (B, Hkv, P + S, D), 0, 0.5))
    attrs = b2.Attributes(is_causal=causal, softcap=softcap, q_num_heads=Hq, kv_num_heads=Hkv)
    if rank3:
        def r3(x):
            return np.ascontiguousarray(x.transpose(0, 2, 1, 3).reshape(B, x.shape[2], -1))
        qd, kd, vd = dev(r3(q16), dt), dev(r3(k16[:, :, P:]), dt), dev(r3(v16[:, :, P:]), dt)
    else:
        qd, kd, vd = dev(q16, dt), dev(k16[:, :, P:].copy(), dt), dev(v16[:, :, P:].copy(), dt)
    pk = dev(k16[:, :, :P].copy(), dt) if P else None
    pv = dev(v16[:, :, :P].copy(), dt) if P else None
    r = b2.Attention()(qd, kd, vd, attrs, None, pk, pv)
    torch.cuda.synchronize()
    y = r.Y.float().cpu().numpy()
    if rank3:
        y = y.reshape(B, S, Hq, D).transpose(0, 2, 1, 3)
    ref = O.attention_f32(UP[dt](q16), UP[dt](k16), UP[dt](v16), is_causal=causal, past_len=P,
                          softcap=softcap)
    return y, as_stored(ref, dt)


PREFILL_TOL = {O.FLOAT16: 1e-3, O.BFLOAT16: 1e-3}


@pytest.mark.parametrize("dt,B,Hq,Hkv,S,P,causal,rank3", [
    (O.FLOAT16, 2, 8, 2, 130, 0, True, False),
    (O.BFLOAT16, 1, 4, 4, 64, 0, True, True),
    (O.FLOAT16, 2, 16, 4, 77, 100, True, False),
    (O.BFLOAT16, 1, 8, 1, 200, 0, False, False),
    (O.FLOAT16, 3, 4, 2, 2, 300, True, False),
    (O.BFLOAT16, 1, 32, 8, 1024, 0, True, True),
    (O.FLOAT16, 1, 8, 8, 65, 63, False, True),
])
def test_prefill_tensor_core(b2, cuda, dt, B, Hq, Hkv, S, P, causal, rank3):
    y, ref = _prefill_case(b2, dt, B, Hq, Hkv, S, P, causal, rank3, seed=90 + S % 11)
    assert rel_l2(y, ref) <= PREFILL_TOL[dt], rel_l2(y, ref)


def test_prefill_tensor_core_softcap(b2, cuda):
    y, ref = _prefill_case(b2, O.FLOAT16, 2, 4, 2, 96, 40, True, False, softcap=3.0, seed=97)
    assert rel_l2(y, ref) <= 1e-3, rel_l2(y, ref)


def test_prefill_tensor_core_kv_cache(b2, cuda):
    """Prefill through a KV cache whose rows past the valid length hold NaN."""
    B, Hq, Hkv, S, P, D = 2, 8, 2, 150, 70, 128
    q16 = O.f32_to_f16_bits(O.randn(101, (B, Hq, S, D), 0, 0.5))
    k16 = O.f32_to_f16_bits(O.randn(102, (B, Hkv, P + S, D), 0, 0.5))
    v16 = O.f32_to_f16_bits(O.randn(103, (B, Hkv, P + S, D), 0, 0.5))
    cache = b2.KVCache(B, Hkv, P + S + 40, D, dtype=torch.float16)
    cache.k.fill_(float("nan"))
    cache.v.fill_(float("nan"))
    cache.k[:, :, :P] = dev(k16[:, :, :P].copy(), O.FLOAT16)
    cache.v[:, :, :P] = dev(v16[:, :, :P].copy(), O.FLOAT16)
    cache.length = P
    r = b2.Attention()(dev(q16, O.FLOAT16), dev(k16[:, :, P:].copy(), O.FLOAT16),
                       dev(v16[:, :, P:].copy(), O.FLOAT16), b2.Attributes(is_causal=True),
                       cache=cache)
    torch.cuda.synchronize()
    ref = oracle_attention(q16, k16, v16, True, P)
    assert rel_l2(r.Y.float().cpu().numpy(), ref) <= 1e-3
    assert cache.length == P + S


def test_prefill_tensor_core_matches_cuda_core_kernel_and_is_deterministic(b2, cuda, monkeypatch):
    B, Hq, Hkv, S, D = 2, 16, 4, 300, 128
    q = torch.randn(B, Hq, S, D, device="cuda").bfloat16() * 0.5
    kk = torch.randn(B, Hkv, S, D, device="cuda").bfloat16() * 0.5
    vv = torch.randn(B, Hkv, S, D, device="cuda").bfloat16() * 0.5
    attrs = b2.Attributes(is_causal=True)
    y1 = b2.Attention()(q, kk, vv, attrs).Y.float().cpu().numpy()
    y2 = b2.Attention()(q, kk, vv, attrs).Y.float().cpu().numpy()
    monkeypatch.setenv("ONNXL_B200_ATTN_KERNEL", "cuda")
    y3 = b2.Attention()(q, kk, vv, attrs).Y.float().cpu().numpy()
    torch.cuda.synchronize()
    assert np.array_equal(y1, y2)
    assert rel_l2(y1, y3) <= 1e-3


@pytest.mark.parametrize("dt,B,Hq,Hkv,S,P,causal,rank3", [
    (O.FLOAT16, 2, 8, 2, 130, 0, True, False),
    (O.BFLOAT16, 1, 8, 1, 200, 0, False, False),
    (O.FLOAT16, 2, 16, 4, 77, 100, True, False),
])
def test_prefill_mma_sync_kernel(b2, cuda, monkeypatch, dt, B, Hq, Hkv, S, P, causal, rank3):
    """The mma.sync prefill kernel (kept beside the tcgen05 one) against the oracle."""
    monkeypatch.setenv("ONNXL_B200_ATTN_KERNEL", "mma")
    y, ref = _prefill_case(b2, dt, B, Hq, Hkv, S, P, causal, rank3, seed=120 + S % 7)
    assert rel_l2(y, ref) <= PREFILL_TOL[dt], rel_l2(y, ref)


def test_prefill_tcgen05_long_causal_gqa(b2, cuda):
    """Many 128-key tiles (re-basing of the running maximum), ragged Sq and L."""
    y, ref = _prefill_case(b2, O.BFLOAT16, 1, 8, 2, 1000, 37, True, True, seed=131)
    assert rel_l2(y, ref) <= PREFILL_TOL[O.BFLOAT16], rel_l2(y, ref)


def test_prefill_tcgen05_matches_mma_sync_and_is_deterministic(b2, cuda, monkeypatch):
    B, Hq, Hkv, S, D = 2, 16, 4, 700, 128
    q = torch.randn(B, Hq, S, D, device="cuda").half() * 0.5
    kk = torch.randn(B, Hkv, S, D, device="cuda").half() * 0.5
    vv = torch.randn(B, Hkv, S, D, device="cuda").half() * 0.5
    attrs = b2.Attributes(is_causal=True)
    y1 = b2.Attention()(q, kk, vv, attrs).Y.float().cpu().numpy()
    y2 = b2.Attention()(q, kk, vv, attrs).Y.float().cpu().numpy()
    monkeypatch.setenv("ONNXL_B200_ATTN_KERNEL", "mma")
    y3 = b2.Attention()(q, kk, vv, attrs).Y.float().cpu().numpy()
    torch.cuda.synchronize()
    assert np.array_equal(y1, y2)
    assert rel_l2(y1, y3) <= 1e-3


# ---------------------------------------------------------------------------
# Bounded waits: a wait that runs out records a code the host reads back.
# ---------------------------------------------------------------------------

def test_bounded_wait_times_out_and_reports(b2, cuda):
    """One kernel thread waits 10 ms on a barrier nothing completes: it gives up,
    records code 1, and the context stays usable for the next call."""
    from onnx_light_b200 import _capi
    lib = _capi.lib()
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.b2_selftest_bounded_wait(10_000_000, C.c_void_p(stream)) == 1
    # the kernels of the tests above finished without any time-out
    assert lib.b2_kernel_status(1) == 0
    x = torch.ones(4, device="cuda")
    assert float((x * 2).sum()) == 8.0
