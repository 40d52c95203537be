"""RMSNormalization, RotaryEmbedding and SwiGLU on the GPU against onnx-light's
own outputs (fixtures) and the oracle.  RMSNormalization and RotaryEmbedding
are bit-exact; SwiGLU calls CUDA's expf (within 2 ulps of the host library),
so FLOAT is held to rel-L2 1e-6 and the half types to the 1e-3 contract."""
import ctypes as C

import numpy as np
import pytest
import torch

import oracle as O
from util import load_fixtures, rel_l2, to_dev

pytestmark = pytest.mark.gpu
META, Z = load_fixtures()
TORCH = {O.FLOAT: torch.float32, O.FLOAT16: torch.float16, O.BFLOAT16: torch.bfloat16}
UP = {O.FLOAT: lambda t: t, O.FLOAT16: O.f16_bits_to_f32, O.BFLOAT16: O.bf16_bits_to_f32}


def dev(raw, dt):
    return to_dev(np.ascontiguousarray(raw)).view(TORCH[dt])


def raw(t):
    if t.dtype in (torch.float16, torch.bfloat16):
        return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
    return t.contiguous().cpu().numpy()


@pytest.mark.parametrize("m", META["dec"], ids=lambda m: m["key"])
def test_decoder_ops_match_reference_fixture(b2, cuda, m):
    k, dt = m["key"], m["dt"]
    if m["op"] == "RMSNormalization":
        y = b2.RMSNormalization()(dev(Z[k + "_x"], dt), dev(Z[k + "_s"], dt), m["axis"], m["eps"])
    elif m["op"] == "RotaryEmbedding":
        pos = to_dev(Z[k + "_p"]) if m["pos"] else None
        y = b2.RotaryEmbedding()(dev(Z[k + "_x"], dt), dev(Z[k + "_c"], dt), dev(Z[k + "_s"], dt),
                                 pos, m["interleaved"], m["rdim"], m["num_heads"])
    else:
        y = b2.SwiGLU()(dev(Z[k + "_a"], dt), dev(Z[k + "_b"], dt), m["alpha"])
    torch.cuda.synchronize()
    got, want = raw(y), Z[k + "_y"]
    if m["op"] != "SwiGLU":
        assert np.array_equal(got.view(np.uint8), want.view(np.uint8))
    else:
        tol = 1e-6 if dt == O.FLOAT else 1e-3
        assert rel_l2(UP[dt](got), UP[dt](want)) <= tol
        # most elements identical (FLOAT: about 89 % measured, the rest 1 ulp apart)
        assert np.mean(got == want) > (0.8 if dt == O.FLOAT else 0.9)


def test_llama_shapes_against_oracle(b2, cuda):
    """A Llama-7B decode step's shapes: RMSNorm over 4096, rotary on 32 heads of
    128 at positions 0..4095 by position_ids, SwiGLU over 11008."""
    B = 8
    x = O.f32_to_f16_bits(O.randn(901, (B, 1, 4096)))
    g = O.f32_to_f16_bits(O.rand_uniform(902, (4096,), 0.5, 1.5))
    y = b2.RMSNormalization()(dev(x, O.FLOAT16), dev(g, O.FLOAT16))
    torch.cuda.synchronize()
    assert np.array_equal(raw(y), O.rms_normalization(x, g, O.FLOAT16))
    q = O.f32_to_f16_bits(O.randn(903, (B, 1, 32 * 128)))
    pos = O.randint(904, (B,), 0, 4095).reshape(B, 1)
    inv = 1.0 / (10000.0 ** (np.arange(0, 128, 2, dtype=np.float64) / 128))
    ang = np.arange(4096)[:, None] * inv[None, :]
    cos = O.f32_to_f16_bits(np.cos(ang).astype(np.float32))
    sin = O.f32_to_f16_bits(np.sin(ang).astype(np.float32))
    r = b2.RotaryEmbedding()(dev(q, O.FLOAT16), dev(cos, O.FLOAT16), dev(sin, O.FLOAT16),
                             to_dev(pos), num_heads=32)
    torch.cuda.synchronize()
    assert np.array_equal(raw(r), O.rotary_embedding(q, cos, sin, O.FLOAT16, pos, num_heads=32))
    a = O.f32_to_f16_bits(O.randn(905, (B, 11008)))
    b = O.f32_to_f16_bits(O.randn(906, (B, 11008)))
    s = b2.SwiGLU()(dev(a, O.FLOAT16), dev(b, O.FLOAT16))
    torch.cuda.synchronize()
    assert rel_l2(O.f16_bits_to_f32(raw(s)), O.f16_bits_to_f32(O.swiglu(a, b, O.FLOAT16))) <= 1e-3


def test_rotary_position_out_of_range_is_reported(b2, cuda):
    from onnx_light_b200 import _capi
    lib = _capi.lib()
    assert lib.b2_kernel_status(1) == 0
    x = torch.ones((1, 1, 2, 8), dtype=torch.float32, device="cuda")
    c = torch.ones((4, 4), dtype=torch.float32, device="cuda")
    pos = torch.tensor([[1, 9]], dtype=torch.int64, device="cuda")  # 9 is past the 4-row cache
    y = b2.RotaryEmbedding()(x, c, c, pos)
    torch.cuda.synchronize()
    assert lib.b2_kernel_status(0) == 4
    buf = C.create_string_buffer(256)
    lib.b2_last_error(buf, 256)
    assert b"position_ids value out of range" in buf.value
    assert lib.b2_kernel_status(1) == 4 and lib.b2_kernel_status(0) == 0
    assert torch.all(y[0, 0, 1] == 0)                # the out-of-range row is zeros
    assert torch.equal(y[0, 0, 0].cpu(), torch.tensor([0.0] * 4 + [2.0] * 4))  # c x1 - s x2, s x1 + c x2


def test_errors(b2, cuda):
    x = torch.zeros((2, 8), dtype=torch.float32, device="cuda")
    with pytest.raises(ValueError, match="scale must have the same dtype"):
        b2.RMSNormalization()(x, torch.zeros(8, dtype=torch.float16, device="cuda"))
    with pytest.raises(ValueError, match="identical shapes"):
        b2.SwiGLU()(x, torch.zeros((2, 4), device="cuda"))
