"""The device-side SplitMix64 generators produce the oracle's exact bytes."""
import numpy as np
import pytest
import torch

import oracle as O
from util import encode_codes

pytestmark = pytest.mark.gpu


def test_uniform_randn_randint_match_oracle(b2, cuda):
    from onnx_light_b200 import synth
    n = 100003
    np.testing.assert_array_equal(synth.uniform(7, (n,), 0.005, 0.02).cpu().numpy(),
                                  O.rand_uniform(7, (n,), 0.005, 0.02))
    np.testing.assert_array_equal(synth.randn(8, (n,), 0.0, 0.5).cpu().numpy(),
                                  O.randn(8, (n,), 0.0, 0.5))
    np.testing.assert_array_equal(synth.randint(9, (n,), -8, 7).cpu().numpy(),
                                  O.randint(9, (n,), -8, 7))
    np.testing.assert_array_equal(synth.randint(10, (n,), -127, 127).cpu().numpy(),
                                  O.randint(10, (n,), -127, 127))


def test_conversions_match_oracle(b2, cuda):
    from onnx_light_b200 import synth, _capi
    f = synth.randn(11, (65537,), 0.0, 300.0)
    fh = f.cpu().numpy()
    assert np.array_equal(synth.convert(f, _capi.FLOAT16).cpu().numpy().view(np.uint16),
                          O.f32_to_f16_bits(fh))
    assert np.array_equal(synth.convert(f, _capi.BFLOAT16).view(torch.int16).cpu().numpy().view(np.uint16),
                          O.f32_to_bf16_bits(fh))
    assert np.array_equal(synth.convert(f, _capi.FLOAT8E4M3FN).data.cpu().numpy(),
                          O.f32_to_f8e4m3fn(fh))
    q = synth.packed_randint(12, (4097,), -8, 7, _capi.INT4)
    assert np.array_equal(q.data.cpu().numpy(), encode_codes(O.randint(12, (4097,), -8, 7), O.INT4))
