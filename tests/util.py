"""Shared test helpers: building quantized inputs on the host with the oracle's
generators, moving them to the device, and comparing results."""
from __future__ import annotations

import os

import numpy as np

import oracle as O

SUB4 = (O.INT4, O.UINT4, O.F4E2M1)
SUB2 = (O.INT2, O.UINT2)
F8 = (O.F8E4M3FN, O.F8E4M3FNUZ, O.F8E5M2, O.F8E5M2FNUZ)

# Value range of the integer codes each quantized dtype is drawn from.
CODE_RANGE = {
    O.UINT8: (0, 255), O.INT8: (-128, 127), O.UINT16: (0, 65535), O.INT16: (-32768, 32767),
    O.INT32: (-(1 << 20), 1 << 20), O.UINT4: (0, 15), O.INT4: (-8, 7), O.F4E2M1: (0, 15),
    O.UINT2: (0, 3), O.INT2: (-2, 1), O.F8E4M3FN: (0, 255), O.F8E4M3FNUZ: (0, 255),
    O.F8E5M2: (0, 255), O.F8E5M2FNUZ: (0, 255), O.F6E2M3: (0, 63), O.F6E3M2: (0, 63),
}


def encode_codes(codes: np.ndarray, dt: int) -> np.ndarray:
    """Integer codes -> raw storage bytes of dtype dt (packed for sub-byte types)."""
    c = np.asarray(codes, np.int64).ravel()
    if dt in SUB4:
        return O.pack_bits(c, 4)
    if dt in SUB2:
        return O.pack_bits(c, 2)
    if dt in (O.F6E2M3, O.F6E3M2):
        n = len(c)
        out = np.zeros(O.packed_nbytes(dt, n), np.uint8)
        for i, v in enumerate(c & 63):
            bo = i * 6
            by, sh = bo // 8, bo % 8
            out[by] |= (int(v) << sh) & 0xff
            if sh > 2:
                out[by + 1] |= int(v) >> (8 - sh)
        return out
    if dt in (O.UINT8, O.INT8) or dt in F8:
        return (c & 0xff).astype(np.uint8)
    if dt in (O.UINT16, O.INT16):
        return (c & 0xffff).astype(np.uint16).view(np.uint8)
    if dt == O.INT32:
        return c.astype(np.int32).view(np.uint8)
    raise ValueError(dt)


def random_q(seed: int, shape, dt: int, lo=None, hi=None) -> np.ndarray:
    lo_, hi_ = CODE_RANGE[dt]
    lo = lo_ if lo is None else lo
    hi = hi_ if hi is None else hi
    n = int(np.prod(shape)) if len(shape) else 1
    return encode_codes(O.randint(seed, (n,), lo, hi), dt)


def scale_raw(values: np.ndarray, s_dt: int) -> np.ndarray:
    v = np.asarray(values, np.float32)
    return v if s_dt == O.FLOAT else O.f32_to_f16_bits(v)


def to_dev(raw: np.ndarray, torch_dtype=None):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(raw)).cuda()
    return t.view(torch_dtype) if torch_dtype is not None else t


# (test id, rel-L2) of every rel_l2 call; conftest writes them to the file named by
# ONNXL_RELERR_LOG at the end of the session (the measured errors per dtype and kernel)
RELERR_LOG = []


def rel_l2(x: np.ndarray, ref: np.ndarray) -> float:
    x = np.asarray(x, np.float64)
    ref = np.asarray(ref, np.float64)
    den = np.linalg.norm(ref)
    v = float(np.linalg.norm(x - ref) / (den if den > 0 else 1.0))
    RELERR_LOG.append((os.environ.get("PYTEST_CURRENT_TEST", "").split(" ")[0], v))
    return v


def load_fixtures():
    """tests/golden/ref_fixtures.npz (produced by the reference kernels): (meta, arrays)."""
    import json
    import os
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "ref_fixtures.npz")
    z = np.load(path)
    meta = json.loads(bytes(z["meta"]).decode())
    return meta, z


def fixture_dq_inputs(m, z):
    """(x_raw, scale_raw, zp_raw or None, y_expected_raw) of a DequantizeLinear fixture."""
    k = m["key"]
    s = z[k + "_s"].view(np.float32 if m["s_dt"] == O.FLOAT else np.uint16)
    zp = z[k + "_z"] if m["zp"] else None
    y = z[k + "_y"].view(np.float32 if m["s_dt"] == O.FLOAT else np.uint16)
    return z[k + "_x"], s, zp, y


def np_int(raw, dt):
    return raw.view(np.int8) if dt == O.INT8 else raw.view(np.uint8)


def attention_fixture(m, z):
    """Inputs and the reference's outputs of one Attention fixture, as raw
    arrays: q, k, v, past_k, past_v (storage type of m["dt"]), mask (float32,
    numpy bool, or uint16 bits with mask_dt), nonpad (int64), y, qk, and the
    expected present_key / present_value (concat(past, new) on axis 2 when the
    generator did not store them; it checked that equality against the
    reference)."""
    k = m["key"]
    f = {"q": z[k + "_q"], "k": z[k + "_k"], "v": z[k + "_v"], "y": z[k + "_y"]}
    f["pk"] = z[k + "_pk"] if m["P"] else None
    f["pv"] = z[k + "_pv"] if m["P"] else None
    kind = m.get("mask_dt", "f32")
    f["mask"] = z[k + "_mask"] if m["mask"] else None
    f["mask_dt"] = {"f32": O.FLOAT, "bool": O.BOOL, "f16": O.FLOAT16, "bf16": O.BFLOAT16}[kind]
    f["nonpad"] = z[k + "_nonpad"] if "nonpad" in m else None
    f["qk"] = z[k + "_qk"] if "qk" in m else None
    if m["P"]:
        if k + "_prk" in z.files:
            f["prk"], f["prv"] = z[k + "_prk"], z[k + "_prv"]
        else:
            f["prk"] = np.concatenate([f["pk"], f["k"]], 2)
            f["prv"] = np.concatenate([f["pv"], f["v"]], 2)
    return f
