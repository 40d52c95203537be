"""Generates tests/golden/ref_fixtures.npz from onnx-light's own kernels.

Run in a container that has the reference tree: ``make -C oracle ref`` builds
oracle/_ref/libref.so from the reference sources, then
``python tests/golden/make_golden.py`` calls the reference kernels on seeded
inputs and stores inputs + outputs.  The committed fixtures let the GPU box
(which has no reference tree) check parity against the reference itself.

Cases cover every DequantizeLinear input type and layout (per-tensor,
per-axis, blocked; with and without zero point; FLOAT and FLOAT16 scales;
NaN/Inf float8 codes; odd element counts), MatMulInteger zero-point modes and
broadcast batches, QLinearMatMul including ties-to-even and saturation, MatMul
in FLOAT/FLOAT16/BFLOAT16 and Attention (GQA, causal, past KV, softcap, mask,
rank-3).
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.dirname(HERE))

import oracle as O  # noqa: E402
from util import CODE_RANGE, encode_codes, scale_raw  # noqa: E402

OUT = os.path.join(HERE, "ref_fixtures.npz")


def dq_cases():
    """(name, x_dt, x_shape, s_dt, s_shape, has_zp, axis) tuples."""
    dts = [O.UINT8, O.INT8, O.UINT16, O.INT16, O.INT32, O.F8E4M3FN, O.F8E4M3FNUZ, O.F8E5M2,
           O.F8E5M2FNUZ, O.UINT4, O.INT4, O.UINT2, O.INT2, O.F4E2M1, O.F6E2M3, O.F6E3M2]
    cases = []
    for dt in dts:
        for s_dt in (O.FLOAT, O.FLOAT16):
            for zp in (False, True):
                cases.append((dt, (7, 5), s_dt, (), zp, 1))              # per-tensor, odd count
                cases.append((dt, (4, 6, 8), s_dt, (6,), zp, 1))         # per-axis, middle axis
                cases.append((dt, (64, 48), s_dt, (2, 48), zp, 0))       # blocked along axis 0
                cases.append((dt, (6, 64), s_dt, (6, 4), zp, 1))         # blocked along the last axis
    return cases


def main():
    arrays = {}
    meta = {"dq": [], "mmi": [], "qlm": [], "mm": [], "att": []}
    seed = 100

    # ---------------- DequantizeLinear ----------------
    for i, (dt, xs, s_dt, ss, has_zp, axis) in enumerate(dq_cases()):
        seed += 10
        n = int(np.prod(xs))
        lo, hi = CODE_RANGE[dt]
        codes = O.randint(seed, (n,), lo, hi)
        x = encode_codes(codes, dt)
        sn = int(np.prod(ss)) if len(ss) else 1
        s = scale_raw(O.rand_uniform(seed + 1, (sn,), 0.01, 2.0), s_dt)
        zp = None
        if has_zp:
            if dt in (O.F8E4M3FN, O.F8E4M3FNUZ, O.F8E5M2, O.F8E5M2FNUZ):
                zcodes = O.randint(seed + 2, (sn,), 0, 40)  # small finite float8 values
            else:
                zlo, zhi = CODE_RANGE[dt]
                zcodes = O.randint(seed + 2, (sn,), max(zlo, -3), min(zhi, 3))
            zp = encode_codes(zcodes, dt)
        y = O.ref_dequantize_linear(x, dt, xs, s, s_dt, ss, zp, ss if has_zp else None, axis)
        k = f"dq{i}"
        arrays[k + "_x"], arrays[k + "_s"], arrays[k + "_y"] = x, s.view(np.uint8), y.view(np.uint8)
        if zp is not None:
            arrays[k + "_z"] = zp
        meta["dq"].append(dict(key=k, x_dt=dt, x_shape=list(xs), s_dt=s_dt, s_shape=list(ss),
                               zp=has_zp, axis=axis))

    # ---------------- MatMulInteger ----------------
    mmi = [
        ((16, 64), O.UINT8, (64, 40), O.INT8, "scalar", "col"),
        ((16, 64), O.INT8, (64, 40), O.INT8, "row", "scalar"),
        ((3, 1, 33, 70), O.UINT8, (2, 70, 17), O.UINT8, "scalar", "none"),
        ((70,), O.INT8, (70, 9), O.UINT8, "none", "col"),
        ((5, 70), O.UINT8, (70,), O.INT8, "row", "none"),
        ((130, 256), O.UINT8, (256, 200), O.INT8, "scalar", "col"),
    ]
    for i, (ash, adt, bsh, bdt, az, bz) in enumerate(mmi):
        seed += 10
        a = encode_codes(O.randint(seed, (int(np.prod(ash)),), *CODE_RANGE[adt]), adt).reshape(ash)
        b = encode_codes(O.randint(seed + 1, (int(np.prod(bsh)),), *CODE_RANGE[bdt]), bdt).reshape(bsh)
        M = ash[-2] if len(ash) > 1 else 1
        N = bsh[-1] if len(bsh) > 1 else 1
        azp = bzp = None
        if az != "none":
            azp = encode_codes(O.randint(seed + 2, ((M if az == "row" else 1),), 100, 130) if adt == O.UINT8
                               else O.randint(seed + 2, ((M if az == "row" else 1),), -5, 5), adt)
        if bz != "none":
            bzp = encode_codes(O.randint(seed + 3, ((N if bz == "col" else 1),), -4, 4) if bdt == O.INT8
                               else O.randint(seed + 3, ((N if bz == "col" else 1),), 120, 130), bdt)
        y = O.ref_matmul_integer(a, adt, b, bdt, azp, bzp,
                                 a_zp_shape=None if azp is None else [azp.size],
                                 b_zp_shape=None if bzp is None else [bzp.size])
        k = f"mmi{i}"
        arrays[k + "_a"], arrays[k + "_b"], arrays[k + "_y"] = a, b, y
        if azp is not None:
            arrays[k + "_az"] = azp
        if bzp is not None:
            arrays[k + "_bz"] = bzp
        meta["mmi"].append(dict(key=k, a_dt=adt, b_dt=bdt, a_shape=list(ash), b_shape=list(bsh),
                                az=azp is not None, bz=bzp is not None))

    # ---------------- QLinearMatMul ----------------
    kat = json.load(open(os.path.join(HERE, "kat_reference_tests.json")))["qlinear_matmul_inputs"][0]
    qcases = []
    for is_int8 in (False, True):
        sh = 127 if is_int8 else 0
        dt = O.INT8 if is_int8 else O.UINT8
        a = np.array([v - sh for v in kat["a"]], np.int64)
        b = np.array([v - sh for v in kat["b"]], np.int64)
        for s_dt in (O.FLOAT, O.FLOAT16):
            qcases.append(dict(a=encode_codes(a, dt).reshape(kat["a_shape"]),
                               b=encode_codes(b, dt).reshape(kat["b_shape"]), dt=dt, s_dt=s_dt,
                               sc=(kat["a_scale"], kat["b_scale"], kat["y_scale"]),
                               zp=(kat["a_zp"] - sh, kat["b_zp"] - sh, kat["y_zp"] - sh)))
    for i, (ash, bsh, dt, ydt) in enumerate([((64, 96), (96, 48), O.UINT8, O.UINT8),
                                             ((2, 33, 70), (70, 19), O.INT8, O.INT8),
                                             ((40, 128), (128, 64), O.UINT8, O.INT8)]):
        seed += 10
        a = encode_codes(O.randint(seed, (int(np.prod(ash)),), *CODE_RANGE[dt]), dt).reshape(ash)
        b = encode_codes(O.randint(seed + 1, (int(np.prod(bsh)),), *CODE_RANGE[dt]), dt).reshape(bsh)
        zp = (3, -2, 5) if dt == O.INT8 else (113, 114, 118)
        if ydt == O.INT8 and dt == O.UINT8:
            zp = (113, 114, -7)
        qcases.append(dict(a=a, b=b, dt=dt, ydt=ydt, s_dt=O.FLOAT, sc=(0.0066, 0.00705, 0.0107 * (1 + i)),
                           zp=zp))
    for i, c in enumerate(qcases):
        ydt = c.get("ydt", c["dt"])
        y = O.ref_qlinear_matmul(c["a"], c["dt"], c["sc"][0], c["zp"][0], c["b"], c["dt"], c["sc"][1],
                                 c["zp"][1], c["sc"][2], c["zp"][2], ydt, scale_dt=c["s_dt"])
        k = f"qlm{i}"
        arrays[k + "_a"], arrays[k + "_b"], arrays[k + "_y"] = c["a"], c["b"], y.view(np.uint8)
        meta["qlm"].append(dict(key=k, dt=c["dt"], ydt=ydt, s_dt=c["s_dt"], sc=list(c["sc"]),
                                zp=list(c["zp"]), a_shape=list(c["a"].shape),
                                b_shape=list(c["b"].shape)))

    # ---------------- MatMul ----------------
    for i, (ash, bsh, dt) in enumerate([((3, 37, 64), (64, 50), O.FLOAT),
                                        ((8, 128), (128, 96), O.FLOAT16),
                                        ((2, 16, 96), (96, 64), O.BFLOAT16)]):
        seed += 10
        a = O.randn(seed, ash)
        b = O.randn(seed + 1, bsh)
        if dt == O.FLOAT16:
            a, b = O.f32_to_f16_bits(a), O.f32_to_f16_bits(b)
        elif dt == O.BFLOAT16:
            a, b = O.f32_to_bf16_bits(a), O.f32_to_bf16_bits(b)
        y = O.ref_matmul(a, b, dt)
        k = f"mm{i}"
        arrays[k + "_a"], arrays[k + "_b"], arrays[k + "_y"] = a, b, y
        meta["mm"].append(dict(key=k, dt=dt))

    # ---------------- Attention ----------------
    # Optional keys: Sk (new keys, default Sq), Dv (V head size, default D),
    # mask_dt ("f32" default, "bool", "f16", "bf16") and mask_shape (default
    # (Sq, P + Sk)), nonpad (nonpad_kv_seqlen per batch), qk (qk_matmul_output
    # mode), lw / rw (window sizes).
    F16, BF16 = O.FLOAT16, O.BFLOAT16
    att = [
        dict(B=2, Hq=8, Hkv=2, Sq=1, P=37, D=64, causal=True, softcap=0.0, mask=False, rank=4, dt=F16),
        dict(B=1, Hq=4, Hkv=4, Sq=9, P=0, D=32, causal=True, softcap=0.0, mask=False, rank=4, dt=F16),
        dict(B=2, Hq=6, Hkv=3, Sq=5, P=11, D=16, causal=False, softcap=5.0, mask=True, rank=4, dt=O.FLOAT),
        dict(B=1, Hq=4, Hkv=2, Sq=7, P=0, D=32, causal=True, softcap=0.0, mask=False, rank=3, dt=BF16),
        dict(B=1, Hq=32, Hkv=8, Sq=1, P=65, D=128, causal=True, softcap=0.0, mask=False, rank=4, dt=F16),
        # BOOL mask with fully masked rows, GQA, past
        dict(B=2, Hq=8, Hkv=2, Sq=4, P=20, D=64, causal=True, softcap=0.0, mask=True, mask_dt="bool",
             rank=4, dt=F16),
        # BFLOAT16 mask shorter than the keys (padded with -inf), qk after the mask
        dict(B=1, Hq=4, Hkv=2, Sq=6, P=0, D=64, causal=False, softcap=0.0, mask=True, mask_dt="bf16",
             mask_shape=(1, 4, 6, 4), rank=4, dt=BF16, qk=2),
        # nonpad_kv_seqlen with the causal frontier it offsets, softmax probabilities
        dict(B=3, Hq=4, Hkv=4, Sq=3, Sk=10, P=0, D=32, causal=True, softcap=0.0, mask=False, rank=4,
             dt=F16, nonpad=[10, 7, 4], qk=3),
        # v_head_size != head_size, softcap, windows, raw scores
        dict(B=2, Hq=6, Hkv=2, Sq=5, P=7, D=32, Dv=16, causal=False, softcap=4.0, mask=False, rank=4,
             dt=O.FLOAT, lw=3, rw=1, qk=0),
        # rank-3 with v_head_size != head_size, scores after the softcap
        dict(B=1, Hq=4, Hkv=2, Sq=5, P=0, D=16, Dv=24, causal=True, softcap=2.0, mask=False, rank=3,
             dt=O.FLOAT, qk=1),
        # BFLOAT16 prefill on the tensor-core path (head 128, no mask), rank 4 and rank 3
        dict(B=1, Hq=8, Hkv=2, Sq=160, P=0, D=128, causal=True, softcap=0.0, mask=False, rank=4, dt=BF16),
        dict(B=2, Hq=4, Hkv=1, Sq=130, P=0, D=128, causal=True, softcap=0.0, mask=False, rank=3, dt=BF16),
        # BFLOAT16 decode with a past (CUDA-core decode)
        dict(B=2, Hq=8, Hkv=2, Sq=1, P=300, D=128, causal=True, softcap=0.0, mask=False, rank=4, dt=BF16),
        # FLOAT16 decode on the tensor-core path, longer past
        dict(B=1, Hq=32, Hkv=8, Sq=1, P=257, D=128, causal=True, softcap=0.0, mask=False, rank=4, dt=F16),
        # FLOAT16 prefill with a past on the tensor-core path
        dict(B=1, Hq=8, Hkv=2, Sq=64, P=100, D=128, causal=True, softcap=0.0, mask=False, rank=4, dt=F16),
        # FLOAT16 inputs with a BFLOAT16 mask (any half mask is promoted)
        dict(B=1, Hq=2, Hkv=1, Sq=5, P=3, D=32, causal=False, softcap=0.0, mask=True, mask_dt="bf16",
             rank=4, dt=F16),
        # Scores that overflow FLOAT in query row 0 (the reference's non-finite
        # rescue, kernel_attention.cc:33-158, makes that row finite), finite in row 1
        dict(B=1, Hq=1, Hkv=1, Sq=2, P=0, Sk=3, D=8, causal=False, softcap=0.0, mask=False, rank=4,
             dt=O.FLOAT, overflow=True),
    ]
    for i, c in enumerate(att):
        seed += 10
        B, Hq, Hkv, Sq, P, D = c["B"], c["Hq"], c["Hkv"], c["Sq"], c["P"], c["D"]
        Sk, Dv = c.get("Sk", Sq), c.get("Dv", D)
        if c["rank"] == 4:
            q = O.randn(seed, (B, Hq, Sq, D), 0, 0.5)
            k = O.randn(seed + 1, (B, Hkv, Sk, D), 0, 0.5)
            v = O.randn(seed + 2, (B, Hkv, Sk, Dv), 0, 0.5)
        else:
            q = O.randn(seed, (B, Sq, Hq * D), 0, 0.5)
            k = O.randn(seed + 1, (B, Sk, Hkv * D), 0, 0.5)
            v = O.randn(seed + 2, (B, Sk, Hkv * Dv), 0, 0.5)
        if c.get("overflow"):
            q[:, :, 0, :] = 1e19                      # q0 . k_j overflows FLOAT for every j
            k = (np.abs(k) + 0.5).astype(np.float32) * np.float32(1e19)
        pk = O.randn(seed + 3, (B, Hkv, P, D), 0, 0.5) if P else None
        pv = O.randn(seed + 4, (B, Hkv, P, Dv), 0, 0.5) if P else None
        mask, mdt = None, None
        if c["mask"]:
            mshape = tuple(c.get("mask_shape", (Sq, P + Sk)))
            kind = c.get("mask_dt", "f32")
            mval = O.randn(seed + 5, mshape, 0, 1.0)
            if kind == "bool":
                mask = mval > -0.3
                mask[..., 1, :] = False  # one fully masked query row
            elif kind == "f16":
                mask, mdt = O.f32_to_f16_bits(mval), O.FLOAT16
            elif kind == "bf16":
                mask, mdt = O.f32_to_bf16_bits(mval), O.BFLOAT16
            else:
                mask = mval
        cv = {O.FLOAT: lambda t: t, O.FLOAT16: O.f32_to_f16_bits, O.BFLOAT16: O.f32_to_bf16_bits}[c["dt"]]
        q, k, v = cv(q), cv(k), cv(v)
        if P:
            pk, pv = cv(pk), cv(pv)
        nonpad = np.array(c["nonpad"], np.int64) if "nonpad" in c else None
        out = O.ref_attention(q, k, v, dt=c["dt"], is_causal=c["causal"], softcap=c["softcap"],
                              mask=mask, past_k=pk, past_v=pv, q_num_heads=Hq, kv_num_heads=Hkv,
                              mask_dt=mdt, nonpad=nonpad, left_window=c.get("lw", -1),
                              right_window=c.get("rw", -1), qk_mode=c.get("qk"))
        y, prk, prv = out[:3]
        kk = f"att{i}"
        arrays.update({kk + "_q": q, kk + "_k": k, kk + "_v": v, kk + "_y": y})
        if P:
            arrays.update({kk + "_pk": pk, kk + "_pv": pv})
            # present = concat(past, new) on axis 2 (kernel_attention.cc:313-339);
            # large presents are stored only as that check, not as arrays.
            if prk.nbytes <= (64 << 10):
                arrays.update({kk + "_prk": prk, kk + "_prv": prv})
            elif c["rank"] == 4:
                assert np.array_equal(prk, np.concatenate([pk, k], 2))
                assert np.array_equal(prv, np.concatenate([pv, v], 2))
            else:
                raise AssertionError("large rank-3 presents are not stored")
        if mask is not None:
            arrays[kk + "_mask"] = mask
        if nonpad is not None:
            arrays[kk + "_nonpad"] = nonpad
        if "qk" in c:
            arrays[kk + "_qk"] = out[3]
        meta["att"].append(dict(key=kk, **c))

    # ---------------- decoder-layer operators ----------------
    meta["dec"] = []
    cvt = {O.FLOAT: lambda t: t.astype(np.float32), O.FLOAT16: O.f32_to_f16_bits,
           O.BFLOAT16: O.f32_to_bf16_bits}
    rms = [((2, 7, 4096), (4096,), -1, O.FLOAT, 1e-5), ((3, 64), (), -1, O.FLOAT16, 1e-6),
           ((2, 3, 40), (1, 40), 1, O.BFLOAT16, 1e-5), ((5, 256), (5, 256), 0, O.FLOAT, 1e-3)]
    for i, (xs, ss, axis, dt, eps) in enumerate(rms):
        seed += 10
        x = cvt[dt](O.randn(seed, xs))
        sc = cvt[dt](O.rand_uniform(seed + 1, ss, 0.5, 1.5) if ss else np.float32(1.25))
        y = O.ref_rms_normalization(x, np.asarray(sc), dt, axis, eps)
        k = f"rms{i}"
        arrays.update({k + "_x": x, k + "_s": np.asarray(sc), k + "_y": y})
        meta["dec"].append(dict(key=k, op="RMSNormalization", dt=dt, axis=axis, eps=eps))
    rot = [((2, 4, 9, 64), None, False, 0, 0, O.FLOAT), ((2, 9, 4 * 64), (2, 9), True, 0, 4, O.FLOAT16),
           ((1, 2, 7, 128), (1, 7), False, 64, 0, O.BFLOAT16), ((3, 5, 2 * 32), (3, 5), False, 0, 2, O.FLOAT)]
    for i, (xs, ps, inter, rdim, nh, dt) in enumerate(rot):
        seed += 10
        x = cvt[dt](O.randn(seed, xs))
        D = xs[3] if len(xs) == 4 else xs[2] // nh
        half = (rdim or D) // 2
        B, S = xs[0], (xs[2] if len(xs) == 4 else xs[1])
        if ps is None:
            cs_shape, pos = (B, S, half), None
        else:
            cs_shape, pos = (32, half), O.randint(seed + 3, (B * S,), 0, 31).reshape(B, S)
        c = cvt[dt](O.rand_uniform(seed + 1, cs_shape, -1.0, 1.0))
        sn = cvt[dt](O.rand_uniform(seed + 2, cs_shape, -1.0, 1.0))
        y = O.ref_rotary_embedding(x, c, sn, dt, pos, inter, rdim, nh)
        k = f"rot{i}"
        arrays.update({k + "_x": x, k + "_c": c, k + "_s": sn, k + "_y": y})
        if pos is not None:
            arrays[k + "_p"] = pos
        meta["dec"].append(dict(key=k, op="RotaryEmbedding", dt=dt, interleaved=inter, rdim=rdim,
                                num_heads=nh, pos=pos is not None))
    for i, (sh, dt, alpha) in enumerate([((4, 11008), O.FLOAT, 1.0), ((3, 1000), O.FLOAT16, 1.702),
                                         ((2, 515), O.BFLOAT16, 1.0)]):
        seed += 10
        a_ = cvt[dt](O.randn(seed, sh))
        b_ = cvt[dt](O.randn(seed + 1, sh))
        y = O.ref_swiglu(a_, b_, dt, alpha)
        k = f"swi{i}"
        arrays.update({k + "_a": a_, k + "_b": b_, k + "_y": y})
        meta["dec"].append(dict(key=k, op="SwiGLU", dt=dt, alpha=alpha))

    arrays["meta"] = np.frombuffer(json.dumps(meta).encode(), np.uint8)
    np.savez_compressed(OUT, **arrays)
    print(f"wrote {OUT}: {sum(len(v) for v in meta.values())} cases, {os.path.getsize(OUT)} bytes")


if __name__ == "__main__":
    main()
