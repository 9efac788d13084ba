"""Pins the oracle against vectors produced by the reference's own NumPy code
(tests/golden/make_golden.py imports Scripts/analysis/expert_reference.py and
fetch_expert.py)."""
import os

import numpy as np
import oracle as O

from godwit_b200.layout import ModelSpec
from godwit_b200.synth import bf16_bits_to_f32

G = np.load(os.path.join(os.path.dirname(__file__), "golden", "reference_numpy.npz"))


def test_dequant_bit_exact_against_reference_numpy():
    w = O.dequant(G["dq_packed"], G["dq_scales"])
    ref = G["dq_w"]
    # the reference NumPy decodes through exp2 and so has no NaN scale; the
    # fixture's scales avoid 0xFF, and every other value must match bit for bit
    assert np.array_equal(w.view(np.uint32), ref.view(np.uint32))


def test_codebook_equals_reference_fp4():
    assert np.array_equal(O.codebook().view(np.uint32), G["fp4"].view(np.uint32))


def _stride(spec, i):
    lay = spec.layout()
    buf = np.zeros(lay.stride, np.uint8)
    parts = {"gate_up_blocks": G[f"e{i}_gu_p"], "gate_up_scales": G[f"e{i}_gu_s"],
             "down_blocks": G[f"e{i}_dn_p"], "down_scales": G[f"e{i}_dn_s"],
             "gate_up_bias": G[f"e{i}_gb"], "down_bias": G[f"e{i}_db"]}
    for k, v in parts.items():
        raw = np.ascontiguousarray(v).view(np.uint8).ravel()
        buf[lay.offsets[k]:lay.offsets[k] + raw.size] = raw
    return buf


def golden_spec():
    return ModelSpec("golden", int(G["H"]), int(G["F"]), 4, 1, 2, 0)


def test_expert_apply_matches_reference_numpy():
    spec = golden_spec()
    for i in range(int(G["n"])):
        x = G[f"e{i}_x"].astype(np.float32)
        y = O.expert_apply(spec, _stride(spec, i), x)
        ref = G[f"e{i}_y"]
        # check-expert's tolerance, relative to mean |y| (main.swift:518-533)
        assert np.max(np.abs(y - ref)) / np.mean(np.abs(ref)) < 5e-3
        y64 = O.expert64(spec, _stride(spec, i), x)
        assert O.rel_l2(y, y64) < 1e-4


def test_int8_quantiser_matches_the_reference_numpy_scheme():
    """Int8Affine.quantize as restated in the oracle (Install/Int8Affine.swift:31-58),
    dequantised in float32, against `int8_affine` of the reference's
    Scripts/analysis/qwen3_quant_quality.py:104-110 on the same rows
    (tests/golden/reference_int8.npz).  The two statements differ only where
    a level lands exactly on .5 (Swift rounds half away from zero, NumPy to
    even) and in the scale a constant group gets (both give back the value)."""
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "reference_int8.npz"))
    w, back = g["w"], g["back"]
    ours = np.empty_like(w)
    ties = np.zeros(w.shape, bool)
    for r in range(w.shape[0]):
        codes, scale, zero = O.int8_quantize_row(w[r])
        s = np.repeat(scale, 64).astype(np.float32)
        z = np.repeat(zero, 64).astype(np.float32)
        ours[r] = codes.astype(np.float32) * s + z
        level = (w[r] - z) / s
        ties[r] = np.abs(level - np.floor(level) - 0.5) < 1e-6
    same = ours.view(np.uint32) == back.view(np.uint32)
    assert np.all(same | ties)
    assert same.mean() > 0.999
