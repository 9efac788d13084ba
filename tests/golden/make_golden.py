"""Generates tests/golden/*.npz by importing the reference's own NumPy code.

Run here, where the reference checkout is mounted (it is not needed at test
time: the vectors are committed):

    python tests/golden/make_golden.py /path/to/rayl15-Godwit

Uses `dequantize`, `FP4`, `bf16`, `ALPHA` and `LIMIT` from
Scripts/analysis/expert_reference.py (:21-47) and `dequantize` from
Scripts/analysis/fetch_expert.py (:39-48), and the expert formula of
expert_reference.py:68-74 (which lives inside its main()) with those
functions.  Inputs are seeded synthetic MXFP4 experts (codes uniform 0..15,
scales 118..124, bf16 biases ~N(0, 0.02)) and x ~N(0, 0.5) in float16 as the
reference's fixture builder draws it.

reference_int8.npz: `int8_affine` of Scripts/analysis/qwen3_quant_quality.py
(:104-110, the reference's NumPy statement of the trunk's affine int8 scheme)
applied to seeded float32 weight rows, including a constant group and a
group holding only two values.
"""
import importlib.util
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def load(path, name):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def main(ref_root):
    er = load(os.path.join(ref_root, "Scripts/analysis/expert_reference.py"), "expert_reference")
    fe = load(os.path.join(ref_root, "Scripts/analysis/fetch_expert.py"), "fetch_expert")
    rng = np.random.default_rng(20240607)

    # 1. dequant vectors, including edge scales (0 -> 2^-127, 254, 255 -> the
    #    reference NumPy gives inf via exp2(128); the Swift decoder gives NaN).
    rows, cols = 8, 128
    packed = rng.integers(0, 256, (rows, cols // 2), dtype=np.uint8)
    scales = rng.integers(100, 140, (rows, cols // 32), dtype=np.uint8)
    scales[0, 0], scales[1, 1], scales[2, 2] = 0, 254, 1
    w_er = er.dequantize(packed.tobytes(), scales.tobytes(), rows, cols)
    w_fe = fe.dequantize(packed.reshape(rows, cols // 32, 16), scales)
    assert np.array_equal(w_er.view(np.uint32), w_fe.view(np.uint32))

    # 2. whole experts (GPT-OSS formula) at a small shape
    H, F = 128, 96
    experts = []
    for e in range(3):
        gu_p = rng.integers(0, 256, (2 * F, H // 2), dtype=np.uint8)
        gu_s = rng.integers(118, 125, (2 * F, H // 32), dtype=np.uint8)
        dn_p = rng.integers(0, 256, (H, F // 2), dtype=np.uint8)
        dn_s = rng.integers(118, 125, (H, F // 32), dtype=np.uint8)
        gb = (np.frombuffer(rng.normal(0, 0.02, 2 * F).astype(np.float32).tobytes(), np.uint32) >> 16).astype(np.uint16)
        db = (np.frombuffer(rng.normal(0, 0.02, H).astype(np.float32).tobytes(), np.uint32) >> 16).astype(np.uint16)
        x = (rng.standard_normal(H) * 0.5).astype(np.float16)
        gu_w = er.dequantize(gu_p.tobytes(), gu_s.tobytes(), 2 * F, H)
        dn_w = er.dequantize(dn_p.tobytes(), dn_s.tobytes(), H, F)
        gate_up = gu_w @ x.astype(np.float32) + er.bf16(gb.tobytes())
        gate, up = gate_up[0::2], gate_up[1::2]
        gate = np.minimum(gate, er.LIMIT)
        up = np.clip(up, -er.LIMIT, er.LIMIT)
        glu = gate / (1.0 + np.exp(-er.ALPHA * gate)) * 1.0
        activated = ((up + 1.0) * glu).astype(np.float16)
        y = dn_w @ activated.astype(np.float32) + er.bf16(db.tobytes())
        experts.append(dict(gu_p=gu_p, gu_s=gu_s, dn_p=dn_p, dn_s=dn_s, gb=gb, db=db, x=x,
                            act=activated, y=y.astype(np.float32)))

    out = dict(dq_packed=packed, dq_scales=scales, dq_w=w_er.astype(np.float32),
               fp4=er.FP4.astype(np.float32), H=H, F=F, n=len(experts))
    for i, ex in enumerate(experts):
        for k, v in ex.items():
            out[f"e{i}_{k}"] = v
    np.savez_compressed(os.path.join(HERE, "reference_numpy.npz"), **out)
    print("wrote", os.path.join(HERE, "reference_numpy.npz"))
    main_int8(ref_root)


def main_int8(ref_root):
    # the module reads tensors over HTTP only from its main(); importing it
    # defines the functions and touches no network
    qq = load(os.path.join(ref_root, "Scripts/analysis/qwen3_quant_quality.py"), "qwen3_quant_quality")
    rng = np.random.default_rng(20240611)
    w = (rng.standard_normal((24, 256)) * 0.02).astype(np.float32)
    w[3, 64:128] = 0.0125                      # a constant group
    w[5, :64] = np.where(np.arange(64) % 2 == 0, -0.5, 0.25).astype(np.float32)  # two values
    back = qq.int8_affine(w.copy(), group=64).astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "reference_int8.npz"), w=w, back=back)
    print("wrote", os.path.join(HERE, "reference_int8.npz"))


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("GODWIT_REFERENCE", ""))
