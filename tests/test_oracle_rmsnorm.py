"""The oracle's RMSNorm (TransformerLayer.normalise, Runtime/TransformerLayer.swift:265-285;
Metal `rmsnorm`, Metal/MoE/router.metal:41-60): hand cases that pin the
semantics (plain multiplicative weight, not Gemma's 1 + weight; eps inside the
square root; f16 output), and agreement with an fp64 restatement to f16
rounding on random rows."""
import numpy as np
import oracle as O

BF16_ONE, BF16_TWO, BF16_HALF = 0x3F80, 0x4000, 0x3F00


def test_unit_rows():
    x = np.ones((1, 8), np.float32)
    w = np.full(8, BF16_ONE, np.uint16)
    assert np.array_equal(O.rmsnorm(x, w, 0.0), np.ones((1, 8), np.float16))
    # mean square 4 -> inverse 1/2; weight 2 -> back to 2
    assert np.array_equal(O.rmsnorm(2 * x, np.full(8, BF16_TWO, np.uint16), 0.0),
                          np.full((1, 8), 2.0, np.float16))
    # the weight multiplies (0.5), it is not added to one
    assert np.array_equal(O.rmsnorm(x, np.full(8, BF16_HALF, np.uint16), 0.0),
                          np.full((1, 8), 0.5, np.float16))


def test_eps_inside_root():
    x = np.array([[3.0, 4.0, 0.0, 0.0]], np.float32)    # mean square 25/4
    w = np.full(4, BF16_ONE, np.uint16)
    got = O.rmsnorm(x, w, 0.75).astype(np.float64)       # 1/sqrt(6.25 + 0.75) = 1/sqrt(7)
    assert np.allclose(got, np.array([[3, 4, 0, 0]]) / np.sqrt(7.0), rtol=1e-3)


def test_matches_fp64_to_f16_rounding():
    rng = np.random.default_rng(7)
    H = 2880
    x = rng.standard_normal((6, H)).astype(np.float32) * np.float32(3)
    wf = (1 + 0.1 * rng.standard_normal(H)).astype(np.float32)
    w = (wf.view(np.uint32) >> 16).astype(np.uint16)    # truncated to bf16 bits
    got = O.rmsnorm(x, w, 1e-5).astype(np.float64)
    w64 = (w.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    x64 = x.astype(np.float64)
    ref = x64 / np.sqrt((x64 * x64).mean(1, keepdims=True) + 1e-5) * w64
    ulp = np.abs(np.spacing(ref.astype(np.float16)).astype(np.float64))
    assert np.all(np.abs(got - ref) <= ulp)
