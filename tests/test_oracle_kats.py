"""Pins the CPU oracle to the reference's own known-answer tests.

Each test names the reference test it restates (paths inside rayl15/Godwit).
"""
import math

import numpy as np
import oracle as O
import pytest

from godwit_b200.layout import GPT_OSS_120B, QWEN3_30B_A3B, ExpertLayout, PAGE


# ---- Tests/GodwitTests/MXFP4Tests.swift ------------------------------------

def test_codebook_shape():  # MXFP4Tests.swift:7-16
    cb = O.codebook()
    assert cb.size == 16 and cb[0] == 0.0 and cb[7] == 6.0
    for c in range(8):
        assert cb[c + 8] == -cb[c]
        assert math.copysign(1.0, cb[c + 8]) == -1.0


def test_scale_decoding():  # MXFP4Tests.swift:18-26
    assert O.decode_scale(127) == 1.0
    assert O.decode_scale(128) == 2.0
    assert O.decode_scale(126) == 0.5
    assert math.isnan(O.decode_scale(0xFF))
    assert O.decode_scale(0) > 0


def test_nibble_order():  # MXFP4Tests.swift:28-43: 0x71 -> [0.5, 6.0]
    packed = np.zeros(16, np.uint8)
    packed[0] = 0x71
    d = O.decode(packed, np.array([127], np.uint8))
    assert d[0] == 0.5 and d[1] == 6.0


def test_scale_applies():  # MXFP4Tests.swift:45-58
    d = O.decode(np.full(16, 0x22, np.uint8), np.array([130], np.uint8))
    assert np.all(d == 8.0)


def test_multi_block_decode():  # MXFP4Tests.swift:60-76
    d = O.decode(np.full(48, 0x22, np.uint8), np.array([127, 128, 126], np.uint8))
    assert d.size == 96 and d[0] == 1.0 and d[32] == 2.0 and d[64] == 0.5


# ---- Tests/GodwitTests/MXFP4EncodeTests.swift ------------------------------

def test_grid_values_round_trip():  # MXFP4EncodeTests.swift:13-41
    mags = [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0]
    w = []
    for e in (-4, -1, 0, 3, 10):
        s = 2.0 ** e
        blk = []
        for m in mags:
            blk += [m * s, -m * s]
        blk += [0.0] * (32 - len(blk))
        w += blk
    w = np.array(w, np.float32)
    p, s = O.encode(w)
    d = O.decode(p, s)
    assert np.array_equal(d, w)


def test_scale_ceils():  # MXFP4EncodeTests.swift:43-58
    assert O.decode_scale(O.scale_byte_for_peak(10)) == 2.0
    assert O.decode_scale(O.scale_byte_for_peak(6)) == 1.0
    assert O.decode_scale(O.scale_byte_for_peak(3)) == 0.5
    for step in range(200):
        peak = np.float32(2.0 ** (step / 8 - 12))
        scale = O.decode_scale(O.scale_byte_for_peak(float(peak)))
        assert peak / scale <= 6.0 + 1e-6


@pytest.mark.parametrize("v,code", [(0.0, 0), (0.24, 0), (0.26, 1), (0.9, 2), (1.4, 3),
                                    (2.6, 5), (4.9, 6), (5.1, 7), (99, 7)])
def test_rounds_to_nearest(v, code):  # MXFP4EncodeTests.swift:60-71
    assert O.code_for_magnitude(v) == code


def test_sign_handling():  # MXFP4EncodeTests.swift:73-90
    w = np.array([1.0, -1.0, 0.0, -0.0] + [0.0] * 28, np.float32)
    p, s = O.encode(w)
    d = O.decode(p, s)
    assert d[0] == 1.0 and d[1] == -1.0
    assert math.copysign(1, d[2]) == 1 and math.copysign(1, d[3]) == -1


def test_short_block_pads():  # MXFP4EncodeTests.swift:92-106
    p, s = O.encode(np.array([1.0, 2.0, 3.0], np.float32))
    assert s.size == 1 and p.size == 16
    d = O.decode(p, s)
    assert list(d[:3]) == [1.0, 2.0, 3.0] and np.all(d[3:] == 0)


def test_zero_block():  # MXFP4EncodeTests.swift:108-114
    p, s = O.encode(np.zeros(32, np.float32))
    assert np.all(p == 0) and s[0] == 127


def test_error_bound():  # MXFP4EncodeTests.swift:116-139
    rng = np.random.default_rng(7)
    w = rng.uniform(-3, 3, 32 * 64).astype(np.float32)
    p, s = O.encode(w)
    d = O.decode(p, s)
    for b in range(s.size):
        sc = O.decode_scale(s[b])
        assert np.all(np.abs(d[b * 32:(b + 1) * 32] - w[b * 32:(b + 1) * 32]) <= sc * 1.0 + 1e-6)


# ---- Tests/GodwitTests/DequantGEMVTests.swift ------------------------------

def test_gemv_hand_case():  # DequantGEMVTests.swift:64-77: 16 x 0x22, scale 127, x = 1 -> 32
    y = O.gemv(np.full((1, 16), 0x22, np.uint8), np.array([[127]], np.uint8), np.ones(32, np.float32))
    assert abs(y[0] - 32.0) < 1e-4


def test_gemv_matches_dequant_dot():
    rng = np.random.default_rng(3)
    p = rng.integers(0, 256, (64, 128), dtype=np.uint8)
    s = rng.integers(120, 134, (64, 8), dtype=np.uint8)
    x = rng.standard_normal(256).astype(np.float16).astype(np.float32)
    y = O.gemv(p, s, x)
    ref = O.dequant64(p, s) @ x.astype(np.float64)
    assert np.max(np.abs(y - ref) / np.maximum(np.abs(ref), 1.0)) < 1e-5
    assert np.array_equal(O.gemv(p, s, x, threads=4), y)


# ---- Router.select (Runtime/Router.swift:78-98) ------------------------------

def test_select_orders_by_logit_and_softmaxes_over_k():
    lg = np.array([0.1, 2.0, -1.0, 3.0, 0.5], np.float32)
    ex, wt = O.router_select(lg, 2)
    assert list(ex) == [3, 1]
    e = np.exp(np.array([3.0, 2.0]) - 3.0)
    assert np.allclose(wt, e / e.sum(), rtol=1e-6)


def test_select_tie_follows_swap_order_not_lowest_index():
    # [a=1, b=1, c=5]: pass 0 swaps c to the front (order [2, 1, 0]); pass 1
    # then keeps position 1 (expert 1) — a lowest-index rule would pick 0.
    ex, _ = O.router_select(np.array([1.0, 1.0, 5.0], np.float32), 2)
    assert list(ex) == [2, 1]


# ---- activations (ActivationTests.swift:62-96; expert.metal:82-102) ---------

GATE = np.array([-4, -2, -1, -0.5, 0, 0.5, 1, 2, 4, 8, -8, 0.1], np.float32)
UP = np.array([1, -1, 2, 0.5, 3, -2, 1, 0.25, -1, 2, 1, -3], np.float32)


def _interleave(g, u):
    gu = np.empty(2 * g.size, np.float32)
    gu[0::2], gu[1::2] = g, u
    return gu


def test_swiglu_matches_silu():  # ActivationTests.swift:78-86
    got = O.act_silu(_interleave(GATE, UP))
    want = GATE / (1 + np.exp(-GATE)) * UP
    assert np.all(np.abs(got - want) < 0.01)


def test_gptoss_activation_clamps_asymmetrically():
    got = O.act_gptoss(_interleave(GATE, UP * 5))
    g = np.minimum(GATE, 7.0)
    u = np.clip(UP * 5, -7, 7)
    want = (u + 1) * g / (1 + np.exp(-1.702 * g))
    assert np.all(np.abs(got - want) <= np.abs(want) * 2 ** -10 + 1e-6)
    # gate has no lower bound: a large negative gate is not clamped
    assert O.act_gptoss(np.array([-20.0, 0.0], np.float32))[0] != O.act_gptoss(np.array([-7.0, 0.0], np.float32))[0]


# ---- layout (InstallLayoutTests.swift:14-60, Qwen3SupportTests.swift:81-109) --

def test_gpt_oss_layout():
    lay = ExpertLayout(2880, 2880, 128)
    assert lay.sizes["gate_up_blocks"] == 5760 * 90 * 16
    assert lay.sizes["gate_up_scales"] == 5760 * 90
    assert lay.sizes["down_blocks"] == 2880 * 90 * 16
    assert lay.sizes["down_scales"] == 2880 * 90
    assert lay.sizes["gate_up_bias"] == 5760 * 2 and lay.sizes["down_bias"] == 2880 * 2
    assert 12.6 < lay.payload_per_expert / 2 ** 20 < 12.7
    assert all(o % PAGE == 0 for o in lay.offsets.values()) and lay.stride % PAGE == 0
    assert 1 - lay.payload_per_expert / lay.stride < 0.01
    assert lay.stride == 13_287_424
    assert 56 < lay.layer_file_size * 36 / 2 ** 30 < 58
    assert GPT_OSS_120B.expert_weight_bytes + GPT_OSS_120B.expert_bias_bytes == 13_236_480


def test_qwen3_layout():
    lay = QWEN3_30B_A3B.layout()
    assert [lay.sizes[s] for s in ("gate_up_blocks", "gate_up_scales", "down_blocks",
                                   "down_scales", "gate_up_bias", "down_bias")] == \
        [1_572_864, 98_304, 786_432, 49_152, 3_072, 4_096]
    assert lay.stride == 2_539_520
    assert QWEN3_30B_A3B.expert_weight_bytes == 2_506_752


# ---- Int8Affine (Tests/GodwitTests/InstallLayoutTests.swift:82-125) --------

def test_int8_round_trip_within_half_a_step():  # InstallLayoutTests.swift:85-98
    rng = np.random.default_rng(5)
    row = rng.uniform(-2, 2, 256).astype(np.float32)
    codes, scale, zero = O.int8_quantize_row(row)
    back = codes.reshape(-1, 64).astype(np.float32) * scale[:, None] + zero[:, None]
    step = np.repeat(scale, 64)
    assert np.all(np.abs(back.ravel() - row) <= step * 0.51)


def test_int8_extremes_exact():  # InstallLayoutTests.swift:100-112
    row = np.zeros(64, np.float32)
    row[0], row[63] = -3, 5
    codes, scale, zero = O.int8_quantize_row(row)
    back = codes.astype(np.float32) * scale[0] + zero[0]
    assert abs(back[0] + 3) < 1e-4 and abs(back[63] - 5) < 1e-3
    assert codes[0] == 0 and codes[63] == 255


def test_int8_constant_group_has_positive_scale():  # InstallLayoutTests.swift:114-121
    row = np.full(64, 1.25, np.float32)
    codes, scale, zero = O.int8_quantize_row(row)
    assert scale[0] > 0
    assert np.all(np.abs(np.zeros(64) * scale[0] + zero[0] - 1.25) < 1e-5)


@pytest.mark.parametrize("v", [0.0, 1.0, -1.0, 0.5, 2.0, -0.25, 1024.0])
def test_bf16_round_trips_representable_values(v):  # InstallLayoutTests.swift:123-127
    bits = O.bf16_from_f32(v)
    assert np.array([bits << 16], np.uint32).view(np.float32)[0] == v


def test_bf16_rounds_to_nearest_even_and_keeps_nan():  # Int8Affine.swift:89-96
    assert O.bf16_from_f32(float(np.array([0x3F808000], np.uint32).view(np.float32)[0])) == 0x3F80  # tie -> even
    assert O.bf16_from_f32(float(np.array([0x3F818000], np.uint32).view(np.float32)[0])) == 0x3F82  # tie -> even
    assert O.bf16_from_f32(float(np.array([0x3F808001], np.uint32).view(np.float32)[0])) == 0x3F81
    nan = O.bf16_from_f32(float("nan"))
    assert (nan & 0x7F80) == 0x7F80 and (nan & 0x7F) != 0


def test_int8_quantize_rejects_ragged_rows():  # Int8Affine.swift:32-33 precondition
    with pytest.raises(ValueError):
        O.int8_quantize_row(np.zeros(100, np.float32))


def test_int8_gemv_restatements_agree():
    """The fp32 restatement of router.metal:65-141 against the fp64 one, and
    both against dequantise-then-multiply."""
    rng = np.random.default_rng(9)
    w = rng.normal(0, 0.02, (48, 320)).astype(np.float32)
    codes, meta = O.int8_quantize(w)
    x = rng.standard_normal((3, 320)).astype(np.float16).astype(np.float32)
    bias = np.array([O.bf16_from_f32(v) for v in rng.normal(0, 0.02, 48)], np.uint16)
    y32 = O.int8_gemv(codes, meta, x, bias, threads=2)
    y64 = O.int8_gemv64(codes, meta, x, bias)
    assert O.rel_l2(y32, y64) < 1e-6
    dq = O.int8_dequant(codes, meta).astype(np.float64)
    b = (bias.astype(np.uint32) << 16).view(np.float32)
    assert O.rel_l2(x.astype(np.float64) @ dq.T + b, y64) < 1e-6
