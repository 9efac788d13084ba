"""Parity of the tensor-core grouped expert GEMMs (gw_grouped.cu).

The tcgen05 path replaces, for layers with many tokens per expert, the
reference's per-assignment GEMVs (ExpertRunner.applyAssignments,
Runtime/ExpertRunner.swift:108-183).  Its results are checked three ways:
against the fp64 restatement of the expert FFN under the device's own routing
(rel-L2 < 1e-3), against the GEMV path on the same inputs (they differ only
in fp32 summation order and the rare f16 rounding of the activation that
follows from it), and through the cases the tiling has edges for: more than
128 tokens on one expert (several token chunks), a 128-row tile that runs
past the matrix (down rows 2880 = 22.5 tiles), a SiLU model without router
bias (Qwen3 shapes), and weight rows whose block scales span 16 binades.
"""
import numpy as np
import oracle as O
import pytest

from godwit_b200 import synth
from godwit_b200.layout import GPT_OSS_20B, QWEN3_30B_A3B
from godwit_b200.runtime import ExpertBank, MoEBlock

pytestmark = pytest.mark.gpu

SMALL_OSS = GPT_OSS_20B.with_(experts=8, layers=1)
SMALL_QWEN = QWEN3_30B_A3B.with_(experts=16, layers=1)


def make_bank(ctx, spec, seed, mutate=None):
    rng = np.random.default_rng(seed)
    bank = ExpertBank(ctx, spec, layers=1)
    st = np.stack([synth.make_expert_stride(spec, rng) for _ in range(spec.experts)])
    if mutate is not None:
        mutate(st, rng)
    for e in range(spec.experts):
        bank.upload_expert(0, e, st[e])
    w, b = synth.make_router(spec, rng)
    bank.upload_router(0, w, b)
    return bank, st, (w, b)


def both_paths(ctx, bank, xb, dtype="bf16", routing=None):
    blk = MoEBlock(ctx, bank)
    try:
        ctx.set_tensor_core_min_tokens(1)
        out_tc, ex, wt = blk.forward(xb, 0, dtype, routing=routing)
        ctx.set_tensor_core_min_tokens(0)
        out_gv, ex2, wt2 = blk.forward(xb, 0, dtype, routing=(ex, wt))
    finally:
        ctx.set_tensor_core_min_tokens(8)
    assert np.array_equal(ex, ex2)
    return out_tc, out_gv, ex, wt


@pytest.fixture(scope="module")
def oss(ctx):
    bank, st, router = make_bank(ctx, SMALL_OSS, 4242)
    yield bank, st, router
    bank.close()


@pytest.mark.parametrize("T", [16, 200, 700])
def test_grouped_matches_oracle_and_gemv(ctx, oss, T):
    bank, st, _ = oss
    spec = bank.spec
    rng = np.random.default_rng(T)
    xb = synth.make_hidden(rng, T, spec.hidden, "bf16")
    out_tc, out_gv, ex, wt = both_paths(ctx, bank, xb)
    assert np.all(np.isfinite(out_tc))
    ref = O.moe_layer64(spec, st, synth.as_f32(xb, "bf16"), ex, wt)
    assert O.rel_l2(out_tc, ref) < 1e-3
    assert O.rel_l2(out_tc, out_gv) < 2e-4
    if T == 700:  # 350 tokens per expert on average: three token chunks each
        assert np.bincount(ex.ravel(), minlength=spec.experts).max() > 256


def test_grouped_f16_input(ctx, oss):
    bank, st, _ = oss
    spec = bank.spec
    rng = np.random.default_rng(5)
    xb = synth.make_hidden(rng, 96, spec.hidden, "f16")
    out_tc, out_gv, ex, wt = both_paths(ctx, bank, xb, "f16")
    ref = O.moe_layer64(spec, st, synth.as_f32(xb, "f16"), ex, wt)
    assert O.rel_l2(out_tc, ref) < 1e-3
    assert O.rel_l2(out_tc, out_gv) < 2e-4


def test_grouped_one_hot_expert(ctx, oss):
    """Every token on experts 0-3, 300 tokens: experts 4-7 idle, each busy
    expert three token chunks (128 + 128 + 44)."""
    bank, st, _ = oss
    spec = bank.spec
    rng = np.random.default_rng(9)
    T = 300
    xb = synth.make_hidden(rng, T, spec.hidden, "bf16")
    ex = np.tile(np.arange(4, dtype=np.int32), (T, 1))
    wt = rng.dirichlet(np.ones(4), T).astype(np.float32)
    out_tc, out_gv, _, _ = both_paths(ctx, bank, xb, routing=(ex, wt))
    ref = O.moe_layer64(spec, st, synth.as_f32(xb, "bf16"), ex, wt)
    assert O.rel_l2(out_tc, ref) < 1e-3
    assert O.rel_l2(out_tc, out_gv) < 2e-4


def test_grouped_qwen3_silu(ctx):
    bank, st, (w, b) = make_bank(ctx, SMALL_QWEN, 77)
    try:
        spec = bank.spec
        assert b is None
        rng = np.random.default_rng(78)
        xb = synth.make_hidden(rng, 64, spec.hidden, "bf16")
        out_tc, out_gv, ex, wt = both_paths(ctx, bank, xb)
        ref = O.moe_layer64(spec, st, synth.as_f32(xb, "bf16"), ex, wt)
        assert O.rel_l2(out_tc, ref) < 1e-3
        assert O.rel_l2(out_tc, out_gv) < 2e-4
    finally:
        bank.close()


def test_grouped_wide_scale_range(ctx):
    """Block scales drawn from 2^8..2^23 (16 binades within a row, several
    times what MXFP4 checkpoints hold) with 1% zero bytes: the per-row
    exponent shift keeps the f16 operands exact.  Wider random spreads are
    not a kernel property this test can pin: with 30+ binades of random-sign
    blocks some gate sums cancel from ~1e8 down to O(1), and then the tensor
    core's fp32 accumulation (not correctly rounded per add) and the GEMV's
    per-block exact partials differ by O(1) on those elements."""
    def widen(st, rng):
        lay = SMALL_OSS.layout()
        for name in ("gate_up_scales", "down_scales"):
            o, n = lay.offsets[name], lay.sizes[name]
            s = rng.integers(135, 151, size=(st.shape[0], n)).astype(np.uint8)
            s[rng.random(s.shape) < 0.01] = 0
            st[:, o:o + n] = s

    bank, st, _ = make_bank(ctx, SMALL_OSS, 31, mutate=widen)
    try:
        spec = bank.spec
        rng = np.random.default_rng(32)
        xb = synth.make_hidden(rng, 128, spec.hidden, "bf16")
        out_tc, out_gv, ex, wt = both_paths(ctx, bank, xb)
        ref = O.moe_layer64(spec, st, synth.as_f32(xb, "bf16"), ex, wt)
        assert np.all(np.isfinite(out_tc))
        assert O.rel_l2(out_tc, ref) < 1e-5
        assert O.rel_l2(out_tc, out_gv) < 1e-5
    finally:
        bank.close()


def test_default_policy_switches_on_tokens_per_expert(ctx, oss):
    """Default: tensor cores once T * k >= 8 * experts (here T >= 16)."""
    bank, st, _ = oss
    spec = bank.spec
    rng = np.random.default_rng(12)
    for T in (8, 32):
        xb = synth.make_hidden(rng, T, spec.hidden, "bf16")
        out, ex, wt = MoEBlock(ctx, bank).forward(xb, 0, "bf16")
        ref = O.moe_layer64(spec, st, synth.as_f32(xb, "bf16"), ex, wt)
        assert O.rel_l2(out, ref) < 1e-3


# ---- block-scaled mode (gw_set_block_scaled): MXFP4 x MXFP8 tcgen05 MMAs ----

def block_scaled(ctx, bank, xb, routing=None):
    blk = MoEBlock(ctx, bank)
    try:
        ctx.set_tensor_core_min_tokens(1)
        ctx.set_block_scaled(True)
        return blk.forward(xb, 0, "bf16", routing=routing)
    finally:
        ctx.set_block_scaled(False)
        ctx.set_tensor_core_min_tokens(8)


@pytest.mark.parametrize("T", [16, 200, 700])
def test_block_scaled_matches_quantised_oracle(ctx, oss, T):
    """Exact oracle: the fp64 layer with the same MXFP8 quantisation of the
    expert inputs and of the f16 activations (oracle.moe_layer64_mx)."""
    bank, st, _ = oss
    spec = bank.spec
    rng = np.random.default_rng(100 + T)
    xb = synth.make_hidden(rng, T, spec.hidden, "bf16")
    out, ex, wt = block_scaled(ctx, bank, xb)
    x = synth.as_f32(xb, "bf16")
    assert np.all(np.isfinite(out))
    assert O.rel_l2(out, O.moe_layer64_mx(spec, st, x, ex, wt)) < 1e-3
    # and the deviation from the reference's f16-activation numerics: two
    # E4M3 quantisations (3 mantissa bits, ~3.6% RMS each) give ~5.7%
    assert O.rel_l2(out, O.moe_layer64(spec, st, x, ex, wt)) < 8e-2


def test_block_scaled_qwen3(ctx):
    bank, st, _ = make_bank(ctx, SMALL_QWEN, 501)
    try:
        spec = bank.spec
        xb = synth.make_hidden(np.random.default_rng(502), 96, spec.hidden, "bf16")
        out, ex, wt = block_scaled(ctx, bank, xb)
        assert O.rel_l2(out, O.moe_layer64_mx(spec, st, synth.as_f32(xb, "bf16"), ex, wt)) < 1e-3
    finally:
        bank.close()
