"""The streamed decode GEMVs (gw_stream.cu) against the per-thread-load GEMV
tiles they replace: the same tile arithmetic, summed in a different order
(independent MMA chains per group here, K split across warps there when few
experts are active), so the layers agree to rel-L2 < 2e-5, and the fp64 oracle
(rel-L2 < 1e-3), for one token, odd token counts, token counts
that need several 4-token chunks per expert, both activations (GPT-OSS
clamped GLU with biases; Qwen3 SiLU without), and a 128-row tile that runs
past the matrix (down rows 2880)."""
import numpy as np
import oracle as O
import pytest

from godwit_b200 import synth
from godwit_b200.layout import GPT_OSS_20B, QWEN3_30B_A3B
from godwit_b200.runtime import ExpertBank, MoEBlock

pytestmark = pytest.mark.gpu


def make_bank(ctx, spec, seed):
    rng = np.random.default_rng(seed)
    bank = ExpertBank(ctx, spec, layers=1)
    st = np.stack([synth.make_expert_stride(spec, rng) for _ in range(spec.experts)])
    for e in range(spec.experts):
        bank.upload_expert(0, e, st[e])
    w, b = synth.make_router(spec, rng)
    bank.upload_router(0, w, b)
    return bank, st


def both(ctx, bank, xb, routing=None):
    blk = MoEBlock(ctx, bank)
    try:
        ctx.set_tensor_core_min_tokens(0)  # keep every size on the GEMV tiles
        ctx.set_decode_streaming(True)
        out_s, ex, wt = blk.forward(xb, 0, "bf16", routing=routing)
        ctx.set_decode_streaming(False)
        out_t, _, _ = blk.forward(xb, 0, "bf16", routing=(ex, wt))
    finally:
        ctx.set_decode_streaming(False)
        ctx.set_tensor_core_min_tokens(8)
    return out_s, out_t, ex, wt


@pytest.fixture(scope="module")
def oss(ctx):
    bank, st = make_bank(ctx, GPT_OSS_20B.with_(experts=8, layers=1), 515)
    yield bank, st
    bank.close()


@pytest.mark.parametrize("T", [1, 3, 6, 40])
def test_streamed_matches_tiles(ctx, oss, T):
    bank, st = oss
    spec = bank.spec
    xb = synth.make_hidden(np.random.default_rng(T), T, spec.hidden, "bf16")
    out_s, out_t, ex, wt = both(ctx, bank, xb)
    assert O.rel_l2(out_s, out_t) < 2e-5
    ref = O.moe_layer64(spec, st, synth.as_f32(xb, "bf16"), ex, wt)
    assert O.rel_l2(out_s, ref) < 1e-3


def test_streamed_many_tokens_on_one_expert(ctx, oss):
    """Every token on experts 0-3: 13 tokens each, four 4-token chunks."""
    bank, st = oss
    spec = bank.spec
    rng = np.random.default_rng(3)
    T = 13
    xb = synth.make_hidden(rng, T, spec.hidden, "bf16")
    ex = np.tile(np.arange(4, dtype=np.int32), (T, 1))
    wt = rng.dirichlet(np.ones(4), T).astype(np.float32)
    out_s, out_t, _, _ = both(ctx, bank, xb, routing=(ex, wt))
    assert O.rel_l2(out_s, out_t) < 2e-5
    assert O.rel_l2(out_s, O.moe_layer64(spec, st, synth.as_f32(xb, "bf16"), ex, wt)) < 1e-3


def test_streamed_qwen3_silu(ctx):
    bank, st = make_bank(ctx, QWEN3_30B_A3B.with_(experts=16, layers=1), 99)
    try:
        spec = bank.spec
        xb = synth.make_hidden(np.random.default_rng(4), 9, spec.hidden, "bf16")
        out_s, out_t, ex, wt = both(ctx, bank, xb)
        assert O.rel_l2(out_s, out_t) < 2e-5
        assert O.rel_l2(out_s, O.moe_layer64(spec, st, synth.as_f32(xb, "bf16"), ex, wt)) < 1e-3
    finally:
        bank.close()
