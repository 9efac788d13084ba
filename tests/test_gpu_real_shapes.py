"""Parity at the BASELINE configurations' real shapes, through the C-ABI.

Every config is run with its full expert count and its real H / F / top-k
(GPT-OSS-20B E=32; GPT-OSS-120B E=128; Qwen3-30B-A3B E=128 top-8; the
GPT-OSS-120B prefill layer at 2048 tokens with the bench's 4x hot-expert
skew), on the seeded synthetic bank the bench uses (gw_bank_fill_synthetic),
over 2-4 layers (the CPU oracle bounds the cost; every layer of a stack has
the same shape).  The oracle reads back the exact resident bytes of each
routed expert (gw_bank_download_expert, itself checked byte-exact against the
reference stride elsewhere) and the router weights are the host-made ones the
test uploads, so host and device hold identical inputs.

Checks and tolerances (written here, per check):
  * routing: top-k ids identical to the fp32 oracle router (Router.select's
    selection-sort rule), except tokens whose k-th / (k+1)-th oracle logits are
    within 1e-4 (flagged near-ties: the device sums in another order); the
    number of flagged tokens is reported.
  * layer output vs the fp64 restatement under the device's own routing:
    rel-L2 <= 1e-3, plus the reference's own layer gate
    (Sources/GodwitCLI/main.swift:690-720: relative RMS error < 2e-3 and every
    |error| / RMS(y) below 4 * max|y| * 2^-11 / RMS(y)).
  * block-scaled prefill vs the fp64 restatement of the same MXFP8
    quantisation (oracle.moe_layer64_mx): rel-L2 <= 1e-3.
"""
import os
import sys

import numpy as np
import oracle as O
import pytest

from godwit_b200 import synth
from godwit_b200.layout import GPT_OSS_20B, GPT_OSS_120B, QWEN3_30B_A3B
from godwit_b200.runtime import ExpertBank, MoEBlock

pytestmark = pytest.mark.gpu
SEED = 7
THREADS = os.cpu_count() or 1


class ResidentStrides:
    """expert id -> the stride the device holds for one layer (downloaded on
    first use and cached; a dict-like view for the oracle functions)."""

    def __init__(self, bank, layer):
        self.bank, self.layer, self.cache = bank, layer, {}

    def __getitem__(self, e):
        e = int(e)
        if e not in self.cache:
            self.cache[e] = self.bank.download_expert(self.layer, e)
        return self.cache[e]


def make_bank(ctx, spec, layers, seed=SEED):
    bank = ExpertBank(ctx, spec, layers=layers)
    bank.fill_synthetic(seed)
    routers = []
    for l in range(layers):
        w, b = synth.hash_router(spec, seed + 1000, l)  # host-made router, uploaded as is
        b = b if spec.router_bias else None
        bank.upload_router(l, w, b)
        routers.append((w, b))
    return bank, routers


def oracle_routing(spec, router, x):
    """fp32 oracle logits [T, E] and top-k [T, k] (Router.logits / select)."""
    w, b = router
    logits = np.stack([O.router_logits(w, b, x[t]) for t in range(x.shape[0])])
    ex = np.stack([O.router_select(logits[t], spec.top_k)[0] for t in range(x.shape[0])])
    return logits, ex


def check_routing(ex, ref_ex, logits, k):
    """Identical top-k except flagged near-ties; returns the flagged count."""
    flagged = 0
    for t in range(ex.shape[0]):
        if list(ex[t]) == list(ref_ex[t]):
            continue
        srt = np.sort(logits[t])[::-1]
        assert np.abs(np.diff(srt[:k + 1])).min() < 1e-4, \
            f"token {t}: device {list(ex[t])} vs oracle {list(ref_ex[t])} with no near-tie"
        flagged += 1
    return flagged


def layer_gate(out, ref):
    """The reference's layer gate (GodwitCLI main.swift:700-720) on fp32 data."""
    y = np.asarray(ref, np.float64).ravel()
    d = np.asarray(out, np.float64).ravel() - y
    rms = max(np.sqrt(np.mean(y * y)), 1e-6)
    rel_rms = np.sqrt(np.mean(d * d)) / rms
    worst = np.max(np.abs(d)) / rms
    bound = 4 * np.max(np.abs(y)) * 2.0 ** -11 / rms
    return rel_rms, worst, bound


def run_layer_case(ctx, bank, routers, spec, layer, T, seed):
    rng = np.random.default_rng(seed)
    xb = synth.make_hidden(rng, T, spec.hidden, "bf16")
    x = synth.as_f32(xb, "bf16")
    out, ex, wt = MoEBlock(ctx, bank).forward(xb, layer, "bf16")
    logits, ref_ex = oracle_routing(spec, routers[layer], x)
    flagged = check_routing(ex, ref_ex, logits, spec.top_k)
    assert flagged <= max(1, T // 100), f"{flagged} near-tie flips in {T} tokens"
    # the device's routing weights are the softmax over its own top-k logits
    for t in range(T):
        sel = logits[t][ex[t]].astype(np.float64)
        p = np.exp(sel - sel.max())
        assert np.allclose(wt[t], p / p.sum(), rtol=1e-5, atol=1e-6)
    ref64 = O.moe_layer64(spec, ResidentStrides(bank, layer), x, ex, wt)
    assert O.rel_l2(out, ref64) <= 1e-3
    rel_rms, worst, bound = layer_gate(out, ref64)
    assert rel_rms < 2e-3 and worst < bound, (rel_rms, worst, bound)
    return out, ex, wt


# ---- config 1: GPT-OSS-20B (E = 32, top-4) --------------------------------------

@pytest.fixture(scope="module")
def oss20(ctx):
    bank, routers = make_bank(ctx, GPT_OSS_20B.with_(layers=3), 3)
    yield bank, routers
    bank.close()


@pytest.mark.parametrize("T", [1, 16])
def test_config1_oss20_layers(ctx, oss20, T):
    bank, routers = oss20
    for layer in (0, 2):
        run_layer_case(ctx, bank, routers, bank.spec, layer, T, 1000 + 10 * T + layer)


# ---- config 2: GPT-OSS-120B (E = 128, top-4) --------------------------------------

@pytest.fixture(scope="module")
def oss120(ctx):
    bank, routers = make_bank(ctx, GPT_OSS_120B.with_(layers=4), 4)
    yield bank, routers
    bank.close()


@pytest.mark.parametrize("T,layer", [(1, 0), (1, 3), (64, 1), (64, 2)])
def test_config2_oss120_layers(ctx, oss120, T, layer):
    bank, routers = oss120
    run_layer_case(ctx, bank, routers, bank.spec, layer, T, 2000 + T + layer)


def test_config2_oss120_graph_stack_vs_fp64_chain(ctx, oss120):
    """gw_moe_stack_forward_async (graph-captured, 4 layers, residual chaining,
    identity norm) against a host-side fp64 chain: stream = x; per layer,
    stream += fp64 layer(bf16(stream)).  Without a norm between layers the
    stream grows to |x| ~ 1e2-1e3, where an fp32 rounding difference can move
    a bf16 input by one ulp; so the fp64 chain applies, per layer, the routing
    the device chose on its own chain (read from an eager per-layer replay,
    which must equal the graph), and that routing is checked against the fp32
    oracle router on the host chain's inputs (near-ties flagged)."""
    import torch
    from godwit_b200 import device as D
    bank, routers = oss120
    spec = bank.spec
    T = 4
    rng = np.random.default_rng(2222)
    xb = synth.make_hidden(rng, T, spec.hidden, "bf16")
    x_dev = torch.from_numpy(xb.view(np.int16)).cuda().view(torch.bfloat16)
    stream = torch.empty(T, spec.hidden, dtype=torch.float32, device="cuda")
    D.bind_stream(ctx)
    try:
        for _ in range(2):  # capture, then a replay of the captured graph
            D.moe_stack(ctx, bank, x_dev, stream)
            torch.cuda.synchronize()
        got = stream.cpu().numpy()
    finally:
        ctx.set_stream(None)
    # eager per-layer replay on the device (fp32 stream, bf16 layer inputs);
    # the fp64 chain runs each layer on the same bf16 inputs, under the routing
    # the device chose there (checked against the fp32 oracle router on those
    # inputs), and accumulates the stream in fp64
    s32 = synth.as_f32(xb, "bf16").astype(np.float32)
    s64 = s32.astype(np.float64)
    for l in range(bank.layers):
        xd = synth.f32_to_bf16_bits(s32)
        out, ex, wt = MoEBlock(ctx, bank).forward(xd, l, "bf16")
        xl = synth.bf16_bits_to_f32(xd)
        logits, ref_ex = oracle_routing(spec, routers[l], xl)
        check_routing(ex, ref_ex, logits, spec.top_k)
        y64 = O.moe_layer64(spec, ResidentStrides(bank, l), xl, ex, wt)
        assert O.rel_l2(out, y64) <= 1e-3, f"layer {l}"
        s32 = s32 + out
        s64 = s64 + y64
    assert O.rel_l2(got, s32) <= 1e-5, "graph replay differs from the eager layer sequence"
    assert O.rel_l2(got, s64) <= 1e-3
    rel_rms, worst, bound = layer_gate(got, s64)
    assert rel_rms < 2e-3 and worst < bound, (rel_rms, worst, bound)


# ---- config 3: Qwen3-30B-A3B (E = 128, top-8, SiLU, no biases) ----------------------

@pytest.fixture(scope="module")
def qwen3(ctx):
    bank, routers = make_bank(ctx, QWEN3_30B_A3B.with_(layers=2), 2)
    yield bank, routers
    bank.close()


@pytest.mark.parametrize("T,layer", [(1, 0), (32, 1)])
def test_config3_qwen3_layers(ctx, qwen3, T, layer):
    bank, routers = qwen3
    out, ex, wt = run_layer_case(ctx, bank, routers, bank.spec, layer, T, 3000 + T + layer)
    assert np.allclose(wt.sum(1), 1.0, atol=1e-5)  # renormalised over the 8


# ---- config 4: GPT-OSS-120B prefill layer, 2048 tokens, 4x skew --------------------

@pytest.mark.parametrize("block_scaled", [True, False])
def test_config4_prefill_layer(ctx, block_scaled):
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from bench import HOT_EXPERTS, skewed_router_bias
    spec = GPT_OSS_120B.with_(layers=1)
    T = 2048
    bank = ExpertBank(ctx, spec, layers=1)
    try:
        bank.fill_synthetic(SEED)
        rng = np.random.default_rng(4000)
        xb = synth.make_hidden(rng, T, spec.hidden, "bf16")
        x = synth.as_f32(xb, "bf16")
        rb, _, hist = skewed_router_bias(spec, x, seed=SEED)
        rw, _ = synth.hash_router(spec, SEED, 0)
        bank.upload_router(0, rw, rb)
        mean = T * spec.top_k / spec.experts
        assert hist[list(HOT_EXPERTS)].mean() >= 3.5 * mean  # the skew is there
        ctx.set_block_scaled(block_scaled)
        out, ex, wt = MoEBlock(ctx, bank).forward(xb, 0, "bf16")
        logits, ref_ex = oracle_routing(spec, (rw, rb), x)
        flagged = check_routing(ex, ref_ex, logits, spec.top_k)
        assert flagged <= T // 100
        strides = ResidentStrides(bank, 0)
        if block_scaled:
            ref = O.moe_layer64_mx(spec, strides, x, ex, wt)
        else:
            ref = O.moe_layer64(spec, strides, x, ex, wt)
        assert O.rel_l2(out, ref) <= 1e-3
    finally:
        ctx.set_block_scaled(False)
        bank.close()
