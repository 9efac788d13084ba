"""Parity of the CUDA path (through the C-ABI) against the CPU oracle.

Tolerances (written here, per check):
  * dequant: bit-exact (NaN positions identical).
  * GEMV: max |y - ref| / max(|ref|, 1) < 1e-3 — DequantGEMVTests.swift:20-42.
  * router logits: |diff| <= 1e-4 * (1 + |ref|) (fp32 sums in another order);
    top-k indices identical except where the oracle's k-th/(k+1)-th logit gap
    is below 1e-4 (flagged near-ties).
  * expert / layer: rel-L2 <= 1e-3 against the fp64 restatement (BASELINE
    target) and max |diff| / mean|ref| < 5e-3 against the fp32 oracle
    (check-expert, main.swift:518-533).
"""
import os

import numpy as np
import oracle as O
import pytest

from godwit_b200 import synth
from godwit_b200._abi import GW_E_ARG, GodwitCUDAError
from godwit_b200.layout import GPT_OSS_20B, QWEN3_30B_A3B
from godwit_b200.runtime import ExpertBank, ExpertRunner, MoEBlock, Router

pytestmark = pytest.mark.gpu


def gemv_err(y, ref):
    return float(np.max(np.abs(y.astype(np.float64) - ref) / np.maximum(np.abs(ref), 1.0)))


# ---- dequant -----------------------------------------------------------------

def test_dequant_bit_exact(ctx):
    rng = np.random.default_rng(11)
    rows, cols = 67, 320
    p = rng.integers(0, 256, (rows, cols // 2), dtype=np.uint8)
    s = rng.integers(0, 256, (rows, cols // 32), dtype=np.uint8)
    s[0, :4] = [0, 1, 254, 255]
    w = ctx.mxfp4_dequant(p, s)
    ref = O.dequant(p, s)
    nan = np.isnan(ref)
    assert np.array_equal(np.isnan(w), nan)
    assert np.array_equal(w[~nan].view(np.uint32), ref[~nan].view(np.uint32))


# ---- GEMV (config 0 and the reference's GEMV tests) ---------------------------

@pytest.mark.parametrize("rows,cols,dtype,bias", [
    (64, 256, "f16", False),      # DequantGEMVTests.swift:20-31
    (32, 2880, "f16", False),     # DequantGEMVTests.swift:33-42
    (2880, 2880, "bf16", True),   # config 0
    (37, 96, "bf16", True),       # ragged rows, odd block count
    (5760, 2880, "f16", True),    # gate_up shape
])
def test_gemv_matches_oracle(ctx, rows, cols, dtype, bias):
    rng = np.random.default_rng(rows * 7 + cols)
    p, s = synth.random_mxfp4(rng, rows, cols)
    xb = synth.make_hidden(rng, 1, cols, dtype)[0]
    b = synth.f32_to_bf16_bits(rng.normal(0, 0.02, rows)) if bias else None
    y = ctx.mxfp4_gemv(p, s, xb, bias=b, dtype=dtype)
    x = synth.as_f32(xb, dtype)
    ref = O.gemv(p, s, x, None if b is None else synth.bf16_bits_to_f32(b))
    assert gemv_err(y, ref) < 1e-3


def test_gemv_hand_case(ctx):  # DequantGEMVTests.swift:64-77
    y = ctx.mxfp4_gemv(np.full((1, 16), 0x22, np.uint8), np.array([[127]], np.uint8),
                       np.ones(32, np.float16), dtype="f16")
    assert abs(y[0] - 32.0) < 1e-4


def test_gemv_wide_scale_range(ctx):
    rng = np.random.default_rng(5)
    p, s = synth.random_mxfp4(rng, 48, 512, lo=100, hi=150)
    xb = synth.make_hidden(rng, 1, 512, "bf16")[0]
    y = ctx.mxfp4_gemv(p, s, xb, dtype="bf16")
    ref = O.dequant64(p, s) @ synth.as_f32(xb, "bf16").astype(np.float64)
    assert np.max(np.abs(y - ref) / np.maximum(np.abs(ref), 1e-30 + np.abs(ref).max() * 1e-6)) < 1e-3


def test_gemv_rejects_bad_shapes(ctx):
    with pytest.raises(GodwitCUDAError) as e:
        ctx.mxfp4_gemv(np.zeros((4, 8), np.uint8), np.zeros((4, 1), np.uint8), np.zeros(16, np.float16))
    assert e.value.status == GW_E_ARG


# ---- bank fixtures -------------------------------------------------------------

def build_bank(ctx, spec, seed, layers=1, shard=(0, 1)):
    rng = np.random.default_rng(seed)
    bank = ExpertBank(ctx, spec, layers=layers, shard_rank=shard[0], shard_count=shard[1])
    strides, routers = [], []
    for l in range(layers):
        st = np.stack([synth.make_expert_stride(spec, rng) for _ in range(spec.experts)])
        w, b = synth.make_router(spec, rng)
        for e in range(spec.experts):
            if bank.owns(e):
                bank.upload_expert(l, e, st[e])
        bank.upload_router(l, w, b)
        strides.append(st)
        routers.append((w, b))
    return bank, strides, routers


SMALL_OSS = GPT_OSS_20B.with_(experts=8, layers=2)
SMALL_QWEN = QWEN3_30B_A3B.with_(experts=16, layers=2)


@pytest.fixture(scope="module")
def oss_bank(ctx):
    bank, strides, routers = build_bank(ctx, SMALL_OSS, 101, layers=2)
    yield bank, strides, routers
    bank.close()


@pytest.fixture(scope="module")
def qwen_bank(ctx):
    bank, strides, routers = build_bank(ctx, SMALL_QWEN, 202, layers=1)
    yield bank, strides, routers
    bank.close()


# ---- router ---------------------------------------------------------------------

def check_topk(ex, ref_ex, logits_ref, k):
    for t in range(ex.shape[0]):
        if list(ex[t]) == list(ref_ex[t]):
            continue
        srt = np.sort(logits_ref[t])[::-1]
        gaps = np.abs(np.diff(srt[:k + 1]))
        assert gaps.min() < 1e-4, f"token {t}: {ex[t]} vs {ref_ex[t]} with no near-tie"


@pytest.mark.parametrize("T,dtype", [(1, "bf16"), (7, "f16"), (64, "bf16")])
def test_router_matches_oracle(ctx, oss_bank, T, dtype):
    bank, strides, routers = oss_bank
    spec = bank.spec
    rng = np.random.default_rng(T)
    xb = synth.make_hidden(rng, T, spec.hidden, dtype)
    x = synth.as_f32(xb, dtype)
    r = Router(ctx, bank)
    lg = r.logits(xb, 1, dtype)
    w, b = routers[1]
    ref = np.stack([O.router_logits(w, b, x[t]) for t in range(T)])
    assert np.all(np.abs(lg - ref) <= 1e-4 * (1 + np.abs(ref)))
    ex, wt = r.route_batch(xb, 1, dtype)
    ref_ex = np.zeros_like(ex)
    for t in range(T):
        e, ww = O.router_select(ref[t], spec.top_k)
        ref_ex[t] = e
        if list(ex[t]) == list(e):
            assert np.allclose(wt[t], ww, rtol=1e-5, atol=1e-6)
    check_topk(ex, ref_ex, ref, spec.top_k)


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_router_logits_do_not_depend_on_the_batch(ctx, oss_bank, dtype):
    """A token's logits and routing are bit-identical whether it is routed
    alone, in a single 8-token chunk or in a larger batch (the router's warp
    count changes with the batch; its summation order does not), as the
    reference routes each token on its own (Router.swift:100-104)."""
    bank, _, _ = oss_bank
    spec = bank.spec
    rng = np.random.default_rng(31)
    xb = synth.make_hidden(rng, 27, spec.hidden, dtype)
    r = Router(ctx, bank)
    full = r.logits(xb, 1, dtype)
    ex_full, wt_full = r.route_batch(xb, 1, dtype)
    for a, b in [(0, 1), (3, 9), (9, 27)]:
        part = r.logits(xb[a:b], 1, dtype)
        assert np.array_equal(part, full[a:b])
        ex, wt = r.route_batch(xb[a:b], 1, dtype)
        assert np.array_equal(ex, ex_full[a:b]) and np.array_equal(wt, wt_full[a:b])


@pytest.mark.parametrize("E,T", [(32, 128), (128, 300), (128, 2048)])
def test_batch_router_matches_oracle(ctx, E, T):
    """Large bf16 batches take the tensor-core router (k_router_mma): same
    logits up to summation order, same top-k (near-ties excepted), same x16."""
    spec = GPT_OSS_20B.with_(experts=E, layers=1)
    bank = ExpertBank(ctx, spec, layers=1)
    try:
        rng = np.random.default_rng(E + T)
        w, b = synth.make_router(spec, rng)
        bank.upload_router(0, w, b)
        xb = synth.make_hidden(rng, T, spec.hidden, "bf16")
        x = synth.as_f32(xb, "bf16")
        r = Router(ctx, bank)
        lg = r.logits(xb, 0, "bf16")
        ref = np.stack([O.router_logits(w, b, x[t]) for t in range(T)])
        assert np.all(np.abs(lg - ref) <= 1e-4 * (1 + np.abs(ref)))
        ex, wt = r.route_batch(xb, 0, "bf16")
        ref_ex = np.zeros_like(ex)
        for t in range(T):
            e, ww = O.router_select(ref[t], spec.top_k)
            ref_ex[t] = e
            if list(ex[t]) == list(e):
                assert np.allclose(wt[t], ww, rtol=1e-5, atol=1e-6)
        check_topk(ex, ref_ex, ref, spec.top_k)
        assert np.mean(np.all(ex == ref_ex, axis=1)) > 0.99
    finally:
        bank.close()


def test_router_tie_rule_on_device(ctx):
    # Router weights that give exact logit ties: experts 0 and 1 tie at 1.0,
    # expert 2 wins with 5.0 — Router.select returns [2, 1], not [2, 0].
    spec = GPT_OSS_20B.with_(experts=3, top_k=2, layers=1, hidden=64, intermediate=32)
    bank = ExpertBank(ctx, spec, layers=1)
    try:
        w = np.zeros((3, 64), np.float32)
        w[0, 0], w[1, 0], w[2, 0] = 1.0, 1.0, 5.0
        bank.upload_router(0, synth.f32_to_bf16_bits(w), None)
        x = np.zeros(64, np.float16)
        x[0] = 1.0
        d = Router(ctx, bank).route(x, 0, "f16")
        assert d.experts == [2, 1]
        ref_e, ref_w = O.router_select(np.array([1.0, 1.0, 5.0], np.float32), 2)
        assert list(ref_e) == d.experts and np.allclose(ref_w, d.weights, rtol=1e-6)
    finally:
        bank.close()


# ---- experts ------------------------------------------------------------------

def test_expert_apply_matches_oracle(ctx, oss_bank):
    bank, strides, _ = oss_bank
    spec = bank.spec
    runner = ExpertRunner(ctx, bank)
    rng = np.random.default_rng(9)
    for e in (0, 5):
        xb = synth.make_hidden(rng, 1, spec.hidden, "f16")[0]
        x = synth.as_f32(xb, "f16")
        y = runner.apply(xb, 0, e, "f16")
        ref = O.expert_apply(spec, strides[0][e], x)
        assert np.max(np.abs(y - ref)) / np.mean(np.abs(ref)) < 5e-3
        assert O.rel_l2(y, O.expert64(spec, strides[0][e], x)) < 1e-3


def test_apply_batch_matches_weighted_sum(ctx, oss_bank):
    bank, strides, _ = oss_bank
    spec = bank.spec
    runner = ExpertRunner(ctx, bank)
    xb = synth.make_hidden(np.random.default_rng(4), 1, spec.hidden, "bf16")[0]
    x = synth.as_f32(xb, "bf16")
    pairs = [(3, 0.5), (1, 0.3), (6, 0.2)]
    y = runner.apply_batch(xb, 0, pairs, "bf16")
    ref = sum(w * O.expert64(spec, strides[0][e], x) for e, w in pairs)
    assert O.rel_l2(y, ref) < 1e-3
    assert np.all(runner.apply_batch(xb, 0, [], "bf16") == 0)


@pytest.mark.parametrize("T,dtype", [(1, "bf16"), (5, "f16"), (64, "bf16")])
def test_moe_layer_matches_oracle(ctx, oss_bank, T, dtype):
    bank, strides, routers = oss_bank
    spec = bank.spec
    rng = np.random.default_rng(100 + T)
    xb = synth.make_hidden(rng, T, spec.hidden, dtype)
    x = synth.as_f32(xb, dtype)
    out, ex, wt = MoEBlock(ctx, bank).forward(xb, 1, dtype)
    w, b = routers[1]
    ref_out, ref_ex, ref_wt = O.moe_layer(spec, strides[1], w, b, x, threads=os.cpu_count() or 1)
    logits = np.stack([O.router_logits(w, b, x[t]) for t in range(T)])
    check_topk(ex, ref_ex, logits, spec.top_k)
    same = np.all(ex == ref_ex, axis=1)
    assert same.mean() > 0.9
    # compare outputs under the device's own routing decision
    ref64 = O.moe_layer64(spec, strides[1], x, ex, wt)
    assert O.rel_l2(out, ref64) < 1e-3
    if T <= 8:
        ref32 = O.moe_layer(spec, strides[1], w, b, x, routing=(ex, wt))[0]
        assert np.max(np.abs(out - ref32)) / np.mean(np.abs(ref32)) < 5e-3
    assert O.rel_l2(out[same], ref_out[same]) < 1e-3


def test_moe_layer_qwen3(ctx, qwen_bank):
    bank, strides, routers = qwen_bank
    spec = bank.spec
    rng = np.random.default_rng(77)
    T = 32
    xb = synth.make_hidden(rng, T, spec.hidden, "bf16")
    x = synth.as_f32(xb, "bf16")
    out, ex, wt = MoEBlock(ctx, bank).forward(xb, 0, "bf16")
    w, b = routers[0]
    assert b is None
    _, ref_ex, ref_wt = O.moe_layer(spec, strides[0], w, None, x)
    logits = np.stack([O.router_logits(w, None, x[t]) for t in range(T)])
    check_topk(ex, ref_ex, logits, spec.top_k)
    assert np.allclose(wt.sum(1), 1.0, atol=1e-5)  # renormalised over the 8
    assert O.rel_l2(out, O.moe_layer64(spec, strides[0], x, ex, wt)) < 1e-3


def test_fixed_routing_equals_apply_assignments(ctx, oss_bank):
    bank, strides, _ = oss_bank
    spec = bank.spec
    rng = np.random.default_rng(8)
    T = 6
    xb = synth.make_hidden(rng, T, spec.hidden, "bf16")
    x = synth.as_f32(xb, "bf16")
    ex = np.stack([rng.permutation(spec.experts)[:spec.top_k] for _ in range(T)]).astype(np.int32)
    wt = rng.dirichlet(np.ones(spec.top_k), T).astype(np.float32)
    out, ex2, wt2 = MoEBlock(ctx, bank).forward(xb, 0, "bf16", routing=(ex, wt))
    assert np.array_equal(ex2, ex) and np.array_equal(wt2, wt)
    assert O.rel_l2(out, O.moe_layer64(spec, strides[0], x, ex, wt)) < 1e-3
    from godwit_b200.runtime import Assignment
    asg = [Assignment(int(ex[t, j]), t, float(wt[t, j])) for t in range(T) for j in range(spec.top_k)]
    out2 = ExpertRunner(ctx, bank).apply_assignments(xb, 0, asg, "bf16")
    assert O.rel_l2(out2, out) < 1e-6


def test_expert_shards_sum_to_the_whole(ctx):
    spec = GPT_OSS_20B.with_(experts=8, layers=1, hidden=256, intermediate=128)
    rng = np.random.default_rng(12)
    T = 9
    xb = synth.make_hidden(rng, T, spec.hidden, "bf16")
    full, strides, routers = build_bank(ctx, spec, 55)
    parts = [build_bank(ctx, spec, 55, shard=(r, 2))[0] for r in range(2)]
    try:
        out, ex, wt = MoEBlock(ctx, full).forward(xb, 0, "bf16")
        psum = np.zeros_like(out)
        for p in parts:
            o, e2, w2 = MoEBlock(ctx, p).forward(xb, 0, "bf16")
            assert np.array_equal(e2, ex)
            psum += o
        assert O.rel_l2(psum, out) < 1e-6
        with pytest.raises(GodwitCUDAError):
            parts[0].upload_expert(0, 1, strides[0][1])  # expert 1 lives on shard 1
    finally:
        for b in [full] + parts:
            b.close()


def test_bank_rejects_bad_calls(ctx, oss_bank):
    bank, strides, _ = oss_bank
    runner = ExpertRunner(ctx, bank)
    x = np.zeros(bank.spec.hidden, np.float16)
    for bad in (lambda: runner.apply(x, 0, bank.spec.experts, "f16"),
                lambda: runner.apply(x, 5, 0, "f16"),
                lambda: runner.apply(np.zeros(10, np.float16), 0, 0, "f16"),
                lambda: bank.upload_expert(0, 0, strides[0][0][:-16])):
        with pytest.raises(GodwitCUDAError) as e:
            bad()
        assert e.value.status == GW_E_ARG


def test_device_synthetic_fill_matches_host_mirror(ctx):
    spec = GPT_OSS_20B.with_(experts=4, layers=2, hidden=128, intermediate=64)
    bank = ExpertBank(ctx, spec, layers=2)
    try:
        bank.fill_synthetic(42)
        lay = spec.layout()
        for l, e in ((0, 0), (1, 3)):
            dev = bank.download_expert(l, e)
            host = synth.hash_expert_stride(spec, 42, l, e)
            for s in ("gate_up_blocks", "gate_up_scales", "down_blocks", "down_scales"):
                o, n = lay.offsets[s], lay.sizes[s]
                assert np.array_equal(dev[o:o + n], host[o:o + n]), s
            o, n = lay.offsets["down_bias"], lay.sizes["down_bias"]
            agree = np.mean(dev[o:o + n].view(np.uint16) == host[o:o + n].view(np.uint16))
            assert agree > 0.99
    finally:
        bank.close()


def test_stack_forward_chains_layers(ctx, oss_bank):
    import torch
    from godwit_b200 import device as D
    bank, strides, routers = oss_bank
    spec = bank.spec
    T = 3
    rng = np.random.default_rng(21)
    xb = synth.make_hidden(rng, T, spec.hidden, "bf16")
    x_dev = torch.from_numpy(xb.view(np.int16)).cuda().view(torch.bfloat16)
    stream = torch.empty(T, spec.hidden, dtype=torch.float32, device="cuda")
    D.bind_stream(ctx)
    D.moe_stack(ctx, bank, x_dev, stream)
    torch.cuda.synchronize()
    got = stream.cpu().numpy()
    # host chain: stream = x; stream += layer_l(bf16(stream))
    s = synth.as_f32(xb, "bf16").astype(np.float32)
    for l in range(bank.layers):
        xl = synth.bf16_bits_to_f32(synth.f32_to_bf16_bits(s))
        o, _, _ = MoEBlock(ctx, bank).forward(synth.f32_to_bf16_bits(xl), l, "bf16")
        s = s + o
    assert O.rel_l2(got, s) < 1e-5
    ctx.set_stream(None)


def test_bank_round_trips_the_reference_stride(ctx, oss_bank):
    # upload re-lays the stride out for the kernels; download restores it
    bank, strides, _ = oss_bank
    for e in (0, 7):
        assert np.array_equal(bank.download_expert(1, e), strides[1][e])
