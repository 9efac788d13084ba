"""The MoE layer entry point that allocates no device memory.

Some callers cannot allocate while they serve: engines that plan every byte
of device memory before the first request, processes under a hard memory cap,
or latency-critical loops where a first-call allocation must not stall or
fail.  gw_moe_forward_noalloc_async keeps the layer's scratch in a fixed
device array inside the library instead.  This file runs last (pytest
collects it after the others) so that a failure here cannot hide any other
test's result; it also passes when run alone in a fresh process.
"""
import numpy as np
import oracle as O
import pytest

from godwit_b200 import synth
from godwit_b200._abi import GW_E_ARG, GodwitCUDAError
from godwit_b200.layout import GPT_OSS_20B
from godwit_b200.runtime import ExpertBank

pytestmark = pytest.mark.gpu


def test_noalloc_layer_matches_workspace_layer_twice(ctx):
    import torch
    from godwit_b200 import device as D

    spec = GPT_OSS_20B.with_(experts=8, layers=1)
    rng = np.random.default_rng(77)
    bank = ExpertBank(ctx, spec, layers=1)
    try:
        for e in range(spec.experts):
            bank.upload_expert(0, e, synth.make_expert_stride(spec, rng))
        w, b = synth.make_router(spec, rng)
        bank.upload_router(0, w, b)
        D.bind_stream(ctx)
        for T in (5, 3):  # two calls in a row, the second with fewer tokens
            xb = synth.make_hidden(rng, T, spec.hidden, "bf16")
            x = torch.from_numpy(xb.view(np.int16)).cuda().view(torch.bfloat16)
            out_ref = torch.empty(T, spec.hidden, dtype=torch.float32, device="cuda")
            out = torch.full_like(out_ref, float("nan"))
            ex_ref = torch.empty(T, spec.top_k, dtype=torch.int32, device="cuda")
            ex = torch.empty_like(ex_ref)
            wt_ref = torch.empty(T, spec.top_k, dtype=torch.float32, device="cuda")
            wt = torch.empty_like(wt_ref)
            D.moe_forward(ctx, bank, 0, x, out_ref, ex_ref, wt_ref)
            D.moe_forward_noalloc(ctx, bank, 0, x, out, ex, wt)
            torch.cuda.synchronize()
            assert torch.equal(ex, ex_ref)
            assert torch.allclose(wt, wt_ref, rtol=1e-6, atol=0)
            # the tolerance of the layer parity tests: rel-L2 <= 1e-3
            assert O.rel_l2(out.cpu().numpy(), out_ref.cpu().numpy()) < 1e-3
    finally:
        ctx.set_stream(None)
        bank.close()


def test_noalloc_first_call_on_a_fresh_context_allocates_nothing(ctx):
    """On a context that has never run a layer (no workspace yet), two calls
    in a row — the second with more tokens — leave the device's free memory
    unchanged, and both match the fp64 oracle under their own routing."""
    import torch
    from godwit_b200 import device as D
    from godwit_b200.runtime import Context

    spec = GPT_OSS_20B.with_(experts=8, layers=1)
    rng = np.random.default_rng(78)
    fresh = Context(0)
    bank = ExpertBank(fresh, spec, layers=1)
    try:
        strides = np.stack([synth.make_expert_stride(spec, rng) for _ in range(spec.experts)])
        for e in range(spec.experts):
            bank.upload_expert(0, e, strides[e])
        w, b = synth.make_router(spec, rng)
        bank.upload_router(0, w, b)
        # load every kernel both token counts use (lazy module loading may
        # reserve device memory on a kernel's first launch) through another
        # context, so that only the no-allocation calls run in the window
        warm = ExpertBank(ctx, spec, layers=1)
        try:
            warm.fill_synthetic(1)
            for T in (3, 9):
                xw = torch.zeros(T, spec.hidden, dtype=torch.bfloat16, device="cuda")
                torch.cuda.synchronize()
                D.moe_forward(ctx, warm, 0, xw, torch.empty(T, spec.hidden, device="cuda"))
            ctx.sync()
        finally:
            warm.close()
        D.bind_stream(fresh)
        cases = []
        for T in (3, 9):
            xb = synth.make_hidden(rng, T, spec.hidden, "bf16")
            cases.append((xb, torch.from_numpy(xb.view(np.int16)).cuda().view(torch.bfloat16),
                          torch.empty(T, spec.hidden, dtype=torch.float32, device="cuda"),
                          torch.empty(T, spec.top_k, dtype=torch.int32, device="cuda"),
                          torch.empty(T, spec.top_k, dtype=torch.float32, device="cuda")))
        torch.cuda.synchronize()
        free = []
        for xb, x, out, ex, wt in cases:
            D.moe_forward_noalloc(fresh, bank, 0, x, out, ex, wt)
            torch.cuda.synchronize()
            free.append(torch.cuda.mem_get_info()[0])
        assert free[1] == free[0], "the second, larger call changed the free device memory"
        for xb, x, out, ex, wt in cases:
            xf = synth.as_f32(xb, "bf16")
            ref = O.moe_layer64(spec, strides, xf, ex.cpu().numpy(), wt.cpu().numpy())
            assert O.rel_l2(out.cpu().numpy(), ref) < 1e-3
    finally:
        fresh.set_stream(None)
        bank.close()
        fresh.close()


def test_noalloc_rejects_token_counts_beyond_its_scratch(ctx):
    import torch
    from godwit_b200 import device as D

    spec = GPT_OSS_20B.with_(experts=8, layers=1)
    bank = ExpertBank(ctx, spec, layers=1)
    try:
        T = 64  # needs more than the fixed 4 MiB at this shape
        x = torch.zeros(T, spec.hidden, dtype=torch.bfloat16, device="cuda")
        out = torch.empty(T, spec.hidden, dtype=torch.float32, device="cuda")
        with pytest.raises(GodwitCUDAError) as e:
            D.moe_forward_noalloc(ctx, bank, 0, x, out)
        assert e.value.status == GW_E_ARG and "scratch" in str(e.value)
    finally:
        bank.close()
