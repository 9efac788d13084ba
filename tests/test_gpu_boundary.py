"""The C-ABI's error contract on the device: timeouts of bounded waits are
reported as GW_E_TIMEOUT without a fault, and misaligned device pointers are
rejected with GW_E_ARG before anything launches."""
import numpy as np
import pytest

from godwit_b200 import synth
from godwit_b200._abi import GW_E_ARG, GW_E_TIMEOUT, GodwitCUDAError, call
from godwit_b200.layout import GPT_OSS_20B
from godwit_b200.runtime import ExpertBank

pytestmark = pytest.mark.gpu


def test_wait_that_runs_out_is_reported_as_timeout(ctx):
    ctx.sync()  # nothing pending
    # a barrier nothing completes, waited on for ~100k cycles (~50 us)
    call("gw_selftest_wait_timeout", ctx.handle, 100_000)
    with pytest.raises(GodwitCUDAError) as e:
        ctx.sync()
    assert e.value.status == GW_E_TIMEOUT
    ctx.sync()  # reported once, then cleared
    # the context is still usable
    y = ctx.mxfp4_gemv(np.full((1, 16), 0x22, np.uint8), np.array([[127]], np.uint8),
                       np.ones(32, np.float16), dtype="f16")
    assert abs(y[0] - 32.0) < 1e-4


def test_misaligned_device_pointers_are_rejected(ctx):
    import torch
    from godwit_b200 import device as D

    spec = GPT_OSS_20B.with_(experts=8, layers=1, hidden=256, intermediate=128)
    bank = ExpertBank(ctx, spec, layers=1)
    try:
        bank.fill_synthetic(3)
        T, H = 2, spec.hidden
        xbuf = torch.zeros(T * H + 8, dtype=torch.bfloat16, device="cuda")
        obuf = torch.zeros(T * H + 4, dtype=torch.float32, device="cuda")
        x_ok, x_bad = xbuf[:T * H].view(T, H), xbuf[1:T * H + 1].view(T, H)     # 2-byte offset
        o_ok, o_bad = obuf[:T * H].view(T, H), obuf[1:T * H + 1].view(T, H)     # 4-byte offset
        ex = torch.zeros(T, spec.top_k, dtype=torch.int32, device="cuda")
        wt = torch.zeros(T, spec.top_k, dtype=torch.float32, device="cuda")
        D.bind_stream(ctx)
        bad_calls = [
            lambda: D.moe_forward(ctx, bank, 0, x_bad, o_ok),
            lambda: D.moe_forward(ctx, bank, 0, x_ok, o_bad),
            lambda: D.moe_forward_noalloc(ctx, bank, 0, x_bad, o_ok),
            lambda: D.moe_forward_noalloc(ctx, bank, 0, x_ok, o_bad),
            lambda: D.moe_apply(ctx, bank, 0, x_bad, ex, wt, o_ok),
            lambda: D.moe_apply(ctx, bank, 0, x_ok, ex, wt, o_bad),
            lambda: D.route(ctx, bank, 0, x_bad, ex, wt),
            lambda: D.moe_stack(ctx, bank, x_bad, o_ok),
            lambda: D.moe_stack(ctx, bank, x_ok, o_bad),
        ]
        before = ctx.launch_count()
        for bad in bad_calls:
            with pytest.raises(GodwitCUDAError) as e:
                bad()
            assert e.value.status == GW_E_ARG and "aligned" in str(e.value)
        assert ctx.launch_count() == before  # nothing launched
        D.moe_forward(ctx, bank, 0, x_ok, o_ok)  # the aligned call runs
        torch.cuda.synchronize()
        assert torch.isfinite(o_ok).all()
    finally:
        ctx.set_stream(None)
        bank.close()
