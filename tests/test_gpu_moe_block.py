"""RMSNorm ahead of the router and the fused MoE block (the MoE half of
TransformerLayer.forward, Runtime/TransformerLayer.swift:140-238) through the
C-ABI: the norm kernel against the oracle's restatement of
TransformerLayer.normalise (:265-285) to one f16 ulp (the kernel sums the
squares as a tree, the reference in index order), and gw_moe_block against
the unfused sequence (oracle norm -> gw_moe_forward -> host residual add),
the fp64 layer (rel-L2 < 1e-3 on the added expert sum), and its device-tensor
async twin (identical)."""
import numpy as np
import oracle as O
import pytest

from godwit_b200 import synth
from godwit_b200._abi import GW_E_ARG, GodwitCUDAError
from godwit_b200.layout import GPT_OSS_20B, QWEN3_30B_A3B
from godwit_b200.runtime import ExpertBank, MoEBlock

pytestmark = pytest.mark.gpu
EPS = 1e-5


def bf16_bits(v: np.ndarray) -> np.ndarray:
    return (np.asarray(v, np.float32).view(np.uint32) >> 16).astype(np.uint16)


def make_bank(ctx, spec, seed):
    rng = np.random.default_rng(seed)
    bank = ExpertBank(ctx, spec, layers=1)
    st = np.stack([synth.make_expert_stride(spec, rng) for _ in range(spec.experts)])
    for e in range(spec.experts):
        bank.upload_expert(0, e, st[e])
    w, b = synth.make_router(spec, rng)
    bank.upload_router(0, w, b)
    return bank, st


@pytest.fixture(scope="module")
def oss(ctx):
    bank, st = make_bank(ctx, GPT_OSS_20B.with_(experts=8, layers=1), 77)
    yield bank, st
    bank.close()


@pytest.mark.parametrize("T,H", [(1, 2880), (7, 2880), (33, 2048)])
def test_rmsnorm_kernel_matches_oracle(ctx, T, H):
    import torch
    from godwit_b200 import device as D
    rng = np.random.default_rng(T * 100 + H)
    x = (rng.standard_normal((T, H)) * 4).astype(np.float32)
    w = bf16_bits(1 + 0.1 * rng.standard_normal(H))
    ref = O.rmsnorm(x, w, EPS)
    xs = torch.from_numpy(x).cuda()
    ws = torch.from_numpy(w.view(np.int16)).cuda()
    out = torch.empty((T, H), dtype=torch.float16, device="cuda")
    torch.cuda.synchronize()
    D.rmsnorm(ctx, xs, ws, EPS, out)
    ctx.sync()
    got = out.cpu().numpy()
    diff = np.abs(got.astype(np.float64) - ref.astype(np.float64))
    ulp = np.abs(np.spacing(ref)).astype(np.float64)
    assert np.all(diff <= ulp)
    assert (got == ref).mean() > 0.99


def test_moe_block_matches_unfused_and_fp64(ctx, oss):
    bank, st = oss
    spec = bank.spec
    rng = np.random.default_rng(5)
    T = 6
    stream = (rng.standard_normal((T, spec.hidden)) * 2).astype(np.float32)
    nw = bf16_bits(1 + 0.05 * rng.standard_normal(spec.hidden))
    import torch
    from godwit_b200 import device as D
    blk = MoEBlock(ctx, bank)
    new, ex, wt = blk.block(stream, 0, nw, EPS)
    # the unfused sequence on the kernel's own normed rows (which agree with
    # the oracle's to one f16 ulp, test_rmsnorm_kernel_matches_oracle)
    nd = torch.empty((T, spec.hidden), dtype=torch.float16, device="cuda")
    sd = torch.from_numpy(stream).cuda()
    wd = torch.from_numpy(nw.view(np.int16)).cuda()
    torch.cuda.synchronize()
    D.rmsnorm(ctx, sd, wd, EPS, nd)
    ctx.sync()
    normed = nd.cpu().numpy()
    out_u, ex_u, wt_u = blk.forward(normed, 0, "f16")
    assert np.array_equal(ex, ex_u)
    assert np.array_equal(wt, wt_u)
    delta = new - stream
    assert np.array_equal(new, stream + out_u)      # the combine's fp32 add, as the host's
    ref = O.moe_layer64(spec, st, normed.astype(np.float64), ex, wt)
    assert O.rel_l2(delta, ref) < 1e-3
    o_ref = O.rmsnorm(stream, nw, EPS)
    assert np.all(np.abs(normed.astype(np.float64) - o_ref) <= np.abs(np.spacing(o_ref)))


def test_moe_block_async_matches_sync(ctx, oss):
    import torch
    from godwit_b200 import device as D
    bank, _ = oss
    spec = bank.spec
    rng = np.random.default_rng(9)
    T = 4
    stream = rng.standard_normal((T, spec.hidden)).astype(np.float32)
    nw = bf16_bits(1 + 0.05 * rng.standard_normal(spec.hidden))
    new, ex, wt = MoEBlock(ctx, bank).block(stream, 0, nw, EPS)
    sd = torch.from_numpy(stream).cuda()
    wd = torch.from_numpy(nw.view(np.int16)).cuda()
    exd = torch.empty((T, spec.top_k), dtype=torch.int32, device="cuda")
    wtd = torch.empty((T, spec.top_k), dtype=torch.float32, device="cuda")
    D.bind_stream(ctx, torch.cuda.current_stream())
    D.moe_block(ctx, bank, 0, sd, wd, EPS, exd, wtd)
    torch.cuda.synchronize()
    assert np.array_equal(sd.cpu().numpy(), new)
    assert np.array_equal(exd.cpu().numpy(), ex)


def test_moe_block_qwen3_silu(ctx):
    bank, st = make_bank(ctx, QWEN3_30B_A3B.with_(experts=16, layers=1), 31)
    try:
        spec = bank.spec
        rng = np.random.default_rng(2)
        stream = rng.standard_normal((3, spec.hidden)).astype(np.float32)
        nw = bf16_bits(1 + 0.05 * rng.standard_normal(spec.hidden))
        new, ex, wt = MoEBlock(ctx, bank).block(stream, 0, nw, 1e-6)
        normed = O.rmsnorm(stream, nw, 1e-6)
        ref = O.moe_layer64(spec, st, normed.astype(np.float64), ex, wt)
        assert O.rel_l2(new - stream, ref) < 1e-3
    finally:
        bank.close()


def test_moe_block_rejects_bad_arguments(ctx, oss):
    import torch
    from godwit_b200 import device as D
    bank, _ = oss
    H = bank.spec.hidden
    nw = torch.zeros(H, dtype=torch.int16, device="cuda")
    buf = torch.zeros(2 * H + 4, dtype=torch.float32, device="cuda")
    with pytest.raises(GodwitCUDAError) as e:      # stream not 16-byte aligned
        D.moe_block(ctx, bank, 0, buf[1:1 + 2 * H].view(2, H), nw, EPS)
    assert e.value.status == GW_E_ARG
    with pytest.raises(GodwitCUDAError) as e:      # negative eps
        D.moe_block(ctx, bank, 0, buf[:2 * H].view(2, H), nw, -1.0)
    assert e.value.status == GW_E_ARG
