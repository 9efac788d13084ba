"""AllToAllEP on the CUDA library: one rank (no process group) routes with
gw_route_async, applies every (token, slot) row as its own one-expert token
(gw_moe_apply_async) and sums the slots in order — the same layer as
gw_moe_forward_async on the same tokens (identical routing, rel-L2 < 1e-5 with both on the GEMV tiles, which split
K differently for a different number of rows); and
two NCCL ranks on two GPUs (skipped with fewer), each with half the tokens and
the experts e % 2 == rank, reproduce the one-GPU stack to rel-L2 < 1e-5."""
import os
import socket

import numpy as np
import oracle as O
import pytest

from godwit_b200 import synth
from godwit_b200.layout import GPT_OSS_20B

pytestmark = pytest.mark.gpu
SPEC = GPT_OSS_20B.with_(experts=8, layers=2)
T = 12


def build(ctx, shard_rank=0, shard_count=1, seed=21):
    from godwit_b200.runtime import ExpertBank
    rng = np.random.default_rng(seed)
    bank = ExpertBank(ctx, SPEC, layers=SPEC.layers, shard_rank=shard_rank, shard_count=shard_count)
    for layer in range(SPEC.layers):
        for e in range(SPEC.experts):
            st = synth.make_expert_stride(SPEC, rng)
            if e % shard_count == shard_rank:
                bank.upload_expert(layer, e, st)
        w, b = synth.make_router(SPEC, rng)
        bank.upload_router(layer, w, b)
    return bank


def hidden():
    return synth.make_hidden(np.random.default_rng(4), T, SPEC.hidden, "bf16")


def test_one_rank_layer_matches_moe_forward(ctx):
    import torch
    from godwit_b200 import device as D
    from godwit_b200.ep import AllToAllEP, CudaOps
    bank = build(ctx)
    # both sides on the GEMV tiles: the 48 one-expert rows would otherwise
    # cross the tensor-core threshold that the 12-token layer does not
    ctx.set_tensor_core_min_tokens(0)
    try:
        D.bind_stream(ctx, torch.cuda.current_stream())
        x = torch.from_numpy(hidden().view(np.int16)).cuda().view(torch.bfloat16)
        ep = AllToAllEP(CudaOps(ctx, bank), SPEC.layers, SPEC.top_k)
        ep.set_capacity(T)  # forward() does this from the ranks' token counts
        got = ep.layer_partial(0, x)
        ref = torch.empty((T, SPEC.hidden), dtype=torch.float32, device="cuda")
        ex = torch.empty((T, SPEC.top_k), dtype=torch.int32, device="cuda")
        wt = torch.empty((T, SPEC.top_k), dtype=torch.float32, device="cuda")
        D.moe_forward(ctx, bank, 0, x, ref, ex, wt)
        rex, _ = CudaOps(ctx, bank).route(0, x)
        torch.cuda.synchronize()
        assert torch.equal(rex, ex)
        assert O.rel_l2(got.cpu().numpy(), ref.cpu().numpy()) < 1e-5
    finally:
        ctx.set_tensor_core_min_tokens(8)
        bank.close()


def _stack(rank, world):
    import torch
    from godwit_b200 import device as D
    from godwit_b200.ep import AllToAllEP, CudaOps
    from godwit_b200.runtime import Context
    ctx = Context(rank)
    bank = build(ctx, rank, world)
    try:
        D.bind_stream(ctx, torch.cuda.current_stream())
        xs = torch.from_numpy(hidden().view(np.int16)).view(torch.bfloat16)
        per = T // world
        x = xs[rank * per:(rank + 1) * per].contiguous().cuda()
        stream = torch.empty((x.shape[0], SPEC.hidden), dtype=torch.float32, device="cuda")
        out = AllToAllEP(CudaOps(ctx, bank), SPEC.layers, SPEC.top_k).forward(x, stream, torch.empty_like(x))
        torch.cuda.synchronize()
        return out.cpu().numpy()
    finally:
        bank.close()
        ctx.close()


def _worker(rank, world, port, out_dir):
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        np.save(os.path.join(out_dir, f"r{rank}.npy"), _stack(rank, world))
    finally:
        dist.destroy_process_group()


def test_two_nccl_ranks_match_one_gpu(tmp_path):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.spawn(_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True)
    got = np.concatenate([np.load(tmp_path / f"r{r}.npy") for r in range(2)])
    one = _stack(0, 1)
    assert O.rel_l2(got, one) < 1e-5


@pytest.mark.parametrize("world,cap", [(1, 48), (3, 24), (3, 4)])
def test_fused_dispatch_and_combine_match_the_torch_packing(ctx, world, cap):
    """gw_ep_dispatch_async / gw_ep_combine_async against the same packing in
    torch ops: identical slot rows, metadata words and per-token sums; a
    capacity too small for a block raises the overflow flag."""
    import torch
    from godwit_b200 import device as D
    from godwit_b200.ep import AllToAllEP, CudaOps
    from godwit_b200.runtime import ExpertBank

    bank = ExpertBank(ctx, SPEC, layers=1)
    try:
        D.bind_stream(ctx, torch.cuda.current_stream())
        g = torch.Generator(device="cuda").manual_seed(world * 100 + cap)
        x = torch.randn((T, SPEC.hidden), device="cuda", generator=g).to(torch.bfloat16)
        ex = torch.stack([torch.randperm(SPEC.experts, device="cuda", generator=g)[:SPEC.top_k]
                          for _ in range(T)]).to(torch.int32)
        wt = torch.rand((T, SPEC.top_k), device="cuda", generator=g)
        ep = AllToAllEP(None, 1, SPEC.top_k, capacity_factor=1.0)
        ep.overflow = torch.zeros((), dtype=torch.bool, device="cuda")
        ref_send, ref_idx = ep._dispatch_torch(x, ex, wt, world, cap)
        ops = CudaOps(ctx, bank)
        send = torch.empty_like(ref_send)
        idx = torch.empty((T * SPEC.top_k,), dtype=torch.int32, device="cuda")
        flag = torch.zeros((), dtype=torch.int32, device="cuda")
        ops.dispatch(x, ex, wt, world, cap, send, idx, flag)
        torch.cuda.synchronize()
        overflowed = bool(ep.overflow)
        assert bool(flag) == overflowed
        H = SPEC.hidden
        meta = send[:, H:].view(torch.int32)
        ref_meta = ref_send[:, H:].view(torch.int32)
        if not overflowed:
            assert torch.equal(idx.to(torch.int64), ref_idx)
            assert torch.equal(meta, ref_meta)
            used = meta[:, 0] >= 0
            assert torch.equal(send[used, :H], ref_send[used, :H])
            back = torch.randn((world * cap, H), device="cuda", generator=g)
            out = torch.empty((T, H), device="cuda")
            ops.combine(back, idx, T, out)
            y = back.index_select(0, ref_idx).view(T, SPEC.top_k, H)
            want = y[:, 0].clone()
            for j in range(1, SPEC.top_k):
                want += y[:, j]
            torch.cuda.synchronize()
            assert torch.equal(out, want)
    finally:
        ctx.set_stream(None)
        bank.close()
