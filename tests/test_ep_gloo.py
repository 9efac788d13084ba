"""Expert-parallel orchestration (godwit_b200/ep.py) on CPU: two gloo ranks,
each owning the experts e % 2 == rank, must reproduce the single-rank layer
stack.  The per-rank compute is the CPU oracle standing in for the CUDA
library (this tests the sharding, the all-reduce combine and the residual
chaining, not the kernels)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from godwit_b200.layout import GPT_OSS_20B

SPEC = GPT_OSS_20B.with_(hidden=64, intermediate=32, experts=6, layers=3)
T = 5


def make_model():
    from godwit_b200 import synth
    rng = np.random.default_rng(3)
    strides = [np.stack([synth.make_expert_stride(SPEC, rng) for _ in range(SPEC.experts)])
               for _ in range(SPEC.layers)]
    routers = [synth.make_router(SPEC, rng) for _ in range(SPEC.layers)]
    x = synth.as_f32(synth.make_hidden(rng, T, SPEC.hidden, "bf16"), "bf16")
    return strides, routers, x


class OracleOps:
    """CPU stand-in with CudaOps' three methods; owns experts e % world == rank."""

    def __init__(self, strides, routers, rank, world):
        import oracle as O
        self.O, self.strides, self.routers, self.rank, self.world = O, strides, routers, rank, world

    def widen(self, x, stream):
        stream.copy_(x.float())

    def moe_partial(self, layer, x, out):
        from godwit_b200.ep import shard_of
        w, b = self.routers[layer]
        xf = x.float().numpy()
        _, ex, wt = self.O.moe_layer(SPEC, self.strides[layer], w, b, xf)
        mine = np.vectorize(lambda e: shard_of(int(e), self.world) == self.rank)(ex)
        ex = np.where(mine, ex, -1).astype(np.int32)
        o, _, _ = self.O.moe_layer(SPEC, self.strides[layer], w, b, xf, routing=(ex, wt))
        out.copy_(torch.from_numpy(o))

    def residual(self, stream, delta, x_out):
        stream.add_(delta)
        x_out.copy_(stream.to(torch.bfloat16))


def run_stack(rank, world):
    from godwit_b200.ep import ReplicatedTokensEP
    strides, routers, x = make_model()
    ops = OracleOps(strides, routers, rank, world)
    xb = torch.from_numpy(x).to(torch.bfloat16)
    stream = torch.empty(T, SPEC.hidden)
    partial = torch.empty_like(stream)
    x_work = torch.empty_like(xb)
    return ReplicatedTokensEP(ops, SPEC.layers).forward(xb, stream, partial, x_work).numpy()


def _worker(rank, world, port, out_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        res = run_stack(rank, world)
        if rank == 0:
            np.save(out_path, res)
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_gloo_ranks_match_one_rank(tmp_path):
    ref = run_stack(0, 1)
    out = tmp_path / "ep.npy"
    mp.spawn(_worker, args=(2, _free_port(), str(out)), nprocs=2, join=True)
    got = np.load(out)
    assert np.abs(got - ref).max() <= 1e-5 * (1 + np.abs(ref).max())


def test_shard_ownership_covers_every_expert_once():
    from godwit_b200.ep import shard_of
    for world in (1, 2, 4, 8):
        owners = [shard_of(e, world) for e in range(128)]
        assert all(0 <= o < world for o in owners)
        assert [owners.count(r) for r in range(world)] == [128 // world] * world
