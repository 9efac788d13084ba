"""All-to-all expert parallelism (godwit_b200/ep.py AllToAllEP) on CPU gloo
ranks: each rank holds a slice of the tokens, routes them, sends every
(token, slot) row to the owner of the slot's expert (e % world), applies the
experts there and returns the weighted outputs, which are summed in slot
order.  The per-rank compute is an elementwise stand-in (router = top-k of
the first E features, expert e = w * tanh((e + 1 + layer) x)), so the
multi-rank stack must equal the one-rank stack exactly; the stand-in also
checks that every row arrives at the rank owning its expert."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

H, E, K, LAYERS = 48, 10, 3, 3
T_TOTAL = 13


class ToyOps:
    def __init__(self, rank, world):
        self.rank, self.world = rank, world

    def widen(self, x, stream):
        stream.copy_(x.float())

    def residual(self, stream, delta, x_out):
        stream.add_(delta)
        x_out.copy_(stream.to(torch.bfloat16))

    def route(self, layer, x):
        logits = x.float()[:, :E]
        top = torch.topk(logits, K, dim=1)
        return top.indices.to(torch.int32), torch.softmax(top.values, dim=1).to(torch.float32)

    def apply_rows(self, layer, rows, experts, weights, out):
        live = experts >= 0  # rows with expert id -1 pad the fixed-capacity blocks
        assert bool(((experts[live].to(torch.int64) % self.world) == self.rank).all()), "row sent to a non-owner"
        y = weights[:, None] * torch.tanh(rows.float() * (experts[:, None].float() + 1 + layer))
        out.copy_(torch.where(live[:, None], y, torch.zeros_like(y)))


def make_x():
    g = torch.Generator().manual_seed(11)
    return torch.randn(T_TOTAL, H, generator=g).to(torch.bfloat16)


def run(rank, world, total=T_TOTAL, capacity_factor=None):
    from godwit_b200.ep import AllToAllEP
    per = -(-total // world)
    x = make_x()[:total][rank * per:min(total, (rank + 1) * per)].contiguous()
    stream = torch.empty(x.shape[0], H)
    x_work = torch.empty_like(x)
    ep = AllToAllEP(ToyOps(rank, world), LAYERS, K, capacity_factor=capacity_factor)
    return ep.forward(x, stream, x_work).numpy()


def _worker(rank, world, port, out_dir, total=T_TOTAL, capacity_factor=None):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        try:
            res = run(rank, world, total, capacity_factor)
        except RuntimeError as e:
            res = np.array([str(e)])
        np.save(os.path.join(out_dir, f"r{rank}.npy"), res)
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 3])
def test_alltoall_ranks_match_one_rank(tmp_path, world):
    ref = run(0, 1)
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    got = np.concatenate([np.load(tmp_path / f"r{r}.npy") for r in range(world)])
    assert got.shape == ref.shape
    assert np.array_equal(got, ref)


def test_rank_without_tokens(tmp_path):
    """Two tokens over three ranks: the last rank holds none but still takes
    part in every exchange (and serves the experts it owns)."""
    ref = run(0, 1, 2)
    mp.spawn(_worker, args=(3, _free_port(), str(tmp_path), 2), nprocs=3, join=True)
    parts = [np.load(tmp_path / f"r{r}.npy") for r in range(3)]
    assert parts[2].shape == (0, H)
    assert np.array_equal(np.concatenate(parts), ref)


def test_one_rank_matches_direct_sum():
    """The single-rank path (no process group) against the layer written out
    directly: stream += sum_j w_j expert_{e_j}(round(stream)) in slot order."""
    ops = ToyOps(0, 1)
    x = make_x()
    stream = x.float().clone()
    xw = x.clone()
    for layer in range(LAYERS):
        ex, wt = ops.route(layer, xw)
        acc = None
        for j in range(K):
            y = wt[:, j:j + 1] * torch.tanh(xw.float() * (ex[:, j:j + 1].float() + 1 + layer))
            acc = y if acc is None else acc + y
        stream += acc
        xw = stream.to(torch.bfloat16)
    assert np.array_equal(run(0, 1), stream.numpy())


def test_bounded_capacity_matches_and_overflow_is_reported(tmp_path):
    """capacity_factor 2 (blocks of ceil(T k / world * 2) + 4 rows) gives the
    same result; a factor too small to hold the rows raises instead of
    dropping any."""
    ref = run(0, 1)
    mp.spawn(_worker, args=(2, _free_port(), str(tmp_path), T_TOTAL, 2.0), nprocs=2, join=True)
    got = np.concatenate([np.load(tmp_path / f"r{r}.npy") for r in range(2)])
    assert np.array_equal(got, ref)
    # 13 tokens x 3 slots over 2 ranks, blocks of ceil(21 * 0.01 / 2) + 4 = 5 rows:
    # some owner receives more than 5 of a sender's 21 slots
    mp.spawn(_worker, args=(2, _free_port(), str(tmp_path), T_TOTAL, 0.01), nprocs=2, join=True)
    msgs = [np.load(tmp_path / f"r{r}.npy") for r in range(2)]
    assert any(m.dtype.kind == "U" and "overflowed" in str(m[0]) for m in msgs)
