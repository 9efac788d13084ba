"""Expert parallelism over torch.distributed (one process per GPU).

The reference is single-device; experts are sharded here by index: rank r
of N holds every expert e with e % N == r (gw_bank_desc.shard_rank /
shard_count), so the 4x-hot experts of a skewed router spread across ranks.

ReplicatedTokensEP — decode.  Every rank holds the same hidden states (as a
replicated attention trunk would produce), routes them identically, runs only
the experts it owns, and the per-token partial sums meet in one all-reduce
per layer.  The all-reduce is the combine step of the MoE block; its output
feeds the residual add of TransformerLayer.forward
(Runtime/TransformerLayer.swift:232-238).

AllToAllEP — prefill and batched decode.  Each rank holds its own token
rows (a slice of the batch), routes them itself (the router weights are
replicated), sends every (token, slot) row to the rank that owns the slot's
expert (NCCL all-to-all of token rows), runs its experts on what it
received, and sends the weighted fp32 expert outputs back (a second
all-to-all); each token's k partials are then summed in slot order, the
order of the single-device combine (k_combine, ExpertRunner's accumulate,
Metal/MoE/expert.metal:107-116).  Bytes per layer and rank: T_r * k rows out
(H in the compute dtype) and back (H fp32), instead of the replicated design's
all-reduce of every token.

The compute is supplied by an ops object so the same orchestration runs on
the CUDA library (CudaOps) and, in the CPU tests, on any stand-in with the
same methods.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


class CudaOps:
    """Per-rank compute on this library's kernels (stream-ordered)."""

    def __init__(self, ctx, bank):
        from . import device as D
        self.D, self.ctx, self.bank = D, ctx, bank

    def widen(self, x: torch.Tensor, stream: torch.Tensor) -> None:
        stream.copy_(x)

    def moe_partial(self, layer: int, x: torch.Tensor, out: torch.Tensor) -> None:
        self.D.moe_forward(self.ctx, self.bank, layer, x, out)

    def residual(self, stream: torch.Tensor, delta: torch.Tensor, x_out: torch.Tensor) -> None:
        if stream.numel():  # a rank may hold no tokens
            self.D.residual_round(self.ctx, stream, delta, x_out)

    def route(self, layer: int, x: torch.Tensor):
        k = self.bank.spec.top_k
        ex = torch.empty((x.shape[0], k), dtype=torch.int32, device=x.device)
        wt = torch.empty((x.shape[0], k), dtype=torch.float32, device=x.device)
        self.D.route(self.ctx, self.bank, layer, x, ex, wt)
        return ex, wt

    def apply_rows(self, layer: int, rows: torch.Tensor, experts: torch.Tensor, weights: torch.Tensor,
                   out: torch.Tensor) -> None:
        """out[r] = weights[r] * expert_{experts[r]}(rows[r]) for owned experts: each row
        becomes a token whose routing lists that one expert (the other k - 1 slots
        empty, which the grouping and the combine skip)."""
        if rows.shape[0] == 0:
            return
        k = self.bank.spec.top_k
        ex = torch.full((rows.shape[0], k), -1, dtype=torch.int32, device=rows.device)
        wt = torch.zeros((rows.shape[0], k), dtype=torch.float32, device=rows.device)
        ex[:, 0] = experts
        wt[:, 0] = weights
        self.D.moe_apply(self.ctx, self.bank, layer, rows, ex, wt, out)


class ReplicatedTokensEP:
    def __init__(self, ops, layers: int, group=None):
        self.ops = ops
        self.layers = layers
        self.group = group

    def forward(self, x: torch.Tensor, stream: torch.Tensor, partial: torch.Tensor,
                x_work: torch.Tensor) -> torch.Tensor:
        """x [T, H] (compute dtype) -> stream [T, H] fp32 after every layer:
        stream = x; for l: stream += allreduce(moe_l^{owned}(round(stream)))."""
        self.ops.widen(x, stream)
        x_work.copy_(x)
        world = dist.get_world_size(self.group) if dist.is_initialized() else 1
        for layer in range(self.layers):
            self.ops.moe_partial(layer, x_work, partial)
            if world > 1:
                dist.all_reduce(partial, op=dist.ReduceOp.SUM, group=self.group)
            self.ops.residual(stream, partial, x_work)
        return stream


def shard_of(expert: int, world: int) -> int:
    """The rank that holds `expert`."""
    return expert % world


class AllToAllEP:
    def __init__(self, ops, layers: int, top_k: int, group=None):
        self.ops = ops
        self.layers = layers
        self.k = top_k
        self.group = group

    def _a2a(self, out: torch.Tensor, inp: torch.Tensor, out_splits, in_splits) -> None:
        if dist.is_initialized() and dist.get_world_size(self.group) > 1:
            dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)
        else:
            out.copy_(inp)

    def layer_partial(self, layer: int, x: torch.Tensor) -> torch.Tensor:
        """This rank's tokens x [T, H] -> [T, H] fp32 weighted expert sum of layer `layer`."""
        world = dist.get_world_size(self.group) if dist.is_initialized() else 1
        T, H = x.shape
        k = self.k
        if T > 0:
            experts, weights = self.ops.route(layer, x)
        else:  # a rank without tokens still takes part in every exchange
            experts = torch.empty((0, k), dtype=torch.int32, device=x.device)
            weights = torch.empty((0, k), dtype=torch.float32, device=x.device)
        flat_e = experts.reshape(-1).to(torch.int64)
        dest = torch.remainder(flat_e, world)
        order = torch.sort(dest, stable=True).indices                  # slots grouped by owner
        send_counts = torch.bincount(dest, minlength=world)
        recv_counts = torch.empty_like(send_counts)
        self._a2a(recv_counts, send_counts, None, None)
        s_split, r_split = send_counts.tolist(), recv_counts.tolist()
        R = sum(r_split)
        send_rows = x.index_select(0, torch.div(order, k, rounding_mode="floor"))
        # expert id and routing weight of each sent row, one int32 pair
        meta = torch.stack([flat_e.index_select(0, order).to(torch.int32),
                            weights.reshape(-1).index_select(0, order).contiguous().view(torch.int32)], 1)
        rows = torch.empty((R, H), dtype=x.dtype, device=x.device)
        rmeta = torch.empty((R, 2), dtype=torch.int32, device=x.device)
        self._a2a(rows, send_rows, r_split, s_split)
        self._a2a(rmeta, meta, r_split, s_split)
        out = torch.empty((R, H), dtype=torch.float32, device=x.device)
        self.ops.apply_rows(layer, rows, rmeta[:, 0].contiguous(), rmeta[:, 1].contiguous().view(torch.float32),
                            out)
        back = torch.empty((T * k, H), dtype=torch.float32, device=x.device)
        self._a2a(back, out, s_split, r_split)
        y = torch.empty_like(back)
        y.index_copy_(0, order, back)
        y = y.view(T, k, H)
        if T == 0:
            return torch.empty((0, H), dtype=torch.float32, device=x.device)
        partial = y[:, 0].clone()
        for j in range(1, k):                                          # slot order, as the combine
            partial += y[:, j]
        return partial

    def forward(self, x: torch.Tensor, stream: torch.Tensor, x_work: torch.Tensor) -> torch.Tensor:
        """x [T, H] (this rank's tokens, compute dtype) -> stream [T, H] fp32:
        stream = x; for l: stream += moe_l(round(stream))."""
        self.ops.widen(x, stream)
        x_work.copy_(x)
        for layer in range(self.layers):
            partial = self.layer_partial(layer, x_work)
            self.ops.residual(stream, partial, x_work)
        return stream
