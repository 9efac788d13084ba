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

The compute is supplied by an ops object so the same orchestration runs on
the CUDA library (CudaOps) and, in the CPU tests, on any stand-in with the
same three methods.
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
        self.D.residual_round(self.ctx, stream, delta, x_out)


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
