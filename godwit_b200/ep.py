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

    def dispatch(self, x: torch.Tensor, experts: torch.Tensor, weights: torch.Tensor, world: int, C: int,
                 send: torch.Tensor, idx: torch.Tensor, overflow: torch.Tensor) -> None:
        """Packs x's (token, slot) rows into send [world * C, H + 4] (see
        AllToAllEP) and records each slot's row in idx [T * k] (one kernel
        for the row plan, one for the copies)."""
        self.D.call("gw_ep_dispatch_async", self.ctx.handle, self.bank.handle, self.D._p(x), self.D.dtype_code(x),
                    x.shape[0], self.D._p(experts), self.D._p(weights), world, C, self.D._p(send), self.D._p(idx),
                    self.D._p(overflow))

    def combine(self, back: torch.Tensor, idx: torch.Tensor, T: int, out: torch.Tensor) -> None:
        """out[t] = sum over slots j of back[idx[t * k + j]], in slot order."""
        self.D.call("gw_ep_combine_async", self.ctx.handle, self.bank.handle, self.D._p(back), self.D._p(idx), T,
                    self.D._p(out))

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
    """Token-sliced expert parallelism with fixed-capacity exchanges.

    Every rank sends each peer a block of exactly C rows (C = capacity per
    peer), so both all-to-alls have equal splits known before the layer runs
    and nothing waits on the host between layers: a (token, slot) row goes to
    position `pos` of its owner's block, where pos counts the earlier slots
    bound for the same owner (computed on the device); unused rows carry
    expert id -1 and are skipped by the owner's grouping.  Each row carries
    its expert id and routing weight in four trailing bf16 columns, so rows
    and metadata travel in one exchange.

    C defaults to the exact bound max_r(T_r) * k (no row can be dropped).
    With `capacity_factor` f, C = ceil(max_r(T_r) * k / world * f) + 4 and
    forward() checks once, at its end, that no block overflowed (raising
    RuntimeError if one did: rows are never dropped silently)."""

    def __init__(self, ops, layers: int, top_k: int, group=None, capacity_factor: float | None = None):
        self.ops = ops
        self.layers = layers
        self.k = top_k
        self.group = group
        self.capacity_factor = capacity_factor
        self.capacity = None
        self.overflow = None      # bool flag of the torch packing
        self.overflow_i32 = None  # int32 flag the library's packing kernel sets

    def _world(self):
        return dist.get_world_size(self.group) if dist.is_initialized() else 1

    def _a2a(self, out: torch.Tensor, inp: torch.Tensor) -> None:
        if self._world() > 1:
            dist.all_to_all_single(out, inp, group=self.group)
        else:
            out.copy_(inp)

    def set_capacity(self, tokens_max: int) -> None:
        world = self._world()
        full = max(1, tokens_max * self.k)
        if self.capacity_factor is None:
            self.capacity = full
        else:
            self.capacity = min(full, int(-(-full * self.capacity_factor // world)) + 4)

    def layer_partial(self, layer: int, x: torch.Tensor) -> torch.Tensor:
        """This rank's tokens x [T, H] -> [T, H] fp32 weighted expert sum of layer `layer`."""
        world = self._world()
        T, H = x.shape
        k, C = self.k, self.capacity
        dev = x.device
        if T > 0:
            experts, weights = self.ops.route(layer, x)
        else:  # a rank without tokens still takes part in every exchange
            experts = torch.empty((0, k), dtype=torch.int32, device=dev)
            weights = torch.empty((0, k), dtype=torch.float32, device=dev)
        if hasattr(self.ops, "dispatch"):  # the library's fused pack / combine kernels
            send = torch.empty((world * C, H + 4), dtype=x.dtype, device=dev)
            idx = torch.empty((max(T * k, 1),), dtype=torch.int32, device=dev)
            if self.overflow_i32 is None:
                self.overflow_i32 = torch.zeros((), dtype=torch.int32, device=dev)
            self.ops.dispatch(x, experts, weights, world, C, send, idx, self.overflow_i32)
        else:
            send, idx = self._dispatch_torch(x, experts, weights, world, C)
        recv = torch.empty_like(send)
        self._a2a(recv, send)
        rows = recv[:, :H].contiguous()
        rmeta = recv[:, H:].view(torch.int32)
        out = torch.zeros((world * C, H), dtype=torch.float32, device=dev)
        self.ops.apply_rows(layer, rows, rmeta[:, 0].contiguous(), rmeta[:, 1].contiguous().view(torch.float32),
                            out)
        back = torch.empty_like(out)
        self._a2a(back, out)
        partial = torch.empty((T, H), dtype=torch.float32, device=dev)
        if T == 0:
            return partial
        if hasattr(self.ops, "combine"):
            self.ops.combine(back, idx, T, partial)
            return partial
        y = back.index_select(0, idx.to(torch.int64)).view(T, k, H)
        partial = y[:, 0].clone()
        for j in range(1, k):                                          # slot order, as the combine
            partial += y[:, j]
        return partial

    def _dispatch_torch(self, x, experts, weights, world: int, C: int):
        """The same packing as the library's gw_ep_dispatch_async, in torch
        ops (for compute stand-ins without it)."""
        T, H = x.shape
        k, dev = self.k, x.device
        flat_e = experts.reshape(-1).to(torch.int64)
        dest = torch.remainder(flat_e, world)
        # position of each slot in its owner's block: earlier slots bound for the same owner
        onehot = torch.nn.functional.one_hot(dest, world)
        pos = (onehot.cumsum(0).gather(1, dest[:, None]).squeeze(1) - 1) if T > 0 else dest
        if self.overflow is not None and T > 0:
            self.overflow |= (pos >= C).any()
        idx = dest * C + torch.clamp(pos, max=C - 1)
        send = torch.zeros((world * C, H + 4), dtype=x.dtype, device=dev)
        meta = send[:, H:].view(torch.int32)                           # [world*C, 2]: expert, weight bits
        meta[:, 0] = -1
        if T > 0:
            slot_tok = torch.div(torch.arange(T * k, device=dev), k, rounding_mode="floor")
            send[idx, :H] = x.index_select(0, slot_tok)
            packed = torch.stack([experts.reshape(-1), weights.reshape(-1).contiguous().view(torch.int32)], 1)
            meta[idx] = packed
        return send, idx

    def forward(self, x: torch.Tensor, stream: torch.Tensor, x_work: torch.Tensor,
                check: bool = True) -> torch.Tensor:
        """x [T, H] (this rank's tokens, compute dtype) -> stream [T, H] fp32:
        stream = x; for l: stream += moe_l(round(stream)).  check=False leaves
        the capacity check to raise_if_overflowed() (a step captured in a CUDA
        graph cannot read the flag back to the host)."""
        if self.capacity is None:  # one exchange of the token counts, then fixed shapes
            t = torch.tensor([x.shape[0]], dtype=torch.int64, device=x.device)
            if self._world() > 1:
                dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)
            self.set_capacity(int(t.item()))
        if self.capacity_factor is not None:
            if self.overflow is None:
                self.overflow = torch.zeros((), dtype=torch.bool, device=x.device)
            self.overflow.zero_()
        if self.overflow_i32 is not None:
            self.overflow_i32.zero_()
        self.ops.widen(x, stream)
        x_work.copy_(x)
        for layer in range(self.layers):
            partial = self.layer_partial(layer, x_work)
            self.ops.residual(stream, partial, x_work)
        if check and self.capacity_factor is not None:
            self.raise_if_overflowed()
        return stream

    def raise_if_overflowed(self) -> None:
        if (self.overflow is not None and bool(self.overflow)) or \
                (self.overflow_i32 is not None and int(self.overflow_i32) != 0):
            raise RuntimeError(f"an all-to-all block overflowed its capacity of {self.capacity} rows; "
                               "raise capacity_factor (or leave it unset for the exact bound)")
