"""Host-side mirror of the reference's expert-path interfaces over the C-ABI.

Names, argument meanings and error behaviour follow the Swift types they
replace, so a caller of the reference finds the same shape here:

  Router        Sources/Godwit/Runtime/Router.swift:11-104
                  logits(hidden, layer) / select(logits) / route(hidden, layer)
  ExpertRunner  Sources/Godwit/Runtime/ExpertRunner.swift:10-363
                  apply(input, layer, expert) / apply_batch(input, layer, experts)
                  / apply_assignments(inputs, layer, assignments) -> outputs
  MoEBlock      the MoE half of TransformerLayer.forward
                  (Sources/Godwit/Runtime/TransformerLayer.swift:140-238)
  ExpertBank    ExpertCache + ModelReader.loadExpertStride
                  (Runtime/ExpertCache.swift, Runtime/ModelReader.swift:73-76),
                  replaced by an HBM-resident bank

The reference's `precondition` failures become `GodwitCUDAError(GW_E_ARG)`
raised before any kernel launch; its thrown Metal errors become the other
`GW_E_*` codes.  All compute runs in the CUDA library; nothing here computes
a result on the CPU.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _abi
from ._abi import GW_DTYPE_BF16, GW_DTYPE_F16, BankDesc, GodwitCUDAError, call
from .layout import ModelSpec

_DTYPES = {"f16": GW_DTYPE_F16, "bf16": GW_DTYPE_BF16}


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def _dtype_code(dtype: str) -> int:
    try:
        return _DTYPES[dtype]
    except KeyError:
        raise GodwitCUDAError(_abi.GW_E_ARG, f"dtype {dtype!r} is neither 'f16' nor 'bf16'") from None


def _bits16(x: np.ndarray, dtype: str) -> np.ndarray:
    """Accepts raw uint16 patterns, float16 arrays (f16) or fp32 (rounded)."""
    x = np.asarray(x)
    if x.dtype == np.uint16:
        return np.ascontiguousarray(x)
    if dtype == "f16":
        return np.ascontiguousarray(x.astype(np.float16)).view(np.uint16)
    from .synth import f32_to_bf16_bits
    return np.ascontiguousarray(f32_to_bf16_bits(x.astype(np.float32)))


class Context:
    """One CUDA device (one process per GPU)."""

    def __init__(self, device: int = 0):
        lib = _abi.load()
        h = C.c_void_p()
        _abi.check(lib.gw_init(device, C.byref(h)))
        self.handle = h
        self.device = device

    def set_stream(self, cuda_stream: int | None) -> None:
        call("gw_ctx_set_stream", self.handle, C.c_void_p(cuda_stream or 0))

    def sync(self) -> None:
        call("gw_sync", self.handle)

    def set_block_scaled(self, enable: bool) -> None:
        """Tensor-core expert layers as block-scaled MXFP4 x MXFP8 MMAs (the
        expert inputs and activations quantised to MXFP8) instead of exact f16."""
        call("gw_set_block_scaled", self.handle, 1 if enable else 0)

    def set_tensor_core_min_tokens(self, min_avg: int) -> None:
        """Experts of a layer run as tensor-core grouped GEMMs when
        T * top_k >= min_avg * experts, else as MXFP4 GEMV tiles (0: always
        GEMV).  Default 8."""
        call("gw_set_tensor_core_min_tokens", self.handle, int(min_avg))

    def launch_count(self) -> int:
        v = C.c_int64()
        call("gw_last_launch_count", self.handle, C.byref(v))
        return v.value

    def profile_enable(self, enable: bool = True) -> None:
        call("gw_profile_enable", self.handle, 1 if enable else 0)

    def profile_read(self) -> dict:
        p = _abi.Profile()
        call("gw_profile_read", self.handle, C.byref(p))
        return {name: getattr(p, name) for name, _ in p._fields_}

    def close(self) -> None:
        if self.handle:
            call("gw_shutdown", self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    # ---- GEMV / dequant (dequant_gemv.metal, MXFP4.swift) ----
    def mxfp4_gemv(self, packed: np.ndarray, scales: np.ndarray, x: np.ndarray, *,
                   bias: np.ndarray | None = None, dtype: str = "f16") -> np.ndarray:
        packed = np.ascontiguousarray(packed, dtype=np.uint8)
        scales = np.ascontiguousarray(scales, dtype=np.uint8)
        rows, cols = packed.shape[0], packed.shape[1] * 2
        xb = _bits16(x, dtype).ravel()
        if xb.size != cols:
            raise GodwitCUDAError(_abi.GW_E_ARG, f"x has {xb.size} values, W has {cols} columns")
        bb = None if bias is None else np.ascontiguousarray(bias, dtype=np.uint16)
        y = np.empty(rows, dtype=np.float32)
        call("gw_mxfp4_gemv", self.handle, _ptr(packed), _ptr(scales), _ptr(bb), _ptr(xb),
             _dtype_code(dtype), _ptr(y), rows, cols)
        return y

    def int8_affine_gemv(self, codes: np.ndarray, meta: np.ndarray, x: np.ndarray, *,
                         bias: np.ndarray | None = None, out: str = "f32") -> np.ndarray:
        """The trunk's int8 projection (int8_affine_gemv, router.metal:65-98, when
        out="f32"; int8_affine_gemv_bias_batched, :107-141, when out="f16").
        codes [rows, cols] uint8, meta [rows, cols/64, 2] bf16 bits (scale, zero),
        x [T, cols] (or [cols]) f16 values, bias [rows] bf16 bits -> y [T, rows]."""
        codes = np.ascontiguousarray(codes, dtype=np.uint8)
        meta = np.ascontiguousarray(meta, dtype=np.uint16)
        rows, cols = codes.shape
        xb = np.atleast_2d(_bits16(x, "f16"))
        if xb.shape[1] != cols:
            raise GodwitCUDAError(_abi.GW_E_ARG, f"x has {xb.shape[1]} columns, W has {cols}")
        T = xb.shape[0]
        bb = None if bias is None else np.ascontiguousarray(bias, dtype=np.uint16)
        code = {"f32": _abi.GW_DTYPE_F32, "f16": _abi.GW_DTYPE_F16}[out]
        y = np.empty((T, rows), dtype=np.float32 if out == "f32" else np.float16)
        call("gw_int8_affine_gemv", self.handle, _ptr(codes), _ptr(meta), _ptr(bb), _ptr(xb), T, rows,
             cols, _ptr(y), code)
        return y

    def mxfp4_dequant(self, packed: np.ndarray, scales: np.ndarray) -> np.ndarray:
        packed = np.ascontiguousarray(packed, dtype=np.uint8)
        scales = np.ascontiguousarray(scales, dtype=np.uint8)
        rows, cols = packed.shape[0], packed.shape[1] * 2
        w = np.empty((rows, cols), dtype=np.float32)
        call("gw_mxfp4_dequant", self.handle, _ptr(packed), _ptr(scales), rows, cols, _ptr(w))
        return w


class ExpertBank:
    """The HBM-resident expert bank of one model (or one expert shard)."""

    def __init__(self, ctx: Context, spec: ModelSpec, *, layers: int | None = None,
                 shard_rank: int = 0, shard_count: int = 1, desc: BankDesc | None = None):
        """`desc` overrides the stride and section spans (e.g. from an
        installation's manifest); by default they follow ExpertLayout."""
        self.ctx = ctx
        self.spec = spec
        self.desc: BankDesc = desc if desc is not None else spec.desc(shard_rank, shard_count, layers)
        self.layers = self.desc.layers
        self.shard_rank, self.shard_count = shard_rank, shard_count
        h = C.c_void_p()
        call("gw_bank_create", ctx.handle, C.byref(self.desc), C.byref(h))
        self.handle = h

    def owns(self, expert: int) -> bool:
        return expert % self.shard_count == self.shard_rank

    def upload_expert(self, layer: int, expert: int, stride_bytes: np.ndarray) -> None:
        b = np.ascontiguousarray(stride_bytes, dtype=np.uint8)
        call("gw_bank_upload_expert", self.handle, layer, expert, _ptr(b), b.size)

    def download_expert(self, layer: int, expert: int) -> np.ndarray:
        b = np.empty(self.desc.expert_stride, dtype=np.uint8)
        call("gw_bank_download_expert", self.handle, layer, expert, _ptr(b), b.size)
        return b

    def upload_router(self, layer: int, weight: np.ndarray, bias: np.ndarray | None) -> None:
        w = np.ascontiguousarray(weight, dtype=np.uint16)
        if w.size != self.spec.experts * self.spec.hidden:
            raise GodwitCUDAError(_abi.GW_E_ARG, "router weight must be [E, H] bf16")
        b = None if bias is None else np.ascontiguousarray(bias, dtype=np.uint16)
        call("gw_bank_upload_router", self.handle, layer, _ptr(w), _ptr(b))

    def fill_synthetic(self, seed: int) -> None:
        call("gw_bank_fill_synthetic", self.handle, C.c_uint64(seed))

    def nbytes(self) -> int:
        v = C.c_int64()
        call("gw_bank_bytes", self.handle, C.byref(v))
        return v.value

    def close(self) -> None:
        if self.handle:
            call("gw_bank_destroy", self.handle)
            self.handle = None


@dataclass
class Decision:
    """Router.Decision: experts highest logit first, softmax over those k."""
    experts: list
    weights: list


class Router:
    def __init__(self, ctx: Context, bank: ExpertBank):
        self.ctx, self.bank = ctx, bank
        self.expert_count = bank.spec.experts
        self.hidden_size = bank.spec.hidden
        self.top_k = bank.spec.top_k

    def logits(self, hidden: np.ndarray, layer: int, dtype: str = "f16") -> np.ndarray:
        xb = _bits16(hidden, dtype)
        T = xb.size // self.hidden_size
        if xb.size != T * self.hidden_size or T == 0:
            raise GodwitCUDAError(_abi.GW_E_ARG, f"expected a multiple of {self.hidden_size} inputs")
        out = np.empty((T, self.expert_count), dtype=np.float32)
        call("gw_router_logits", self.ctx.handle, self.bank.handle, layer, _ptr(xb),
             _dtype_code(dtype), T, _ptr(out))
        return out[0] if np.asarray(hidden).ndim == 1 else out

    def route_batch(self, hidden: np.ndarray, layer: int, dtype: str = "f16"):
        xb = _bits16(hidden, dtype)
        T = xb.size // self.hidden_size
        if xb.size != T * self.hidden_size or T == 0:
            raise GodwitCUDAError(_abi.GW_E_ARG, f"expected a multiple of {self.hidden_size} inputs")
        ex = np.empty((T, self.top_k), dtype=np.int32)
        wt = np.empty((T, self.top_k), dtype=np.float32)
        call("gw_route", self.ctx.handle, self.bank.handle, layer, _ptr(xb), _dtype_code(dtype),
             T, _ptr(ex), _ptr(wt))
        return ex, wt

    def route(self, hidden: np.ndarray, layer: int, dtype: str = "f16") -> Decision:
        ex, wt = self.route_batch(np.asarray(hidden).reshape(1, -1), layer, dtype)
        return Decision(experts=[int(e) for e in ex[0]], weights=[float(w) for w in wt[0]])


@dataclass
class Assignment:
    """ExpertRunner.Assignment: one expert's work for one token."""
    expert: int
    token: int
    routing_weight: float


class ExpertRunner:
    def __init__(self, ctx: Context, bank: ExpertBank):
        self.ctx, self.bank = ctx, bank
        self.hidden_size = bank.spec.hidden
        self.intermediate_size = bank.spec.intermediate

    def apply(self, input: np.ndarray, layer: int, expert: int, dtype: str = "f16") -> np.ndarray:
        xb = _bits16(input, dtype).ravel()
        if xb.size != self.hidden_size:
            raise GodwitCUDAError(_abi.GW_E_ARG, f"expected {self.hidden_size} inputs")
        y = np.empty(self.hidden_size, dtype=np.float32)
        call("gw_expert_apply", self.ctx.handle, self.bank.handle, layer, expert, _ptr(xb),
             _dtype_code(dtype), _ptr(y))
        return y

    def apply_batch(self, input: np.ndarray, layer: int, experts: list, dtype: str = "f16") -> np.ndarray:
        xb = _bits16(input, dtype).ravel()
        if xb.size != self.hidden_size:
            raise GodwitCUDAError(_abi.GW_E_ARG, f"expected {self.hidden_size} inputs")
        ex = np.array([e for e, _ in experts], dtype=np.int32)
        wt = np.array([w for _, w in experts], dtype=np.float32)
        y = np.empty(self.hidden_size, dtype=np.float32)
        call("gw_expert_apply_batch", self.ctx.handle, self.bank.handle, layer, _ptr(xb),
             _dtype_code(dtype), len(experts), _ptr(ex), _ptr(wt), _ptr(y))
        return y

    def apply_assignments(self, inputs: np.ndarray, layer: int, assignments: list,
                          dtype: str = "f16") -> np.ndarray:
        """Applies (expert, token, weight) triples; outputs[t] = sum of weighted
        expert outputs routed to t.  Each token may list each expert once and at
        most top_k experts (the router's invariant)."""
        xb = _bits16(inputs, dtype)
        T = xb.size // self.hidden_size
        k = self.bank.spec.top_k
        ex = np.full((T, k), -1, dtype=np.int32)
        wt = np.zeros((T, k), dtype=np.float32)
        fill = np.zeros(T, dtype=np.int64)
        for a in assignments:
            t = a.token
            if not 0 <= t < T:
                raise GodwitCUDAError(_abi.GW_E_ARG, f"token {t} out of range")
            if fill[t] >= k:
                raise GodwitCUDAError(_abi.GW_E_ARG, f"token {t} has more than top_k={k} assignments")
            ex[t, fill[t]], wt[t, fill[t]] = a.expert, a.routing_weight
            fill[t] += 1
        out = np.zeros((T, self.hidden_size), dtype=np.float32)
        # Unfilled positions (-1) must be skipped: route them through the
        # fixed-routing forward, which ignores ids outside [0, E) only on the
        # device path; the host entry validates ids, so fill them per token.
        if (fill == k).all():
            call("gw_moe_forward", self.ctx.handle, self.bank.handle, layer, _ptr(xb),
                 _dtype_code(dtype), T, _ptr(ex), _ptr(wt), _ptr(out), None, None)
            return out
        for t in range(T):
            n = int(fill[t])
            if n:
                out[t] = self.apply_batch(xb[t * self.hidden_size:(t + 1) * self.hidden_size],
                                          layer, list(zip(ex[t, :n].tolist(), wt[t, :n].tolist())),
                                          dtype)
        return out


class MoEBlock:
    """Route every token, then run the experts grouped by expert, on the GPU."""

    def __init__(self, ctx: Context, bank: ExpertBank):
        self.ctx, self.bank = ctx, bank

    def forward(self, hidden: np.ndarray, layer: int, dtype: str = "f16", *,
                routing: tuple | None = None):
        xb = _bits16(hidden, dtype)
        H, k = self.bank.spec.hidden, self.bank.spec.top_k
        T = xb.size // H
        if xb.size != T * H or T == 0:
            raise GodwitCUDAError(_abi.GW_E_ARG, f"expected a multiple of {H} inputs")
        out = np.empty((T, H), dtype=np.float32)
        ex = np.empty((T, k), dtype=np.int32)
        wt = np.empty((T, k), dtype=np.float32)
        ein = win = None
        if routing is not None:
            ein = np.ascontiguousarray(routing[0], dtype=np.int32)
            win = np.ascontiguousarray(routing[1], dtype=np.float32)
        call("gw_moe_forward", self.ctx.handle, self.bank.handle, layer, _ptr(xb),
             _dtype_code(dtype), T, _ptr(ein), _ptr(win), _ptr(out), _ptr(ex), _ptr(wt))
        return out, ex, wt

    def block(self, stream: np.ndarray, layer: int, norm_weight_bits: np.ndarray, eps: float):
        """The MoE half of TransformerLayer.forward (Runtime/TransformerLayer.swift:140-238):
        RMSNorm of the fp32 residual `stream` [T, H] with the layer's bf16 post-attention
        norm weight (raw uint16 bits, [H]), routing and experts on the f16 result, and
        the weighted expert sum added into the stream.  Returns (new stream, experts,
        weights); the argument is not modified."""
        H, k = self.bank.spec.hidden, self.bank.spec.top_k
        st = np.array(stream, dtype=np.float32, order="C", copy=True).reshape(-1, H)
        nw = np.ascontiguousarray(norm_weight_bits, dtype=np.uint16)
        if nw.size != H:
            raise GodwitCUDAError(_abi.GW_E_ARG, f"norm weight has {nw.size} values, expected {H}")
        T = st.shape[0]
        ex = np.empty((T, k), dtype=np.int32)
        wt = np.empty((T, k), dtype=np.float32)
        call("gw_moe_block", self.ctx.handle, self.bank.handle, layer, _ptr(st), _ptr(nw),
             float(eps), T, _ptr(ex), _ptr(wt))
        return st, ex, wt
