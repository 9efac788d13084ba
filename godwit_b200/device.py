"""Stream-ordered device-pointer API over torch tensors.

PyTorch supplies device memory, the current stream and torch.distributed;
every kernel that runs is this library's.  Tensors are passed as raw device
pointers to the `_async` entry points of include/godwit_cuda.h on the
current torch stream.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _abi
from ._abi import GW_DTYPE_BF16, GW_DTYPE_F16, call
from .runtime import Context, ExpertBank

_TORCH_DTYPES = {torch.float16: GW_DTYPE_F16, torch.bfloat16: GW_DTYPE_BF16}


def _p(t: torch.Tensor | None):
    return None if t is None else C.c_void_p(t.data_ptr())


def dtype_code(t: torch.Tensor) -> int:
    try:
        return _TORCH_DTYPES[t.dtype]
    except KeyError:
        raise _abi.GodwitCUDAError(_abi.GW_E_ARG, f"unsupported activation dtype {t.dtype}") from None


def bind_stream(ctx: Context, stream: torch.cuda.Stream | None = None) -> torch.cuda.Stream:
    """Orders the library's work on `stream` (default: torch's current stream).

    The legacy default stream has handle 0, which the C-ABI reads as "the
    context's own stream"; in that case a dedicated torch stream is created and
    made current, so torch ops, CUDA events and the library share one stream.
    """
    s = stream or torch.cuda.current_stream(ctx.device)
    if s.cuda_stream == 0:
        s = torch.cuda.Stream(device=ctx.device)
        torch.cuda.set_stream(s)
    ctx.set_stream(s.cuda_stream)
    return s


def gemv_batched(ctx: Context, packed: torch.Tensor, scales: torch.Tensor, bias: torch.Tensor | None,
                 x: torch.Tensor, y: torch.Tensor) -> None:
    """packed [R, rows, cols/2] u8, scales [R, rows, cols/32] u8, bias [R, rows]
    bf16 (as int16/uint16/bf16 storage) or None, x [R or 1, cols], y [R, rows] f32."""
    R, rows, half = packed.shape
    cols = half * 2
    x_stride = 0 if x.shape[0] == 1 else x.stride(0)
    call("gw_mxfp4_gemv_batched_async", ctx.handle, R, _p(packed), packed.stride(0), _p(scales),
         scales.stride(0), _p(bias), 0 if bias is None else bias.stride(0), _p(x), x_stride,
         dtype_code(x), _p(y), y.stride(0), rows, cols)


def int8_affine_gemv(ctx: Context, codes: torch.Tensor, meta: torch.Tensor, bias: torch.Tensor | None,
                     x: torch.Tensor, y: torch.Tensor) -> None:
    """codes [rows, cols] u8, meta [rows, cols/64, 2] bf16 bits (any 16-bit
    storage), bias [rows] bf16 bits or None, x [T, cols] f16 -> y [T, rows]
    (float32: int8_affine_gemv; float16: int8_affine_gemv_bias_batched)."""
    rows, cols = codes.shape
    if x.dtype != torch.float16:
        raise _abi.GodwitCUDAError(_abi.GW_E_ARG, f"x must be float16 (got {x.dtype})")
    code = {torch.float32: _abi.GW_DTYPE_F32, torch.float16: GW_DTYPE_F16}.get(y.dtype)
    if code is None:
        raise _abi.GodwitCUDAError(_abi.GW_E_ARG, f"y must be float32 or float16 (got {y.dtype})")
    call("gw_int8_affine_gemv_async", ctx.handle, _p(codes), _p(meta), _p(bias), _p(x), x.shape[0], rows,
         cols, _p(y), code)


def moe_forward(ctx: Context, bank: ExpertBank, layer: int, x: torch.Tensor, out: torch.Tensor,
                experts: torch.Tensor | None = None, weights: torch.Tensor | None = None) -> None:
    T = x.shape[0]
    call("gw_moe_forward_async", ctx.handle, bank.handle, layer, _p(x), dtype_code(x), T, _p(out),
         _p(experts), _p(weights))


def moe_forward_noalloc(ctx: Context, bank: ExpertBank, layer: int, x: torch.Tensor,
                        out: torch.Tensor, experts: torch.Tensor | None = None,
                        weights: torch.Tensor | None = None) -> None:
    """moe_forward without any device allocation: the layer's scratch is the
    library's fixed device array (for callers that plan memory up front or may
    not allocate while serving).  Limited to small T; calls must not overlap."""
    call("gw_moe_forward_noalloc_async", ctx.handle, bank.handle, layer, _p(x), dtype_code(x),
         x.shape[0], _p(out), _p(experts), _p(weights))


def moe_apply(ctx: Context, bank: ExpertBank, layer: int, x: torch.Tensor, experts: torch.Tensor,
              weights: torch.Tensor, out: torch.Tensor, accumulate: bool = False) -> None:
    call("gw_moe_apply_async", ctx.handle, bank.handle, layer, _p(x), dtype_code(x), x.shape[0],
         _p(experts), _p(weights), _p(out), 1 if accumulate else 0)


def moe_stack(ctx: Context, bank: ExpertBank, x: torch.Tensor, stream_out: torch.Tensor) -> None:
    call("gw_moe_stack_forward_async", ctx.handle, bank.handle, _p(x), dtype_code(x), x.shape[0],
         _p(stream_out))


def residual_round(ctx: Context, stream: torch.Tensor, delta: torch.Tensor | None,
                   x_out: torch.Tensor | None) -> None:
    call("gw_residual_round_async", ctx.handle, _p(stream), _p(delta), _p(x_out),
         GW_DTYPE_BF16 if x_out is None else dtype_code(x_out), stream.numel())


def rmsnorm(ctx: Context, stream: torch.Tensor, weight_bits: torch.Tensor, eps: float,
            out: torch.Tensor) -> None:
    """out [T, H] f16 = RMSNorm(stream [T, H] fp32) with the bf16 weight (int16/uint16 bits or bfloat16)."""
    T, H = stream.shape
    call("gw_rmsnorm_async", ctx.handle, _p(stream), _p(weight_bits), float(eps), T, H, _p(out))


def moe_block(ctx: Context, bank: ExpertBank, layer: int, stream: torch.Tensor, norm_weight: torch.Tensor,
              eps: float, experts: torch.Tensor | None = None, weights: torch.Tensor | None = None) -> None:
    """The MoE half of a transformer layer on device tensors: stream [T, H] fp32
    += MoE(RMSNorm(stream)) in place (norm_weight: bf16 bits [H])."""
    call("gw_moe_block_async", ctx.handle, bank.handle, layer, _p(stream), _p(norm_weight), float(eps),
         stream.shape[0], _p(experts), _p(weights))


def route(ctx: Context, bank: ExpertBank, layer: int, x: torch.Tensor, experts: torch.Tensor,
          weights: torch.Tensor) -> None:
    """experts [T, k] int32, weights [T, k] fp32 = the router's decision for x [T, H]."""
    call("gw_route_async", ctx.handle, bank.handle, layer, _p(x), dtype_code(x), x.shape[0], _p(experts),
         _p(weights))
