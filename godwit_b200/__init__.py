"""godwit_b200 — B200-native (sm_100a) MoE expert hot path of rayl15/Godwit.

The compute lives in `libgodwit_cuda.so` (CUDA kernels behind the C-ABI of
include/godwit_cuda.h).  This package holds the ctypes binding, the host-side
mirror of the reference's Router / ExpertRunner interfaces, the stride layout
and model presets, the seeded synthetic generators, and the expert-parallel
orchestration over torch.distributed.
"""
from ._abi import (GW_ACT_GPTOSS_CLAMPED, GW_ACT_SILU, GW_DTYPE_BF16, GW_DTYPE_F16,
                   GodwitCUDAError, LIB_PATH, load)
from .layout import GPT_OSS_20B, GPT_OSS_120B, PRESETS, QWEN3_30B_A3B, ExpertLayout, ModelSpec

__all__ = ["GodwitCUDAError", "LIB_PATH", "load", "ExpertLayout", "ModelSpec", "PRESETS",
           "GPT_OSS_20B", "GPT_OSS_120B", "QWEN3_30B_A3B", "GW_ACT_GPTOSS_CLAMPED",
           "GW_ACT_SILU", "GW_DTYPE_F16", "GW_DTYPE_BF16"]
