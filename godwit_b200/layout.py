"""Expert stride layout and model presets.

`ExpertLayout` restates `ExpertLayout.init` (Sources/Godwit/Install/InstallLayout.swift:50-92):
six sections per expert in the order gate_up_blocks, gate_up_scales,
down_blocks, down_scales, gate_up_bias, down_bias, each starting on a 16 KiB
page, the stride rounded up to a page.  The presets mirror ArchitectureSpec's
(Sources/Godwit/Model/ArchitectureSpec.swift:207-299).
"""
from __future__ import annotations

from dataclasses import dataclass, field

from ._abi import GW_ACT_GPTOSS_CLAMPED, GW_ACT_SILU, SECTIONS, BankDesc

PAGE = 16384


def align_up(v: int) -> int:
    return (v + PAGE - 1) // PAGE * PAGE


@dataclass
class ExpertLayout:
    hidden: int
    intermediate: int
    experts: int
    offsets: dict = field(init=False)
    sizes: dict = field(init=False)
    stride: int = field(init=False)

    def __post_init__(self):
        H, F = self.hidden, self.intermediate
        gu_rows, dn_rows = 2 * F, H
        self.sizes = {
            "gate_up_blocks": gu_rows * (H // 32) * 16,
            "gate_up_scales": gu_rows * (H // 32),
            "down_blocks": dn_rows * (F // 32) * 16,
            "down_scales": dn_rows * (F // 32),
            "gate_up_bias": gu_rows * 2,
            "down_bias": dn_rows * 2,
        }
        cursor = 0
        self.offsets = {}
        for s in SECTIONS:
            cursor = align_up(cursor)
            self.offsets[s] = cursor
            cursor += self.sizes[s]
        self.stride = align_up(cursor)

    @property
    def payload_per_expert(self) -> int:
        return sum(self.sizes.values())

    @property
    def layer_file_size(self) -> int:
        return self.stride * self.experts

    def expert_offset(self, expert: int) -> int:
        if not 0 <= expert < self.experts:
            raise IndexError(f"expert {expert} out of range")
        return expert * self.stride


@dataclass(frozen=True)
class ModelSpec:
    """The expert-path slice of ArchitectureSpec."""
    name: str
    hidden: int
    intermediate: int
    experts: int
    layers: int
    top_k: int
    activation: int
    limit: float = 7.0
    alpha: float = 1.702
    expert_bias: bool = True
    router_bias: bool = True

    def layout(self) -> ExpertLayout:
        return ExpertLayout(self.hidden, self.intermediate, self.experts)

    def desc(self, shard_rank: int = 0, shard_count: int = 1, layers: int | None = None) -> BankDesc:
        lay = self.layout()
        d = BankDesc()
        d.hidden, d.intermediate, d.experts = self.hidden, self.intermediate, self.experts
        d.layers = self.layers if layers is None else layers
        d.top_k, d.activation = self.top_k, self.activation
        d.limit, d.alpha = self.limit, self.alpha
        d.has_router_bias = 1 if self.router_bias else 0
        d.shard_rank, d.shard_count = shard_rank, shard_count
        d.expert_stride = lay.stride
        for i, s in enumerate(SECTIONS):
            d.section_offset[i] = lay.offsets[s]
            d.section_length[i] = lay.sizes[s]
        return d

    def with_(self, **kw) -> "ModelSpec":
        args = dict(self.__dict__)
        args.update(kw)
        return ModelSpec(**args)

    # Algorithmic bytes (the roofline numerators).
    @property
    def expert_weight_bytes(self) -> int:
        """MXFP4 packed + scale bytes of one expert (both projections)."""
        lay = self.layout()
        return sum(lay.sizes[s] for s in SECTIONS[:4])

    @property
    def expert_bias_bytes(self) -> int:
        return (4 * self.intermediate + 2 * self.hidden) if self.expert_bias else 0

    @property
    def router_bytes(self) -> int:
        return self.experts * self.hidden * 2 + (self.experts * 2 if self.router_bias else 0)


GPT_OSS_20B = ModelSpec("gpt-oss-20b", 2880, 2880, 32, 24, 4, GW_ACT_GPTOSS_CLAMPED)
GPT_OSS_120B = ModelSpec("gpt-oss-120b", 2880, 2880, 128, 36, 4, GW_ACT_GPTOSS_CLAMPED)
QWEN3_30B_A3B = ModelSpec("qwen3-30b-a3b", 2048, 768, 128, 48, 8, GW_ACT_SILU,
                          expert_bias=False, router_bias=False)

PRESETS = {s.name: s for s in (GPT_OSS_20B, GPT_OSS_120B, QWEN3_30B_A3B)}
