"""Seeded synthetic inputs.

Two generators:

* `hash_*` — host mirror of the device generator behind
  `gw_bank_fill_synthetic` (a splitmix64 counter hash, see
  csrc/gw_internal.h:mix64).  Codes and scales are bit-identical to the
  device's; bf16 normals come from the same uniforms through Box-Muller in
  float64 and agree with the device except where the two libm's last-bit
  differences cross a bf16 rounding boundary.
* `make_expert_stride` / `make_router` — numpy `default_rng(seed)` banks for
  the parity tests: codes uniform over 0..15 (two per byte, low nibble = even
  column), E8M0 scales uniform over 118..124, bf16 biases ~N(0, 0.02),
  written into the installed stride layout (InstallLayout.swift:56-91).
  Qwen3-shaped experts are built from separate gate and up matrices
  interleaved row-wise, gate row j -> gate_up row 2j, up row j -> row 2j+1
  (Install/Installer.swift:442-455).
"""
from __future__ import annotations

import numpy as np

from .layout import ExpertLayout, ModelSpec

M64 = np.uint64(0xFFFFFFFFFFFFFFFF)


def mix64(z: np.ndarray) -> np.ndarray:
    z = np.asarray(z, dtype=np.uint64)
    with np.errstate(over="ignore"):
        z = z + np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
    return z ^ (z >> np.uint64(31))


def section_key(seed: int, layer: int, expert: int, section: int) -> int:
    inner = mix64(np.uint64((layer << 40) | (expert << 8) | section))
    return int(mix64(np.uint64(seed) ^ inner))


def hash_codes(key: int, n: int) -> np.ndarray:
    words = mix64(np.uint64(key) + np.arange((n + 7) // 8, dtype=np.uint64))
    return words.view(np.uint8)[:n].copy()  # little-endian: byte j of word = bits 8j..8j+7


def hash_scales(key: int, n: int) -> np.ndarray:
    h = mix64(np.uint64(key) + np.arange(n, dtype=np.uint64))
    return (np.uint64(118) + h % np.uint64(7)).astype(np.uint8)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bit patterns (NaN kept quiet)."""
    b = np.asarray(x, dtype=np.float32).view(np.uint32)
    rounded = (b + np.uint32(0x7FFF) + ((b >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    out = rounded.astype(np.uint16)
    out[nan] = 0x7FC0
    return out


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def hash_bf16_normal(key: int, count: int, std: float = 0.02) -> np.ndarray:
    j = np.arange(count, dtype=np.uint64)
    k = np.uint64(key)
    with np.errstate(over="ignore"):
        u1 = ((mix64(k + np.uint64(2) * j) >> np.uint64(11)).astype(np.float64) + 0.5) / 2.0 ** 53
        u2 = (mix64(k + np.uint64(2) * j + np.uint64(1)) >> np.uint64(11)).astype(np.float64) / 2.0 ** 53
    z = np.sqrt(-2.0 * np.log(u1)) * np.cos(2.0 * np.pi * u2) * std
    # as the device: float64 -> fp32 (nearest), then fp32 -> bf16 (nearest even)
    return f32_to_bf16_bits(z.astype(np.float32))


def f64_to_bf16_bits(z: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float64 -> bf16 (no double rounding through fp32)."""
    z = np.asarray(z, dtype=np.float64)
    f32 = z.astype(np.float32)  # nearest fp32
    # resolve the rare case where fp32 rounding lands exactly on a bf16 tie
    bits = f32.view(np.uint32)
    lower = bits & np.uint32(0xFFFF0000)
    upper = lower + np.uint32(0x10000)
    lo = lower.view(np.float32).astype(np.float64)
    hi = upper.view(np.float32).astype(np.float64)
    dlo, dhi = np.abs(z - lo), np.abs(z - hi)
    pick_hi = (dhi < dlo) | ((dhi == dlo) & ((lower >> np.uint32(16)) & np.uint32(1)).astype(bool))
    out = np.where(pick_hi, upper, lower) >> np.uint32(16)
    return out.astype(np.uint16)


def hash_expert_stride(spec: ModelSpec, seed: int, layer: int, expert: int) -> np.ndarray:
    """The stride gw_bank_fill_synthetic writes for (layer, expert)."""
    lay = spec.layout()
    buf = np.zeros(lay.stride, dtype=np.uint8)
    kinds = ("codes", "scales", "codes", "scales", "bf16", "bf16")
    from ._abi import SECTIONS
    for s, (name, kind) in enumerate(zip(SECTIONS, kinds)):
        key = section_key(seed, layer, expert, s)
        n, off = lay.sizes[name], lay.offsets[name]
        if kind == "codes":
            buf[off:off + n] = hash_codes(key, n)
        elif kind == "scales":
            buf[off:off + n] = hash_scales(key, n)
        elif spec.expert_bias:
            buf[off:off + n] = hash_bf16_normal(key, n // 2).view(np.uint8)
    return buf


def hash_router(spec: ModelSpec, seed: int, layer: int):
    kw = section_key(seed, layer, 0xFFFF, 6)
    kb = section_key(seed, layer, 0xFFFF, 7)
    w = hash_bf16_normal(kw, spec.experts * spec.hidden).reshape(spec.experts, spec.hidden)
    b = hash_bf16_normal(kb, spec.experts) if spec.router_bias else np.zeros(spec.experts, np.uint16)
    return w, b


# ---- numpy default_rng banks for the parity tests ---------------------------

def random_mxfp4(rng: np.random.Generator, rows: int, cols: int, lo: int = 118, hi: int = 124):
    packed = rng.integers(0, 256, size=(rows, cols // 2), dtype=np.uint8)
    scales = rng.integers(lo, hi + 1, size=(rows, cols // 32), dtype=np.uint8)
    return packed, scales


def make_expert_stride(spec: ModelSpec, rng: np.random.Generator, *,
                       separate_gate_up: bool | None = None) -> np.ndarray:
    lay = spec.layout()
    H, F = spec.hidden, spec.intermediate
    buf = np.zeros(lay.stride, dtype=np.uint8)
    if separate_gate_up is None:
        separate_gate_up = not spec.expert_bias  # Qwen3-shaped: separate projections
    if separate_gate_up:
        gp, gs = random_mxfp4(rng, F, H)
        up, us = random_mxfp4(rng, F, H)
        gu_p, gu_s = interleave_rows(gp, up), interleave_rows(gs, us)
    else:
        gu_p, gu_s = random_mxfp4(rng, 2 * F, H)
    dn_p, dn_s = random_mxfp4(rng, H, F)
    parts = {"gate_up_blocks": gu_p, "gate_up_scales": gu_s,
             "down_blocks": dn_p, "down_scales": dn_s}
    if spec.expert_bias:
        parts["gate_up_bias"] = f32_to_bf16_bits(rng.normal(0, 0.02, 2 * F))
        parts["down_bias"] = f32_to_bf16_bits(rng.normal(0, 0.02, H))
    for name, arr in parts.items():
        raw = np.ascontiguousarray(arr).view(np.uint8).ravel()
        assert raw.size == lay.sizes[name], (name, raw.size, lay.sizes[name])
        buf[lay.offsets[name]:lay.offsets[name] + raw.size] = raw
    return buf


def interleave_rows(gate: np.ndarray, up: np.ndarray) -> np.ndarray:
    """gate_up row 2j = gate row j, row 2j+1 = up row j (Installer.swift:442-455)."""
    out = np.empty((2 * gate.shape[0],) + gate.shape[1:], dtype=gate.dtype)
    out[0::2] = gate
    out[1::2] = up
    return out


def make_router(spec: ModelSpec, rng: np.random.Generator):
    w = f32_to_bf16_bits(rng.normal(0, 0.02, (spec.experts, spec.hidden)))
    b = f32_to_bf16_bits(rng.normal(0, 0.02, spec.experts)) if spec.router_bias else None
    return w, b


def make_hidden(rng: np.random.Generator, T: int, H: int, dtype: str = "bf16") -> np.ndarray:
    """Hidden states ~N(0, 1) as raw 16-bit patterns of `dtype`."""
    x = rng.standard_normal((T, H)).astype(np.float32)
    if dtype == "bf16":
        return f32_to_bf16_bits(x)
    return x.astype(np.float16).view(np.uint16)


def as_f32(bits: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "bf16":
        return bf16_bits_to_f32(bits)
    return np.asarray(bits, dtype=np.uint16).view(np.float16).astype(np.float32)
