"""Python face of the CPU oracle — TEST INFRASTRUCTURE ONLY.

Wraps oracle/liboracle.so (the C restatement in mxfp4_oracle.c) and adds an
fp64 NumPy restatement of the MoE layer for the rel-L2 gate.  Only tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline leg import this module;
the product library never calls it.

Parity pinning: see tests/test_oracle_kats.py (the reference's own
known-answer tests) and tests/golden/ (vectors produced by importing the
reference's NumPy twin, Scripts/analysis/expert_reference.py).
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "liboracle.so")

_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            import subprocess
            import sys
            subprocess.run([sys.executable, os.path.join(os.path.dirname(HERE), "godwit_b200",
                                                         "build.py")], check=True)
        L = C.CDLL(LIB)
        P, I64, F = C.c_void_p, C.c_int64, C.c_float
        L.gwo_decode_scale.restype = F
        L.gwo_decode_scale.argtypes = [C.c_uint8]
        L.gwo_codebook.restype = F
        L.gwo_codebook.argtypes = [C.c_int]
        L.gwo_decode.argtypes = [P, P, I64, P]
        L.gwo_scale_byte_for_peak.restype = C.c_uint8
        L.gwo_scale_byte_for_peak.argtypes = [F]
        L.gwo_code_for_magnitude.restype = C.c_uint8
        L.gwo_code_for_magnitude.argtypes = [F]
        L.gwo_encode.restype = I64
        L.gwo_encode.argtypes = [P, I64, P, P]
        L.gwo_gemv.argtypes = [P, P, P, P, I64, I64, P]
        L.gwo_gemv_mt.argtypes = [P, P, P, P, I64, I64, P, C.c_int]
        L.gwo_router_logits.argtypes = [P, P, P, I64, I64, P]
        L.gwo_router_select.argtypes = [P, C.c_int, C.c_int, P, P]
        L.gwo_act_gptoss.argtypes = [P, I64, F, F, P]
        L.gwo_act_silu.argtypes = [P, I64, P]
        L.gwo_expert_apply.argtypes = [P, P, I64, I64, C.c_int, F, F, P, P]
        L.gwo_moe_layer.argtypes = [P, I64, P, I64, I64, I64, C.c_int, C.c_int, F, F, P, P, P,
                                    I64, P, P, P, P, P]
        L.gwo_moe_layer_mt.argtypes = [P, I64, P, I64, I64, I64, C.c_int, C.c_int, F, F, P, P,
                                       P, I64, P, P, P, C.c_int]
        L.gwo_dequant64_mt.argtypes = [P, P, I64, I64, P, C.c_int]
        L.gwo_bf16_from_f32.restype = C.c_uint16
        L.gwo_bf16_from_f32.argtypes = [F]
        L.gwo_int8_quantize_row.restype = C.c_int
        L.gwo_int8_quantize_row.argtypes = [P, I64, P, P, P]
        L.gwo_int8_dequant.argtypes = [P, P, I64, I64, P]
        L.gwo_int8_gemv_mt.argtypes = [P, P, P, P, I64, I64, I64, P, C.c_int]
        _lib = L
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


# ---- MXFP4 codec (MXFP4.swift) ---------------------------------------------

def decode_scale(byte: int) -> float:
    return lib().gwo_decode_scale(byte)


def codebook() -> np.ndarray:
    return np.array([lib().gwo_codebook(i) for i in range(16)], dtype=np.float32)


def decode(packed: np.ndarray, scales: np.ndarray) -> np.ndarray:
    packed = np.ascontiguousarray(packed, dtype=np.uint8)
    scales = np.ascontiguousarray(scales, dtype=np.uint8)
    nb = scales.size
    out = np.empty(nb * 32, dtype=np.float32)
    lib().gwo_decode(_p(packed), _p(scales), nb, _p(out))
    return out


def dequant(packed: np.ndarray, scales: np.ndarray) -> np.ndarray:
    rows = packed.shape[0]
    return decode(packed, scales).reshape(rows, -1)


def scale_byte_for_peak(peak: float) -> int:
    return lib().gwo_scale_byte_for_peak(peak)


def code_for_magnitude(v: float) -> int:
    return lib().gwo_code_for_magnitude(v)


def encode(w: np.ndarray):
    w = _f32(w).ravel()
    nb = (w.size + 31) // 32
    packed = np.zeros(nb * 16, dtype=np.uint8)
    scales = np.zeros(nb, dtype=np.uint8)
    lib().gwo_encode(_p(w), w.size, _p(packed), _p(scales))
    return packed, scales


# ---- GEMV / router / activation / expert / layer ----------------------------

def gemv(packed, scales, x, bias=None, threads: int = 1) -> np.ndarray:
    """referenceMXFP4 (+ bias): x and bias as float values."""
    packed = np.ascontiguousarray(packed, dtype=np.uint8)
    scales = np.ascontiguousarray(scales, dtype=np.uint8)
    rows, cols = packed.shape[0], packed.shape[1] * 2
    x = _f32(x)
    b = None if bias is None else _f32(bias)
    y = np.empty(rows, dtype=np.float32)
    if threads > 1:
        lib().gwo_gemv_mt(_p(packed), _p(scales), _p(b), _p(x), rows, cols, _p(y), threads)
    else:
        lib().gwo_gemv(_p(packed), _p(scales), _p(b), _p(x), rows, cols, _p(y))
    return y


def router_logits(w_bf16, b_bf16, x) -> np.ndarray:
    w = np.ascontiguousarray(w_bf16, dtype=np.uint16)
    E, H = w.shape
    b = None if b_bf16 is None else np.ascontiguousarray(b_bf16, dtype=np.uint16)
    out = np.empty(E, dtype=np.float32)
    lib().gwo_router_logits(_p(w), _p(b), _p(_f32(x)), E, H, _p(out))
    return out


def router_select(logits, k: int):
    lg = _f32(logits)
    ex = np.empty(k, dtype=np.int32)
    wt = np.empty(k, dtype=np.float32)
    lib().gwo_router_select(_p(lg), lg.size, k, _p(ex), _p(wt))
    return ex, wt


def act_gptoss(gate_up, limit=7.0, alpha=1.702):
    gu = _f32(gate_up)
    out = np.empty(gu.size // 2, dtype=np.float32)
    lib().gwo_act_gptoss(_p(gu), gu.size // 2, limit, alpha, _p(out))
    return out


def act_silu(gate_up):
    gu = _f32(gate_up)
    out = np.empty(gu.size // 2, dtype=np.float32)
    lib().gwo_act_silu(_p(gu), gu.size // 2, _p(out))
    return out


def _offsets(spec) -> np.ndarray:
    from godwit_b200._abi import SECTIONS
    lay = spec.layout()
    return np.array([lay.offsets[s] for s in SECTIONS], dtype=np.int64)


def expert_apply(spec, stride: np.ndarray, x) -> np.ndarray:
    so = _offsets(spec)
    y = np.empty(spec.hidden, dtype=np.float32)
    lib().gwo_expert_apply(_p(np.ascontiguousarray(stride, dtype=np.uint8)), _p(so), spec.hidden,
                           spec.intermediate, spec.activation, spec.limit, spec.alpha,
                           _p(_f32(x)), _p(y))
    return y


def moe_layer(spec, strides: np.ndarray, router_w, router_b, x, routing=None, threads: int = 1):
    """strides: uint8 [E, stride] of one layer; x float [T, H].
    Returns (out [T, H], experts [T, k], weights [T, k])."""
    so = _offsets(spec)
    strides = np.ascontiguousarray(strides, dtype=np.uint8)
    x = _f32(x)
    T = x.shape[0]
    k = spec.top_k
    out = np.empty((T, spec.hidden), dtype=np.float32)
    ex = np.empty((T, k), dtype=np.int32)
    wt = np.empty((T, k), dtype=np.float32)
    rw = np.ascontiguousarray(router_w, dtype=np.uint16)
    rb = None if router_b is None else np.ascontiguousarray(router_b, dtype=np.uint16)
    if routing is None and threads > 1:
        lib().gwo_moe_layer_mt(_p(strides), strides.shape[1], _p(so), spec.hidden,
                               spec.intermediate, spec.experts, k, spec.activation, spec.limit,
                               spec.alpha, _p(rw), _p(rb), _p(x), T, _p(out), _p(ex), _p(wt),
                               threads)
        return out, ex, wt
    ein = win = None
    if routing is not None:
        ein = np.ascontiguousarray(routing[0], dtype=np.int32)
        win = np.ascontiguousarray(routing[1], dtype=np.float32)
    lib().gwo_moe_layer(_p(strides), strides.shape[1], _p(so), spec.hidden, spec.intermediate,
                        spec.experts, k, spec.activation, spec.limit, spec.alpha, _p(rw), _p(rb),
                        _p(x), T, _p(ein), _p(win), _p(out), _p(ex), _p(wt))
    return out, ex, wt


# ---- fp64 NumPy restatement (layer_reference.py:70-98, expert_reference.py:35-74) ----

FP4 = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
                -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0], dtype=np.float64)


def dequant64(packed: np.ndarray, scales: np.ndarray) -> np.ndarray:
    rows = packed.shape[0]
    nb = scales.shape[1]
    blocks = packed.reshape(rows, nb, 16)
    out = np.empty((rows, nb, 32), dtype=np.float64)
    out[:, :, 0::2] = FP4[blocks & 0x0F]
    out[:, :, 1::2] = FP4[blocks >> 4]
    out *= np.exp2(scales.astype(np.float64) - 127.0)[:, :, None]
    return out.reshape(rows, nb * 32)


def dequant64_fast(packed: np.ndarray, scales: np.ndarray, rows: int, cols: int) -> np.ndarray:
    """dequant64 through the C restatement, row-parallel on all host threads
    (same values: every code x 2^(scale-127) is exact in fp64)."""
    out = np.empty((rows, cols), dtype=np.float64)
    lib().gwo_dequant64_mt(_p(np.ascontiguousarray(packed, dtype=np.uint8)),
                           _p(np.ascontiguousarray(scales, dtype=np.uint8)), rows, cols, _p(out),
                           os.cpu_count() or 1)
    return out


def expert_sections(spec, stride: np.ndarray):
    from godwit_b200.synth import bf16_bits_to_f32
    lay = spec.layout()
    H, F = spec.hidden, spec.intermediate

    def sec(name):
        o = lay.offsets[name]
        return stride[o:o + lay.sizes[name]]

    gu = dequant64_fast(sec("gate_up_blocks"), sec("gate_up_scales"), 2 * F, H)
    dn = dequant64_fast(sec("down_blocks"), sec("down_scales"), H, F)
    gb = bf16_bits_to_f32(sec("gate_up_bias").view(np.uint16)).astype(np.float64)
    db = bf16_bits_to_f32(sec("down_bias").view(np.uint16)).astype(np.float64)
    return gu, gb, dn, db


def expert64(spec, stride: np.ndarray, x: np.ndarray, round_act: bool = True, cache=None) -> np.ndarray:
    gu, gb, dn, db = cache if cache is not None else expert_sections(spec, stride)
    g = gu @ np.asarray(x, np.float64) + gb
    gate, up = g[0::2], g[1::2]
    if spec.activation == 0:
        gate = np.minimum(gate, spec.limit)
        up = np.clip(up, -spec.limit, spec.limit)
        a = (up + 1.0) * (gate / (1.0 + np.exp(-spec.alpha * gate)))
    else:
        a = (gate / (1.0 + np.exp(-gate))) * up
    if round_act:  # the reference stores the activation as half (expert.metal:101)
        a = a.astype(np.float16).astype(np.float64)
    return dn @ a + db


def moe_layer64(spec, strides: np.ndarray, x: np.ndarray, experts: np.ndarray,
                weights: np.ndarray, round_act: bool = True) -> np.ndarray:
    """fp64 layer for a given routing (selection is checked separately),
    expert-major so each expert is dequantised once."""
    T = x.shape[0]
    x = np.asarray(x, np.float64)
    out = np.zeros((T, spec.hidden), dtype=np.float64)
    for e in np.unique(experts):
        if e < 0:
            continue
        gu, gb, dn, db = expert_sections(spec, strides[int(e)])
        tt, jj = np.nonzero(experts == e)
        g = x[tt] @ gu.T + gb
        gate, up = g[:, 0::2], g[:, 1::2]
        if spec.activation == 0:
            gate = np.minimum(gate, spec.limit)
            up = np.clip(up, -spec.limit, spec.limit)
            a = (up + 1.0) * (gate / (1.0 + np.exp(-spec.alpha * gate)))
        else:
            a = (gate / (1.0 + np.exp(-gate))) * up
        if round_act:
            a = a.astype(np.float16).astype(np.float64)
        y = a @ dn.T + db
        np.add.at(out, tt, y * np.asarray(weights, np.float64)[tt, jj][:, None])
    return out


# ---- MXFP8 activations (config 4's block-scaled tensor-core mode) ----------
#
# Not part of the reference (which feeds f16 activations to every expert
# GEMV); it restates the OCP MX recipe the device quantiser follows, so the
# block-scaled path has an exact oracle: per 32-value block along K, shared
# exponent X = floor(log2(max |x|)) - 8 (8 = E4M3's largest exponent), stored
# as the E8M0 byte X + 127 clamped to [0, 254] (0 for an all-zero block);
# elements = x / 2^X rounded to nearest-even E4M3, saturated to +-448.

def quantize_mxfp8(x: np.ndarray):
    """x [rows, K] (K % 32 == 0) -> (codes uint8 [rows, K] E4M3, scales
    uint8 [rows, K/32] E8M0)."""
    import ml_dtypes
    x = np.asarray(x, np.float32)
    rows, K = x.shape
    xb = x.reshape(rows, K // 32, 32)
    amax = np.abs(xb).max(-1)
    _, ex = np.frexp(amax)                      # amax = m * 2^ex, m in [0.5, 1)
    byte = np.where(amax > 0, np.clip(ex - 1 - 8 + 127, 0, 254), 0).astype(np.int64)
    q = xb * np.exp2(127.0 - byte)[..., None]   # exact power-of-two scaling (float64)
    q = np.clip(q, -448.0, 448.0).astype(np.float32).astype(ml_dtypes.float8_e4m3fn)
    return q.view(np.uint8).reshape(rows, K), byte.astype(np.uint8)


def dequantize_mxfp8(codes: np.ndarray, scales: np.ndarray) -> np.ndarray:
    import ml_dtypes
    rows, K = codes.shape
    v = codes.view(ml_dtypes.float8_e4m3fn).astype(np.float64).reshape(rows, K // 32, 32)
    return (v * np.exp2(scales.astype(np.float64) - 127.0)[..., None]).reshape(rows, K)


def moe_layer64_mx(spec, strides: np.ndarray, x: np.ndarray, experts: np.ndarray,
                   weights: np.ndarray) -> np.ndarray:
    """moe_layer64 with the block-scaled mode's activation handling: the
    expert inputs quantised to MXFP8, the activations rounded to f16 (as the
    reference stores them) and then quantised to MXFP8 for the down
    projection."""
    T = x.shape[0]
    xq = dequantize_mxfp8(*quantize_mxfp8(np.asarray(x, np.float32)))
    out = np.zeros((T, spec.hidden), dtype=np.float64)
    for e in np.unique(experts):
        if e < 0:
            continue
        gu, gb, dn, db = expert_sections(spec, strides[int(e)])
        tt, jj = np.nonzero(experts == e)
        g = xq[tt] @ gu.T + gb
        gate, up = g[:, 0::2], g[:, 1::2]
        if spec.activation == 0:
            gate = np.minimum(gate, spec.limit)
            up = np.clip(up, -spec.limit, spec.limit)
            a = (up + 1.0) * (gate / (1.0 + np.exp(-spec.alpha * gate)))
        else:
            a = (gate / (1.0 + np.exp(-gate))) * up
        a = a.astype(np.float16).astype(np.float32)
        a = dequantize_mxfp8(*quantize_mxfp8(a))
        y = a @ dn.T + db
        np.add.at(out, tt, y * np.asarray(weights, np.float64)[tt, jj][:, None])
    return out


def rmsnorm(stream: np.ndarray, weight_bits: np.ndarray, eps: float) -> np.ndarray:
    """TransformerLayer.normalise (Runtime/TransformerLayer.swift:265-285): per token,
    sumSquares accumulated in index order in fp32 (value * value, then +=),
    inverse = 1 / sqrt(sumSquares / width + eps) in fp32, out = Float16(value *
    inverse * bf16(weight)).  stream fp32 [T, H], weight_bits uint16 [H] -> f16 [T, H]."""
    x = np.asarray(stream, dtype=np.float32)
    x = x.reshape(-1, x.shape[-1])
    H = x.shape[1]
    w = (np.asarray(weight_bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)
    # np.cumsum over float32 adds strictly left to right (no pairwise blocking)
    ss = np.cumsum(x * x, axis=1, dtype=np.float32)[:, -1]
    inv = np.float32(1) / np.sqrt(ss / np.float32(H) + np.float32(eps))
    return ((x * inv[:, None]) * w[None, :]).astype(np.float16)


def moe_block64(spec, strides: np.ndarray, stream: np.ndarray, normed: np.ndarray,
                experts: np.ndarray, weights: np.ndarray) -> np.ndarray:
    """The MoE half of TransformerLayer.forward (:140-238) in fp64 given the
    normed f16 input and the routing: stream + moe_layer64(normed)."""
    return np.asarray(stream, dtype=np.float64) + moe_layer64(spec, strides, normed.astype(np.float64),
                                                              experts, weights)


# ---- int8 affine trunk projections (Install/Int8Affine.swift, router.metal:65-141)

def bf16_from_f32(v: float) -> int:
    """BFloat16.fromFloat (Int8Affine.swift:89-96)."""
    return int(lib().gwo_bf16_from_f32(float(v)))


def int8_quantize_row(row):
    """Int8Affine.quantize(row:) -> (codes uint8 [n], scale fp32 [n/64], zero fp32 [n/64])."""
    row = _f32(row)
    n = row.size
    codes = np.empty(n, np.uint8)
    scale = np.empty(n // 64, np.float32)
    zero = np.empty(n // 64, np.float32)
    if lib().gwo_int8_quantize_row(_p(row), n, _p(codes), _p(scale), _p(zero)) != 0:
        raise ValueError(f"row width {n} is not a multiple of 64")
    return codes, scale, zero


def int8_quantize(w):
    """A [rows, cols] fp32 matrix -> (codes uint8 [rows, cols], meta uint16 bf16 bits
    [rows, cols/64, 2]) in the installer's trunk layout (Installer.swift:315-345)."""
    w = _f32(w)
    rows, cols = w.shape
    codes = np.empty((rows, cols), np.uint8)
    meta = np.empty((rows, cols // 64, 2), np.uint16)
    for r in range(rows):
        c, s, z = int8_quantize_row(w[r])
        codes[r] = c
        meta[r, :, 0] = [bf16_from_f32(v) for v in s]
        meta[r, :, 1] = [bf16_from_f32(v) for v in z]
    return codes, meta


def int8_dequant(codes, meta) -> np.ndarray:
    codes = np.ascontiguousarray(codes, np.uint8)
    meta = np.ascontiguousarray(meta, np.uint16)
    rows, cols = codes.shape
    out = np.empty((rows, cols), np.float32)
    lib().gwo_int8_dequant(_p(codes), _p(meta), rows, cols, _p(out))
    return out


def int8_gemv(codes, meta, x, bias=None, threads: int = 1) -> np.ndarray:
    """fp32 restatement of int8_affine_gemv(_bias_batched): x [T, cols] (f16
    values) -> [T, rows] fp32 (before the batched kernel's f16 rounding)."""
    codes = np.ascontiguousarray(codes, np.uint8)
    meta = np.ascontiguousarray(meta, np.uint16)
    rows, cols = codes.shape
    x = _f32(np.atleast_2d(x))
    T = x.shape[0]
    b = None if bias is None else np.ascontiguousarray(bias, np.uint16)
    y = np.empty((T, rows), np.float32)
    lib().gwo_int8_gemv_mt(_p(codes), _p(meta), _p(b), _p(x), T, rows, cols, _p(y), threads)
    return y


def int8_gemv64(codes, meta, x, bias=None) -> np.ndarray:
    """fp64 restatement of the same projection: (code*scale + zero) . x + bias."""
    codes = np.asarray(codes, np.uint8)
    rows, cols = codes.shape
    m = np.asarray(meta, np.uint16).reshape(rows, cols // 64, 2).astype(np.uint32) << 16
    sc = m[..., 0].view(np.float32).astype(np.float64)
    zr = m[..., 1].view(np.float32).astype(np.float64)
    w = codes.reshape(rows, cols // 64, 64).astype(np.float64) * sc[..., None] + zr[..., None]
    y = np.atleast_2d(np.asarray(x, np.float64)) @ w.reshape(rows, cols).T
    if bias is not None:
        y = y + (np.asarray(bias, np.uint16).astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    return y


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))
