"""The C-ABI library loads and exports every symbol include/godwit_cuda.h
declares; host-side checks that need no GPU."""
import ctypes as C
import os
import re

import numpy as np
import pytest

from godwit_b200 import _abi
from godwit_b200.layout import GPT_OSS_20B, GPT_OSS_120B, QWEN3_30B_A3B, ExpertLayout
from godwit_b200 import synth

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "godwit_cuda.h")


def declared_functions():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^GW_API\s+[\w\s\*]+?\b(gw_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_the_boundary():
    names = declared_functions()
    for required in ("gw_init", "gw_shutdown", "gw_bank_create", "gw_bank_upload_expert",
                     "gw_bank_upload_router", "gw_route", "gw_expert_apply", "gw_moe_forward",
                     "gw_mxfp4_gemv", "gw_mxfp4_dequant", "gw_sync", "gw_last_error"):
        assert required in names


def test_library_exports_every_declared_symbol():
    lib = C.CDLL(_abi.LIB_PATH)
    for name in declared_functions():
        assert hasattr(lib, name), name
    assert set(declared_functions()) == set(_abi.SIGNATURES), \
        set(declared_functions()) ^ set(_abi.SIGNATURES)


def test_version_and_empty_error():
    lib = _abi.load()
    assert lib.gw_version() >= 100
    assert lib.gw_last_error() is not None


def test_layout_default_matches_python_layout():
    lib = _abi.load()
    for spec in (GPT_OSS_20B, GPT_OSS_120B, QWEN3_30B_A3B):
        d = _abi.BankDesc()
        _abi.check(lib.gw_layout_default(spec.hidden, spec.intermediate, spec.experts,
                                         spec.layers, spec.top_k, spec.activation, C.byref(d)))
        lay = spec.layout()
        assert d.expert_stride == lay.stride
        for i, s in enumerate(_abi.SECTIONS):
            assert d.section_offset[i] == lay.offsets[s]
            assert d.section_length[i] == lay.sizes[s]


def test_layout_default_rejects_bad_shapes():
    lib = _abi.load()
    d = _abi.BankDesc()
    st = lib.gw_layout_default(2880, 100, 32, 1, 4, 0, C.byref(d))
    assert st == _abi.GW_E_ARG
    assert b"multiples of 32" in lib.gw_last_error()


def test_null_arguments_rejected_before_any_device_work():
    lib = _abi.load()
    assert lib.gw_init(0, None) == _abi.GW_E_ARG
    assert lib.gw_sync(None) == _abi.GW_E_ARG
    assert lib.gw_bank_destroy(None) == _abi.GW_E_ARG
    assert lib.gw_shutdown(None) == _abi.GW_E_ARG
    assert lib.gw_int8_affine_gemv(None, None, None, None, None, 1, 16, 64, None, _abi.GW_DTYPE_F32) == _abi.GW_E_ARG
    assert lib.gw_int8_affine_gemv_async(None, None, None, None, None, 1, 16, 64, None,
                                         _abi.GW_DTYPE_F32) == _abi.GW_E_ARG
    assert lib.gw_ep_dispatch_async(None, None, None, 0, 1, None, None, 2, 4, None, None, None) == _abi.GW_E_ARG
    assert lib.gw_ep_combine_async(None, None, None, None, 1, None) == _abi.GW_E_ARG
    assert lib.gw_moe_forward_noalloc_async(None, None, 0, None, 0, 1, None, None, None) == _abi.GW_E_ARG


def test_synthetic_hash_generator_is_deterministic_and_in_range():
    key = synth.section_key(1234, 3, 17, 1)
    s = synth.hash_scales(key, 1000)
    assert s.min() >= 118 and s.max() <= 124 and len(set(s.tolist())) == 7
    c = synth.hash_codes(key, 4096)
    assert np.array_equal(c, synth.hash_codes(key, 4096))
    assert abs(c.mean() - 127.5) < 8
    b = synth.bf16_bits_to_f32(synth.hash_bf16_normal(key, 20000))
    assert abs(b.std() - 0.02) < 0.001 and abs(b.mean()) < 0.001
    assert synth.mix64(np.uint64(0)) == np.uint64(0xE220A8397B1DCDAF)  # splitmix64(0) first output


def test_bf16_rounding_helpers():
    x = np.array([1.0, 1.00390625, 1.005859375, -2.5, 3.0e-40], np.float32)
    b = synth.f32_to_bf16_bits(x)
    back = synth.bf16_bits_to_f32(b)
    assert back[0] == 1.0 and back[3] == -2.5
    assert back[1] == 1.0  # tie -> even
    assert synth.f64_to_bf16_bits(np.array([1.00390625]))[0] == synth.f32_to_bf16_bits(np.array([1.0], np.float32))[0]


def test_interleave_rows_follows_installer_order():
    g = np.arange(6).reshape(3, 2)
    u = 100 + np.arange(6).reshape(3, 2)
    gu = synth.interleave_rows(g, u)
    assert np.array_equal(gu[0], g[0]) and np.array_equal(gu[1], u[0]) and np.array_equal(gu[4], g[2])


def test_make_expert_stride_fills_the_layout():
    rng = np.random.default_rng(0)
    for spec in (GPT_OSS_20B.with_(hidden=64, intermediate=96), QWEN3_30B_A3B.with_(hidden=64, intermediate=32)):
        buf = synth.make_expert_stride(spec, rng)
        lay = spec.layout()
        assert buf.size == lay.stride
        sc = buf[lay.offsets["gate_up_scales"]:lay.offsets["gate_up_scales"] + lay.sizes["gate_up_scales"]]
        assert sc.min() >= 118 and sc.max() <= 124
        bias = buf[lay.offsets["down_bias"]:lay.offsets["down_bias"] + lay.sizes["down_bias"]]
        assert bool(np.any(bias)) == spec.expert_bias


def test_bindings_match_header_argument_counts():
    """Every ctypes signature has as many arguments as its declaration."""
    text = open(HEADER).read()
    for m in re.finditer(r"^GW_API\s+[\w\s\*]+?\b(gw_\w+)\s*\(([^;]*?)\)\s*;", text, flags=re.M | re.S):
        name, params = m.group(1), " ".join(m.group(2).split())
        n = 0 if params in ("", "void") else params.count(",") + 1
        assert len(_abi.SIGNATURES[name][1]) == n, (name, n, len(_abi.SIGNATURES[name][1]))
