"""The .gwt installation reader: manifest checks on CPU, the bank it loads
against the oracle on the GPU."""
import json

import numpy as np
import oracle as O
import pytest

from godwit_b200 import gwt, synth
from godwit_b200.layout import GPT_OSS_20B, QWEN3_30B_A3B

SPEC = GPT_OSS_20B.with_(experts=6, layers=2, hidden=256, intermediate=128)


def make_install(root, spec=SPEC, seed=5):
    rng = np.random.default_rng(seed)
    strides = [np.stack([synth.make_expert_stride(spec, rng) for _ in range(spec.experts)])
               for _ in range(spec.layers)]
    routers = [synth.make_router(spec, rng) for _ in range(spec.layers)]
    gwt.write_install(str(root), spec, strides, routers)
    return strides, routers


def test_manifest_round_trip(tmp_path):
    make_install(tmp_path)
    m = gwt.read_manifest(str(tmp_path))
    gwt.validate(str(tmp_path), m)
    s = gwt.spec_of(m)
    assert (s.hidden, s.intermediate, s.experts, s.layers, s.top_k) == (256, 128, 6, 2, 4)
    assert s.activation == SPEC.activation and s.router_bias


def test_qwen_spec_from_manifest(tmp_path):
    spec = QWEN3_30B_A3B.with_(experts=4, layers=1, hidden=128, intermediate=64)
    make_install(tmp_path, spec)
    s = gwt.spec_of(gwt.read_manifest(str(tmp_path)))
    assert s.top_k == 8 and not s.router_bias and s.activation == spec.activation


def test_incomplete_install_is_rejected(tmp_path):
    with pytest.raises(gwt.InstallError, match="manifest"):
        gwt.read_manifest(str(tmp_path))
    make_install(tmp_path)
    p = gwt.layer_path(str(tmp_path), 1)
    with open(p, "r+b") as f:
        f.truncate(100)
    with pytest.raises(gwt.InstallError, match="layer 1"):
        gwt.validate(str(tmp_path), gwt.read_manifest(str(tmp_path)))


def test_wrong_format_version_is_rejected(tmp_path):
    make_install(tmp_path)
    mp = tmp_path / "manifest.json"
    m = json.loads(mp.read_text())
    m["formatVersion"] = 1
    mp.write_text(json.dumps(m))
    with pytest.raises(gwt.InstallError, match="format"):
        gwt.read_manifest(str(tmp_path))


@pytest.mark.gpu
def test_loaded_bank_matches_oracle(ctx, tmp_path):
    from godwit_b200.runtime import MoEBlock
    strides, routers = make_install(tmp_path)
    bank, spec = gwt.load_bank(ctx, str(tmp_path))
    try:
        assert np.array_equal(bank.download_expert(1, 3), strides[1][3])
        rng = np.random.default_rng(1)
        xb = synth.make_hidden(rng, 7, spec.hidden, "bf16")
        out, ex, wt = MoEBlock(ctx, bank).forward(xb, 1, "bf16")
        x = synth.as_f32(xb, "bf16")
        _, ref_ex, _ = O.moe_layer(spec, strides[1], routers[1][0], routers[1][1], x)
        assert (ex == ref_ex).mean() > 0.9
        assert O.rel_l2(out, O.moe_layer64(spec, strides[1], x, ex, wt)) < 1e-3
    finally:
        bank.close()


def test_streamed_strides_are_the_install_bytes(tmp_path):
    """The read-ahead loader yields every owned expert's stride in order, byte
    for byte, through two alternating buffers."""
    from godwit_b200 import gwt
    spec = GPT_OSS_20B.with_(hidden=64, intermediate=32, experts=5, layers=2)
    rng = np.random.default_rng(2)
    strides = [np.stack([synth.make_expert_stride(spec, rng) for _ in range(spec.experts)])
               for _ in range(spec.layers)]
    routers = [synth.make_router(spec, rng) for _ in range(spec.layers)]
    gwt.write_install(str(tmp_path), spec, strides, routers)
    m = gwt.read_manifest(str(tmp_path))
    stride = int(m["expertStride"])
    bufs = [np.empty(stride, np.uint8) for _ in range(2)]
    for layer in range(spec.layers):
        got = [(e, b.copy()) for e, b in gwt.stream_strides(str(tmp_path), layer, [1, 3, 4], stride, bufs)]
        assert [e for e, _ in got] == [1, 3, 4]
        for e, b in got:
            assert np.array_equal(b, strides[layer][e])


def test_streamed_read_past_the_file_is_an_install_error(tmp_path):
    from godwit_b200 import gwt
    spec = GPT_OSS_20B.with_(hidden=64, intermediate=32, experts=2, layers=1)
    rng = np.random.default_rng(3)
    strides = [np.stack([synth.make_expert_stride(spec, rng) for _ in range(spec.experts)])]
    gwt.write_install(str(tmp_path), spec, strides, [synth.make_router(spec, rng)])
    stride = int(gwt.read_manifest(str(tmp_path))["expertStride"])
    bufs = [np.empty(stride, np.uint8) for _ in range(2)]
    with pytest.raises(gwt.InstallError):
        list(gwt.stream_strides(str(tmp_path), 0, [0, 5], stride, bufs))


@pytest.mark.timeout(60)
def test_layer_file_that_cannot_be_opened_is_an_install_error(tmp_path):
    """A layer file that disappears (or cannot be opened) after the manifest
    check ends the read-ahead thread with an InstallError the consumer sees,
    instead of leaving the consumer waiting for a stride forever."""
    import os
    from godwit_b200 import gwt
    spec = GPT_OSS_20B.with_(hidden=64, intermediate=32, experts=2, layers=1)
    rng = np.random.default_rng(4)
    strides = [np.stack([synth.make_expert_stride(spec, rng) for _ in range(spec.experts)])]
    gwt.write_install(str(tmp_path), spec, strides, [synth.make_router(spec, rng)])
    stride = int(gwt.read_manifest(str(tmp_path))["expertStride"])
    os.remove(gwt.layer_path(str(tmp_path), 0))
    bufs = [np.empty(stride, np.uint8) for _ in range(2)]
    with pytest.raises(gwt.InstallError):
        list(gwt.stream_strides(str(tmp_path), 0, [0, 1], stride, bufs))
