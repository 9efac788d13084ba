"""The trunk's int8 affine projections on the B200, through the C-ABI, against
the CPU restatements of int8_affine_gemv / int8_affine_gemv_bias_batched
(Sources/Godwit/Metal/MoE/router.metal:65-141).

Bar: fp32 outputs within rel-L2 1e-5 of the fp64 oracle (the products are
exact on the tensor cores; only the fp32 accumulation order differs) and
within 1e-5 relative of the fp32 restatement per value; f16 outputs within
half an f16 ulp of the fp64 result plus an fp32 accumulation allowance of
1e-5 of the largest output (values near zero come from cancelling group
terms, so their error is absolute, not relative: the reference's own fp32
restatement misses a bare one-ulp bar on such values).
"""
import numpy as np
import oracle as O
import pytest

from godwit_b200._abi import GW_E_ARG, GodwitCUDAError

pytestmark = pytest.mark.gpu


def synthetic(rng, rows, cols):
    """Codes uniform over 0..255, bf16 scales ~ 2e-4 (the step of a +-0.025
    weight range) and zero points ~ -0.025, as an installed trunk tensor holds."""
    codes = rng.integers(0, 256, (rows, cols), dtype=np.uint8)
    sc = (rng.uniform(1.0, 3.0, (rows, cols // 64)) * 1e-4).astype(np.float32)
    zr = (-sc * 127.5 * rng.uniform(0.8, 1.2, sc.shape)).astype(np.float32)
    meta = np.stack([_bf16(sc), _bf16(zr)], -1)
    return codes, meta


def _bf16(a):
    b = np.ascontiguousarray(a, np.float32).view(np.uint32)
    return ((b + (((b >> 16) & 1) + 0x7FFF)) >> 16).astype(np.uint16)


def hidden(rng, T, cols):
    return rng.standard_normal((T, cols)).astype(np.float16)


def check_f16(y, ref64):
    want = ref64.astype(np.float16)
    ulp = np.spacing(np.abs(want)).astype(np.float64)  # the larger ulp at a power of two
    err = np.abs(y.astype(np.float64) - ref64)
    assert np.all(err <= 0.5001 * ulp + 1e-5 * np.max(np.abs(ref64)))


def test_quantised_head_slice_matches_oracle(ctx):
    """A quantised (Int8Affine.quantize) head slice, one token, fp32 out: the
    shape of ModelRunner's output-head projection."""
    rng = np.random.default_rng(1)
    w = rng.normal(0, 0.02, (512, 2880)).astype(np.float32)
    codes, meta = O.int8_quantize(w)
    x = hidden(rng, 1, 2880)
    y = ctx.int8_affine_gemv(codes, meta, x)
    ref64 = O.int8_gemv64(codes, meta, x.astype(np.float32))
    ref32 = O.int8_gemv(codes, meta, x.astype(np.float32))
    assert O.rel_l2(y, ref64) < 1e-5
    assert np.max(np.abs(y - ref32)) <= 1e-5 * np.max(np.abs(ref32))


@pytest.mark.parametrize("rows,cols,T", [(1, 64, 1), (1000, 128, 1), (20, 448, 3), (4096, 2880, 1)])
def test_fp32_out_shapes(ctx, rows, cols, T):
    rng = np.random.default_rng(rows + cols + T)
    codes, meta = synthetic(rng, rows, cols)
    x = hidden(rng, T, cols)
    y = ctx.int8_affine_gemv(codes, meta, x)
    assert y.shape == (T, rows)
    assert O.rel_l2(y, O.int8_gemv64(codes, meta, x.astype(np.float32))) < 1e-5


@pytest.mark.parametrize("rows,cols,T", [(5120, 2880, 1), (5120, 2880, 5), (5120, 2880, 8), (5120, 2880, 13),
                                         (2880, 4096, 16), (640, 2880, 32), (640, 2880, 41), (272, 1024, 70)])
def test_bias_batched_f16_out(ctx, rows, cols, T):
    """int8_affine_gemv_bias_batched: attention q/k/v (5120 x 2880) and o
    (2880 x 4096) shapes, token counts across the 8/16/32-token passes."""
    rng = np.random.default_rng(3 * rows + T)
    codes, meta = synthetic(rng, rows, cols)
    bias = _bf16(rng.normal(0, 0.02, rows))
    x = hidden(rng, T, cols)
    y = ctx.int8_affine_gemv(codes, meta, x, bias=bias, out="f16")
    assert y.dtype == np.float16 and y.shape == (T, rows)
    check_f16(y, O.int8_gemv64(codes, meta, x.astype(np.float32), bias))


def test_device_pointer_entry_matches_host_entry(ctx):
    import torch
    from godwit_b200 import device as D

    rng = np.random.default_rng(11)
    rows, cols, T = 1536, 2880, 4
    codes, meta = synthetic(rng, rows, cols)
    bias = _bf16(rng.normal(0, 0.02, rows))
    x = hidden(rng, T, cols)
    host = ctx.int8_affine_gemv(codes, meta, x, bias=bias)
    D.bind_stream(ctx)
    try:
        dc = torch.from_numpy(codes).cuda()
        dm = torch.from_numpy(meta.view(np.int16)).cuda()
        db = torch.from_numpy(bias.view(np.int16)).cuda()
        dx = torch.from_numpy(x).cuda()
        y = torch.empty((T, rows), dtype=torch.float32, device="cuda")
        D.int8_affine_gemv(ctx, dc, dm, db, dx, y)
        y16 = torch.empty((T, rows), dtype=torch.float16, device="cuda")
        D.int8_affine_gemv(ctx, dc, dm, db, dx, y16)
        torch.cuda.synchronize()
        assert np.array_equal(y.cpu().numpy(), host)
        assert np.array_equal(y16.cpu().numpy(), host.astype(np.float16))
    finally:
        ctx.set_stream(None)


def test_rejects_bad_shapes_before_launch(ctx):
    codes = np.zeros((16, 96), np.uint8)
    meta = np.zeros((16, 1, 2), np.uint16)
    with pytest.raises(GodwitCUDAError) as e:
        ctx.int8_affine_gemv(codes, meta, np.zeros((1, 96), np.float16))
    assert e.value.status == GW_E_ARG and "multiple of 64" in str(e.value)
