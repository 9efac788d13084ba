"""The MXFP8 quantiser of the oracle (the block-scaled mode's activation
format): scale choice, rounding, saturation, zero blocks, and error bound."""
import numpy as np
import oracle as O


def test_known_blocks():
    x = np.zeros((3, 64), np.float32)
    x[0, :32] = 1.0                      # amax 1 = 2^0 -> X = -8, byte 119, codes 256 -> 0x78 (256 in E4M3)
    x[1, :32] = np.linspace(-3, 3, 32)   # amax 3 -> floor(log2 3) = 1 -> X = -7, byte 120
    x[2, 32:] = 0.0                      # zero block -> byte 0, codes 0
    codes, scales = O.quantize_mxfp8(x)
    assert scales[0, 0] == 119 and scales[1, 0] == 120 and scales[2, 1] == 0
    assert np.all(codes[0, :32] == 0x78)
    assert np.all(codes[2, 32:] == 0)
    back = O.dequantize_mxfp8(codes, scales)
    assert np.array_equal(back[0, :32], np.ones(32))


def test_saturation_and_error_bound():
    rng = np.random.default_rng(0)
    x = (rng.standard_normal((64, 256)) * np.exp2(rng.integers(-20, 20, (64, 1)))).astype(np.float32)
    x[0, 5] = 1.9999 * 2 ** 3  # block max just under a power of two: codes up to 511.9 -> 448 after saturation
    codes, scales = O.quantize_mxfp8(x)
    back = O.dequantize_mxfp8(codes, scales)
    blocks = np.abs(x).reshape(64, 8, 32).max(-1)
    err = np.abs(back - x).reshape(64, 8, 32).max(-1)
    # RN to 3 mantissa bits: |err| <= 2^-4 * (block max), saturation adds at most 12.5 %
    assert np.all(err <= blocks * 0.13)
    assert np.isfinite(back).all()
