"""The arithmetic facts the prefill matmul's bit-exactness rests on (gemm.cu), checked on the host.

The int4 operand tiles hold 16 * v: a two's complement nibble moved into the high half of its byte is the int8
16 * v. The MMA's group sums are then 16 * isum, and the epilogue forms fl(isum * ws) as one fma on a biased
integer: v = 12582912 + 16 * isum (exact in fp32 while |16 * isum| < 2^22), fma(v, ws / 16, -12582912 * ws / 16),
whose exact value is isum * ws, so the fma rounds it once. The reference computes fl((float)isum * ws)
(qwen.c:436-456), and (float)isum is exact for these sums.
"""
import numpy as np

BIAS = 12582912.0  # 1.5 * 2^23: the fp32 numbers in [2^23, 2^24) are the integers


def _nibble(x):
    """Two's complement value of a 4-bit field."""
    return x - 16 if x >= 8 else x


def test_high_half_nibble_is_sixteen_v():
    for b in range(256):
        lo, hi = _nibble(b & 15), _nibble(b >> 4)
        assert np.int8(np.uint8((b << 4) & 0xF0)) == 16 * lo
        assert np.int8(np.uint8(b & 0xF0)) == 16 * hi


def test_sixteen_isum_inside_the_exact_range():
    # a group: 32 products of int4 weights (-8 .. 7) and int8 activations (-128 .. 127 at the extremes)
    extreme = 32 * 8 * 128
    assert 16 * extreme < 2**22
    for s in (-extreme, -1, 0, 1, extreme):
        v = np.float32(BIAS + 16 * s)
        assert float(v) == BIAS + 16 * s  # representable: the biased integer is exact


def test_fma_with_a_sixteenth_of_the_scale_rounds_isum_times_ws_once():
    rng = np.random.default_rng(7)
    extreme = 32 * 8 * 128
    isums = np.concatenate([rng.integers(-extreme, extreme + 1, 20000), [-extreme, extreme, 0, 1, -1]])
    # every finite fp16 scale, positive and negative, subnormals included
    halves = np.arange(0, 0x7C00, dtype=np.uint16)
    ws_all = np.concatenate([halves.view(np.float16), -halves.view(np.float16)]).astype(np.float32)
    ws = ws_all[rng.integers(0, ws_all.size, isums.size)]
    w16 = (ws.astype(np.float64) / 16.0).astype(np.float32)
    assert np.array_equal(w16.astype(np.float64), ws.astype(np.float64) / 16.0)  # ws / 16 is exact
    ncw = (np.float32(-BIAS) * w16).astype(np.float32)
    assert np.array_equal(ncw.astype(np.float64), -BIAS * w16.astype(np.float64))  # -12582912 * ws / 16 is exact
    v = (BIAS + 16.0 * isums).astype(np.float32)
    # the fma's exact value (every term is exact in double: 24-bit and 11-bit significands), rounded once to fp32
    exact = v.astype(np.float64) * w16.astype(np.float64) + ncw.astype(np.float64)
    assert np.array_equal(exact, isums.astype(np.float64) * ws.astype(np.float64))
    fma = exact.astype(np.float32)
    ref = (isums.astype(np.float32) * ws).astype(np.float32)  # the reference's fl((float)isum * ws)
    assert np.array_equal(fma.view(np.uint32), ref.view(np.uint32))
