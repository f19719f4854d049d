"""The exactness the int4 M >= 129 layout relies on, checked on the CPU.

The convert warps write w_hi = fp16(q * s) (an fp16 multiply) and
w_lo = fp16(q * s - w_hi) (an fp16 FMA, exact), scale w_lo by 2^8 in fp16 and
keep the high byte of its bit pattern as an E5M2 value. That is lossless when
2^8 w_lo has at most 3 significant bits and is a normal fp16: q * s has at most
14 (11 of s, 3 of |q| <= 8), w_hi keeps 11. Checked here for every q in
[-8, 7] and every fp16 scale in the BASELINE range [0.001, 0.02]."""
import numpy as np


def _fp16_scales(lo: float, hi: float) -> np.ndarray:
    a = np.frombuffer(np.float16(lo).tobytes(), np.uint16)[0]
    b = np.frombuffer(np.float16(hi).tobytes(), np.uint16)[0]
    return np.arange(a, b + 1, dtype=np.uint16).view(np.float16)


def _e5m2_high_byte(x16: np.ndarray) -> np.ndarray:
    """Keep the high byte of each fp16 bit pattern (the E5M2 value), back as fp16."""
    return (x16.view(np.uint16) & np.uint16(0xFF00)).view(np.float16)


def test_remainder_of_fp16_product_is_exact_in_e5m2():
    s = _fp16_scales(0.001, 0.02)
    assert s.size == 4359  # every fp16 value in [0.001, 0.02]
    q = np.arange(-8, 8, dtype=np.float16)
    exact = q.astype(np.float64)[:, None] * s.astype(np.float64)[None, :]
    w_hi = (q[:, None] * s[None, :]).astype(np.float16)  # fp16 multiply, round to nearest
    rem = exact - w_hi.astype(np.float64)
    w_lo = rem.astype(np.float16)
    assert np.array_equal(w_lo.astype(np.float64), rem)  # the fp16 FMA's result is exact
    lo256 = (w_lo.astype(np.float64) * 256).astype(np.float16)
    assert np.array_equal(lo256.astype(np.float64), rem * 256)
    nz = lo256 != 0
    assert np.all(np.abs(lo256[nz].astype(np.float64)) >= 2.0 ** -14)  # normal fp16 (and E5M2)
    e5 = _e5m2_high_byte(lo256)
    assert np.array_equal(e5, lo256)                     # the dropped low byte is zero
    # and the pair carries the product exactly
    recon = w_hi.astype(np.float64) + e5.astype(np.float64) / 256
    assert np.array_equal(recon, exact)


def test_fp16_product_alone_loses_bits():
    # Without the remainder term a sizeable share of the products is rounded.
    s = _fp16_scales(0.001, 0.02)
    q = np.arange(-8, 8, dtype=np.float16)
    exact = q.astype(np.float64)[:, None] * s.astype(np.float64)[None, :]
    w_hi = (q[:, None] * s[None, :]).astype(np.float16).astype(np.float64)
    assert np.mean(w_hi != exact) > 0.3
