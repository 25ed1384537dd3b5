"""The decode kernels' activation encoding (no GPU), restated in numpy with the float32
operations the kernels issue (csrc/gemv.cu m1_digits_chunk, digit4f, residual_digit;
csrc/q4asym.cu takes the same steps inline, with the exponent clamped at 14 instead of 18
because its factor 2^(E - 140) carries no 16 for 16 q weights).

Per 32-block with E the biased exponent of its largest magnitude (at least 18) and
up = 2^(140 - E):
  * X = rint(x * up) from the float sum x * up + 1.5 * 2^23 (the product is exact, the sum
    rounds once, to nearest even), whose low bits hold X;
  * the digits X = 256 h + sext8(X): byte 0 of that sum is the low digit, byte 1 of the same
    sum with 128 more is h;
  * for fp32 rows a second image X2 = rint(R * 2^15) of the remainder R = x * up - X, which
    is exact in float32 and at most 1/2 in magnitude.

These pin what the s8 MMAs rely on (every digit fits a signed byte, X and X2 fit 2^14) and the
bounds the GPU tests check: one image keeps every element within 2^-14 of its block's largest
magnitude, two images within 2^-29.  A block whose largest magnitude is below 2^-109 is encoded
with the clamped exponent (its factor must stay a normal float), so its bound is absolute:
2^-123 with one image, 2^-138 with two.
"""
import numpy as np
import pytest

MAGIC = np.float32(12582912.0)        # 1.5 * 2^23: an exponent whose ulp is 1
MAGIC_HI = np.float32(12583040.0)     # ... + 128, the high digit's rounding offset
BASE = 0x4B400000                     # the bits of MAGIC


def block_up(xb):
    """2^(140 - E) for one block (float32), E clamped to 18 as the kernels do."""
    e = int((xb.view(np.uint32) & 0x7FFFFFFF).max() >> 23)
    e = max(e, 18)
    return np.array((267 - e) << 23, np.uint32).view(np.float32)[()]


def encode(xb, up):
    """One image of a float32 block: X, its two digits, and the float32 remainder R."""
    xs = xb * up                                     # exact: up is a power of two
    r = (xs + MAGIC).astype(np.float32)              # one rounding
    h = (xs + MAGIC_HI).astype(np.float32)
    X = r.view(np.uint32).astype(np.int64) - BASE
    lo = (r.view(np.uint32) & 0xFF).astype(np.uint8).view(np.int8).astype(np.int64)
    hi = ((h.view(np.uint32) >> 8) & 0xFF).astype(np.uint8).view(np.int8).astype(np.int64)
    rem = (xs - (r - MAGIC)).astype(np.float32)      # x * up - X, the kernels' FMA
    return X, lo, hi, rem


def images(x):
    """Both images of a float32 row, per 32-block: (X, X2, up) as arrays of the row's shape."""
    x = np.ascontiguousarray(x, np.float32).reshape(-1, 32)
    X = np.zeros(x.shape, np.int64)
    X2 = np.zeros(x.shape, np.int64)
    ups = np.zeros(x.shape[0], np.float64)
    for b, xb in enumerate(x):
        up = block_up(xb)
        X[b], lo, hi, rem = encode(xb, up)
        assert (X[b] == 256 * hi + lo).all()                   # the digit split
        assert np.abs(hi).max() <= 64 and np.abs(X[b]).max() <= 1 << 14
        # the remainder is exact in float32 and at most 1/2
        exact = xb.astype(np.float64) * float(up) - X[b]
        assert (rem.astype(np.float64) == exact).all()
        assert np.abs(exact).max() <= 0.5
        X2[b], lo2, hi2, _ = encode(rem, np.float32(32768.0))
        assert (X2[b] == 256 * hi2 + lo2).all()
        assert np.abs(hi2).max() <= 64 and np.abs(X2[b]).max() <= 1 << 14
        ups[b] = float(up)
    return X, X2, ups


def _rows():
    rng = np.random.default_rng(7)
    k = 32 * 64
    normal = rng.normal(0, 1, k).astype(np.float32)
    wide = (rng.choice([-1.0, 1.0], k) * np.exp2(rng.uniform(-30, 18, k))).astype(np.float32)
    wide[rng.random(k) < 0.1] = 0.0
    wide[64:96] = 0.0                                 # an all-zero block
    wide[160:192] = 1e-7
    wide[170] = -5e4                                  # one outlier over tiny values
    wide[224:256] = 1e-35                             # tiny values (below 2^-109: clamped exponent)
    wide[256:288] = np.float32(1e-40)                 # subnormal values
    wide[288:320] = -2.0                              # equal values
    return {"normal": normal, "dynamic range": wide}


@pytest.mark.parametrize("name", ["normal", "dynamic range"])
def test_two_images_hold_fp32_rows_to_2e_minus_29_of_the_block(name):
    x = _rows()[name]
    X, X2, ups = images(x)
    xb = x.reshape(-1, 32).astype(np.float64)
    blk_max = np.abs(xb).max(axis=1, keepdims=True)
    one = X / ups[:, None]
    two = (X + X2 * 2.0 ** -15) / ups[:, None]
    assert (np.abs(xb - one) <= np.maximum(2.0 ** -14 * blk_max, 2.0 ** -123)).all()
    assert (np.abs(xb - two) <= np.maximum(2.0 ** -29 * blk_max, 2.0 ** -138)).all()
    # the relative bounds hold for every block at or above 2^-109
    ok = blk_max[:, 0] >= 2.0 ** -109
    assert (np.abs(xb - one)[ok] <= 2.0 ** -14 * blk_max[ok]).all()
    assert (np.abs(xb - two)[ok] <= 2.0 ** -29 * blk_max[ok]).all()


def test_bf16_values_within_seven_binades_are_exact_in_one_image():
    rng = np.random.default_rng(3)
    x = rng.normal(0, 1, 32 * 32).astype(np.float32)
    x = (x.view(np.uint32) & 0xFFFF0000).view(np.float32)      # bf16 values
    X, X2, ups = images(x)
    xb = x.reshape(-1, 32).astype(np.float64)
    blk_max = np.abs(xb).max(axis=1, keepdims=True)
    near = np.abs(xb) >= blk_max * 2.0 ** -6                     # the block's top 7 binades
    assert (X2[near] == 0).all()
    assert (X[near] / np.broadcast_to(ups[:, None], X.shape)[near] == xb[near]).all()
