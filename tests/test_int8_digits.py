"""The integer digit form of a GEMV input that the int8 units multiply (host restatement).

The step kernel feeds int8 weights to `tcgen05.mma.kind::i8` with the input written, per 32-input
block, as q = rint(x * 2^(26 - E)) (E = the exponent of the block's largest |x|) split into four
int8 digits q = d0 * 2^21 + d1 * 2^14 + d2 * 2^7 + d3 (d0 signed in [-64, 63], d1..d3 in [0, 127]);
the tensor core's s32 sums of weights x digits are exact and the readout combines them as
2^14 (128 s0 + s1) + (128 s2 + s3). These tests pin the arithmetic claims the kernel relies on:
digit ranges (int8, no overflow of the s32 sums or of the pair combination), the exact
reconstruction of q, and the representation error bound of 2^-28 of the block's largest input.
"""
import numpy as np


def digits(x):
    """Restatement of digitize4_n for one 32-input block: (d[4, 32] int64, scale 2^(E - 26))."""
    x = np.asarray(x, dtype=np.float32)
    m = np.float32(np.abs(x).max())
    eb = max(int((m.view(np.uint32) >> 23) & 0xFF), 26)               # biased exponent, clamped
    mul = np.uint32((280 - eb) << 23).view(np.float32)                  # 2^(153 - eb)
    scale = float(np.uint32((eb - 26) << 23).view(np.float32))          # 2^(eb - 153)
    q = np.rint((x * mul).astype(np.float32)).astype(np.int64)
    d = np.stack([q >> 21, (q >> 14) & 127, (q >> 7) & 127, q & 127])
    return d, scale, q


def test_digit_ranges_and_exact_reconstruction():
    rng = np.random.default_rng(0)
    for trial in range(2000):
        mag = 10.0 ** rng.uniform(-30, 30)
        x = (rng.standard_normal(32) * np.exp(rng.standard_normal(32) * 3) * mag).astype(np.float32)
        d, scale, q = digits(x)
        assert np.all(np.abs(q) < 2 ** 27)
        assert d[0].min() >= -64 and d[0].max() <= 63
        assert d[1:].min() >= 0 and d[1:].max() <= 127
        assert np.array_equal(d[0] * 2 ** 21 + d[1] * 2 ** 14 + d[2] * 2 ** 7 + d[3], q)
        # representation error: at most half a unit of q, i.e. 2^-28 of the block's largest |x|
        err = np.abs(q * scale - x.astype(np.float64)).max()
        assert err <= 0.5 * scale * (1 + 1e-12)
        assert err <= 2.0 ** -27 * float(np.abs(x).max()) + 1e-300


def test_s32_sums_and_pair_combination_do_not_overflow():
    # worst case: 32 weights of |q| = 127 against extreme digits
    w = np.full(32, -127, dtype=np.int64)
    d = np.stack([np.full(32, -64), np.full(32, 127), np.full(32, 127), np.full(32, 127)])
    s = d @ w
    assert np.abs(s).max() < 2 ** 31
    hi = s[0] * 128 + s[1]
    lo = s[2] * 128 + s[3]
    assert abs(hi) < 2 ** 31 and abs(lo) < 2 ** 31


def test_block_dot_product_matches_fp64():
    rng = np.random.default_rng(1)
    for trial in range(200):
        x = (rng.standard_normal(32) * rng.uniform(0.01, 100)).astype(np.float32)
        wq = rng.integers(-127, 128, 32)
        ws = float(np.float16(abs(rng.normal(0, 0.02)) / 127))
        d, scale, _ = digits(x)
        s = d @ wq                                                       # the exact s32 sums
        combined = 16384.0 * float(s[0] * 128 + s[1]) + float(s[2] * 128 + s[3])
        got = ws * scale * combined
        want = ws * float(wq @ x.astype(np.float64))
        tol = ws * 32 * 127 * 2.0 ** -27 * float(np.abs(x).max())
        assert abs(got - want) <= tol + 1e-300
