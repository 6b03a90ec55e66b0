"""The requantiser's round-half-away-from-zero (C roundf) is computed as
trunc(y + copysign(0.5 - 2^-25, y)) in float32. This checks that identity on
every float in [0.25, 2) (where a wrong carry could occur), on the ties and
their neighbours up to 256 and on a random sample of the q8_0 range. (All
floats of magnitude below 256 were checked once the same way.)

The q8_0 scale amax / 127 uses a multiply and a fused multiply-add in place of
a division; the tests below check it against IEEE division on every float in
[1, 2) and in the binade at the cutoff 2^-100, and on a sample of every binade
above (all non-negative floats from 2^-100 up were checked once the same
way)."""
import numpy as np

C = np.float32(0.49999997)


def _round_away_formula(y):
    return np.trunc((y + np.copysign(C, y)).astype(np.float32))


def _round_away_exact(y):
    yd = y.astype(np.float64)
    return np.copysign(np.floor(np.abs(yd) + 0.5), yd)


def _check(y):
    y = np.concatenate([y, -y]).astype(np.float32)
    assert np.array_equal(_round_away_formula(y), _round_away_exact(y))


def test_constant_is_predecessor_of_half():
    assert C == np.nextafter(np.float32(0.5), np.float32(0))


def test_every_float_in_quarter_to_two():
    lo = int(np.float32(0.25).view(np.uint32))
    hi = int(np.float32(2.0).view(np.uint32))
    for start in range(lo, hi, 1 << 23):
        b = np.arange(start, min(start + (1 << 23), hi), dtype=np.uint32)
        _check(b.view(np.float32))


def test_ties_and_neighbours_up_to_256():
    k = np.arange(0, 256, dtype=np.float32) + np.float32(0.5)
    near = [k]
    x = k
    for _ in range(4):
        x_up = np.nextafter(x, np.float32(np.inf))
        x_dn = np.nextafter(x, np.float32(0))
        near += [x_up, x_dn]
        x = x_up
    _check(np.concatenate(near))


def test_random_sample_of_q8_range():
    rng = np.random.default_rng(0)
    _check(rng.uniform(-128, 128, 1 << 22).astype(np.float32))


# The q8_0 scale amax / 127 is computed on the device as RN(x zh + RN(x zl)),
# zh = RN(1/127), zl = RN(1/127 - zh) (division by a constant known in
# advance, Brisebarre, Muller and Raina 2004), for x >= 2^-100; below that the
# device divides. Products of two float32 values and the sum here are exact in
# float64, so each float32 cast is the single rounding of the device operation.
ZH = np.float32(float.fromhex("0x1.020408p-7"))
ZL = np.float32(float.fromhex("0x1.020408p-35"))


def _div127_formula(x):
    u = (x.astype(np.float64) * np.float64(ZL)).astype(np.float32)
    return (x.astype(np.float64) * np.float64(ZH) + u.astype(np.float64)).astype(np.float32)


def _check_div127(x):
    x = x.astype(np.float32)
    assert np.array_equal(_div127_formula(x).view(np.uint32),
                          (x / np.float32(127.0)).view(np.uint32))


def test_div127_constants():
    from fractions import Fraction
    inv = Fraction(1, 127)
    assert abs(Fraction(float(ZH)) - inv) <= abs(Fraction(float(np.nextafter(ZH, np.float32(1)))) - inv)
    assert abs(Fraction(float(ZH)) - inv) <= abs(Fraction(float(np.nextafter(ZH, np.float32(0)))) - inv)
    r = inv - Fraction(float(ZH))
    assert abs(Fraction(float(ZL)) - r) <= abs(Fraction(float(np.nextafter(ZL, np.float32(1)))) - r)
    assert abs(Fraction(float(ZL)) - r) <= abs(Fraction(float(np.nextafter(ZL, np.float32(0)))) - r)


def test_div127_every_float_in_one_to_two_and_near_the_cutoff():
    for lo_f, hi_f in ((1.0, 2.0), (2.0 ** -100, 2.0 ** -99)):
        lo = int(np.float32(lo_f).view(np.uint32))
        hi = int(np.float32(hi_f).view(np.uint32))
        _check_div127(np.arange(lo, hi, dtype=np.uint32).view(np.float32))


def test_div127_random_sample_of_every_binade():
    rng = np.random.default_rng(1)
    lo = int(np.float32(2.0 ** -100).view(np.uint32))
    hi = int(np.float32(np.finfo(np.float32).max).view(np.uint32))
    b = rng.integers(lo, hi, 1 << 23, dtype=np.uint64).astype(np.uint32)
    _check_div127(b.view(np.float32))
    _check_div127(np.array([np.inf, 0.0], dtype=np.float32))
