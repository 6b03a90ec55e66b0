"""The requantiser's round-half-away-from-zero (C roundf) is computed as
trunc(y + copysign(0.5 - 2^-25, y)) in float32. This checks that identity on
every float in [0.25, 2) (where a wrong carry could occur), on the ties and
their neighbours up to 256 and on a random sample of the q8_0 range. (All
floats of magnitude below 256 were checked once the same way.)"""
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
