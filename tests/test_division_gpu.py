"""The prefill epilogue's division against IEEE binary32 division, bit for bit.

The contract's last step is one RN division per output element, fl(O_row / l_row)
(reference/lssab8_golden.py:333, reference/lssab8_torch.py:266-271).  The kernel computes it
from the row's correctly rounded reciprocal with Markstein's correction and falls back to the
IEEE division outside a safe exponent window; lssab8_selftest_div runs that exact device code.
numpy's float32 division is IEEE round-to-nearest-even, so it is the reference here.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def _device_div(y, l):
    from lockstep_b200 import _lib
    dev = torch.device("cuda:0")
    ty = torch.from_numpy(y).to(dev)
    tl = torch.from_numpy(l).to(dev)
    out = torch.empty_like(ty)
    with torch.cuda.device(dev):
        _lib.check(_lib.load().lssab8_selftest_div(ty.data_ptr(), tl.data_ptr(), ty.numel(), out.data_ptr(),
                                                   torch.cuda.current_stream(dev).cuda_stream), "lssab8_selftest_div")
    torch.cuda.synchronize(dev)
    return out.cpu().numpy()


def _check(y, l):
    y = np.ascontiguousarray(y, dtype=np.float32)
    l = np.ascontiguousarray(l, dtype=np.float32)
    with np.errstate(all="ignore"):
        want = y / l
    got = _device_div(y, l)
    bad = np.nonzero(got.view(np.uint32) != want.view(np.uint32))[0]
    assert bad.size == 0, "first mismatches: %s" % [(float(y[i]), float(l[i]), float(got[i]), float(want[i]))
                                                     for i in bad[:5]]


def test_division_realistic_ranges():
    rng = np.random.default_rng(11)
    n = 1 << 22
    l = rng.uniform(1.0, 2.0 ** 21, n).astype(np.float32)               # l_row: sums of 8-bit weights
    y = (rng.standard_normal(n) * np.exp2(rng.integers(-40, 41, n))).astype(np.float32)
    _check(y, l)


def test_division_near_midpoints():
    # y / l within a few units of 2^-40 ulp of a rounding midpoint: the hard cases for any
    # division that is not correctly rounded
    rng = np.random.default_rng(12)
    n = 1 << 22
    l = (rng.integers(1 << 23, 1 << 24, n) * np.exp2(rng.integers(-23, 8, n))).astype(np.float32)
    mant = rng.integers(1 << 23, 1 << 24, n).astype(np.float64) + 0.5      # a midpoint's significand
    qmid = mant * np.exp2(rng.integers(-40, 0, n))
    y = (qmid * l.astype(np.float64)).astype(np.float32)
    _check(y, l)


def test_division_all_significands_of_l():
    # every significand of l in one binade against random numerators, and the numerators'
    # neighbours in ulps
    rng = np.random.default_rng(13)
    l = (np.arange(1 << 23, 1 << 24, dtype=np.float64) * 2.0 ** -23).astype(np.float32)
    y = rng.uniform(1.0, 2.0, l.size).astype(np.float32)
    _check(y, l)
    _check(np.nextafter(y, np.float32(3.0)), l)
    _check(np.nextafter(y, np.float32(0.0)) * np.float32(2.0 ** 20), l * np.float32(2.0 ** -5))


def test_division_edges():
    f = np.float32
    tiny, huge = np.finfo(np.float32).tiny, np.finfo(np.float32).max
    sub = f(tiny) * f(0.25)
    ys = np.array([0.0, -0.0, sub, -sub, tiny, 1e-30, 2.0 ** -31, 2.0 ** -32, 2.0 ** 32, 2.0 ** 31 * 1.99,
                   1e30, huge, -huge, 1.0, -1.0, 3.0, 1.0 / 3.0], dtype=np.float32)
    ls = np.array([1.0, 3.0, 2.0 ** -31, 2.0 ** -32, 2.0 ** 32, 1e-30, 1e30, sub, tiny, huge, 7.0, 1.5,
                   2.0 ** 31 * 1.99, 255.0, 65025.0], dtype=np.float32)
    Y, Lg = np.meshgrid(ys, ls, indexing="ij")
    _check(Y.ravel(), Lg.ravel())
