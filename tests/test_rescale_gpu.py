"""The prefill fold's running-maximum rescale against the contract's, bit for bit.

The contract rescales a binary32 value by 2^-D by subtracting D from its exponent field and
flushing to +0 when the field would drop below 1 (zero and subnormal inputs flush too;
reference/lssab8_golden.py:293-301).  The kernel does it with one paired multiply by 2^-D
rounded toward zero with flush-to-zero for D <= 126, and with a compare-and-select above;
lssab8_selftest_rescale runs that exact device code followed by the fold's add of a zero term
(which turns a flushed -0 into +0, as the fold's real term does).
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

DS = [0, 1, 2, 5, 23, 64, 100, 125, 126, 127, 128, 150, 200, 252, 253, 254, 255, 1000]


def _contract(x, d):
    u = x.view(np.uint32).astype(np.int64)
    e = (u >> 23) & 0xFF
    ne = e - d
    keep = (e >= 1) & (ne >= 1)
    out = np.where(keep, (u & 0x807FFFFF) | (np.maximum(ne, 0) << 23), 0).astype(np.uint32)
    return np.where(d <= 0, x.view(np.uint32), out)


def _device(x, d):
    from lockstep_b200 import _lib
    dev = torch.device("cuda:0")
    tx = torch.from_numpy(x).to(dev)
    td = torch.from_numpy(d).to(dev)
    out = torch.empty_like(tx)
    with torch.cuda.device(dev):
        _lib.check(_lib.load().lssab8_selftest_rescale(tx.data_ptr(), td.data_ptr(), d.size, out.data_ptr(),
                                                       torch.cuda.current_stream(dev).cuda_stream),
                   "lssab8_selftest_rescale")
    torch.cuda.synchronize(dev)
    return out.cpu().numpy()


def _check(x, dpair):
    x = np.ascontiguousarray(x, dtype=np.float32)
    dpair = np.ascontiguousarray(dpair, dtype=np.int32)
    assert x.size == 2 * dpair.size
    # the contract's rescale, then the same add of a zero term (-0 + 0 == +0; all else unchanged)
    want = (_contract(x, np.repeat(dpair.astype(np.int64), 2)).view(np.float32) + np.float32(0.0)).view(np.uint32)
    got = _device(x, dpair).view(np.uint32)
    bad = np.nonzero(got != want)[0]
    assert bad.size == 0, "first mismatches (x, D, got, want): %s" % [
        (float(x[i]), int(dpair[i // 2]), hex(int(got[i])), hex(int(want[i]))) for i in bad[:5]]


def _boundary_values(d, rng):
    """Every exponent field near the flush boundary for D, extreme significands, both signs."""
    exps = sorted({0, 1, 2, 253, 254} | {e for e in (d - 2, d - 1, d, d + 1, d + 2) if 0 <= e <= 254})
    sig = np.concatenate([np.array([0, 1, 2, (1 << 23) - 2, (1 << 23) - 1, 1 << 22], dtype=np.uint32),
                          rng.integers(0, 1 << 23, 4096, dtype=np.uint32)])
    u = (np.array(exps, dtype=np.uint32)[:, None] << 23) | sig[None, :]
    u = np.concatenate([u.ravel(), u.ravel() | np.uint32(0x80000000)])
    return u.view(np.float32)


def test_rescale_boundaries():
    rng = np.random.default_rng(21)
    xs, ds = [], []
    for d in DS:
        x = _boundary_values(d, rng)
        if x.size % 2:
            x = np.append(x, np.float32(1.0))
        xs.append(x)
        ds.append(np.full(x.size // 2, d, dtype=np.int32))
    _check(np.concatenate(xs), np.concatenate(ds))


def test_rescale_random_finite():
    rng = np.random.default_rng(22)
    n = 1 << 22
    u = rng.integers(0, 1 << 32, n, dtype=np.uint64).astype(np.uint32)
    u = np.where((u & 0x7F800000) == 0x7F800000, u & 0xBFFFFFFF, u)    # finite values only
    d = rng.choice(np.array(DS + list(range(1, 40)), dtype=np.int32), n // 2)
    _check(u.view(np.float32), d)


def test_rescale_fold_magnitudes():
    # the values the fold actually rescales: O of a few hundred to a few million units of 2^-e_v,
    # by the small D that successive block maxima produce
    rng = np.random.default_rng(23)
    n = 1 << 22
    x = (rng.standard_normal(n) * np.exp2(rng.integers(-150, 60, n))).astype(np.float32)
    d = rng.integers(1, 40, n // 2).astype(np.int32)
    _check(x, d)
