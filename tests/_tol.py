"""Parity tolerances shared by the GPU tests (values from the north star of
this backend): fp32 elementwise/row ops rel 1e-5 / abs 1e-6 against the
oracle; dot |g - r| <= sqrt(K) * (1e-6 + 1e-5 |r|); long fp32 sums against an
fp64 sum, |g - s64| <= 1e-5 * sum|x| (the oracle's own sequential fp32 sum
is not a tighter reference than that)."""
import numpy as np

REL, ABS = 1e-5, 1e-6


def assert_close(got, ref, rel=REL, abs_=ABS, what=""):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    assert got.shape == ref.shape, f"{what}: shape {got.shape} vs {ref.shape}"
    err = np.abs(got - ref)
    lim = abs_ + rel * np.abs(ref)
    bad = err > lim
    if bad.any():
        i = np.argmax(err - lim)
        raise AssertionError(f"{what}: {bad.sum()} of {bad.size} outside rel {rel}/abs {abs_}; "
                             f"worst at {np.unravel_index(i, err.shape)}: got {got.ravel()[i]!r} ref {ref.ravel()[i]!r}")


def assert_dot_close(got, ref, K, what=""):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    lim = np.sqrt(K) * (1e-6 + 1e-5 * np.abs(ref))
    err = np.abs(got - ref)
    bad = err > lim
    if bad.any():
        i = np.argmax(err - lim)
        raise AssertionError(f"{what}: {bad.sum()} of {bad.size} outside sqrt(K)-scaled tolerance; worst "
                             f"got {got.ravel()[i]!r} ref {ref.ravel()[i]!r} (K={K})")


def assert_sum_close(got, x, what=""):
    x64 = np.asarray(x, np.float64)
    s64 = x64.sum()
    lim = 1e-5 * np.abs(x64).sum() + 1e-6
    assert abs(float(got) - s64) <= lim, f"{what}: {float(got)!r} vs fp64 {s64!r} (limit {lim})"
