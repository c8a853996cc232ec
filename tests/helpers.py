"""Shared test helpers (tolerances, seeded inputs)."""
import numpy as np


def rms(x):
    x = np.asarray(x, dtype=np.float64)
    return float(np.sqrt(np.mean(x * x))) if x.size else 0.0


def assert_close(got, ref, rtol, what="", atol_rms=None):
    """|got - ref| <= rtol * (|ref| + atol_rms * rms(ref)) elementwise.

    atol_rms defaults to 1: an error floor proportional to the data's scale, so
    elements that cancel to ~0 are judged against the magnitude of their
    inputs rather than their own (for which no relative bound is meaningful)."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    assert got.shape == ref.shape, f"{what}: shape {got.shape} vs {ref.shape}"
    assert np.isfinite(got).all(), f"{what}: non-finite values"
    floor = (1.0 if atol_rms is None else atol_rms) * rms(ref)
    err = np.abs(got - ref)
    bound = rtol * (np.abs(ref) + floor)
    bad = err > bound
    if bad.any():
        i = np.unravel_index(np.argmax(err / np.maximum(bound, 1e-300)), err.shape)
        raise AssertionError(f"{what}: {bad.sum()} / {bad.size} elements out of tolerance "
                             f"(rtol {rtol}); worst at {i}: got {got[i]!r} ref {ref[i]!r} "
                             f"max|err| {err.max():.3e}")
