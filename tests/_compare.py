"""Comparison helpers for the GPU-vs-oracle parity tests."""

import numpy as np
import torch


def as_np(x):
    if isinstance(x, torch.Tensor):
        return x.detach().cpu().numpy()
    return np.asarray(x)


def mismatch(actual, expected, rtol, atol):
    a = as_np(actual).astype(np.float64)
    e = as_np(expected).astype(np.float64)
    assert a.shape == e.shape, (a.shape, e.shape)
    bad = ~(np.abs(a - e) <= atol + rtol * np.abs(e))
    bad |= np.isnan(a) != np.isnan(e)
    return bad


def assert_close(actual, expected, rtol, atol, max_bad_frac=0.0, name=""):
    """Elementwise |a - e| <= atol + rtol |e| for all but ``max_bad_frac`` of the
    elements (the same criterion as torch.testing.assert_close)."""
    bad = mismatch(actual, expected, rtol, atol)
    frac = bad.mean() if bad.size else 0.0
    if frac > max_bad_frac:
        a = as_np(actual).astype(np.float64)
        e = as_np(expected).astype(np.float64)
        err = np.abs(a - e)
        i = np.unravel_index(np.argmax(err - rtol * np.abs(e)), err.shape)
        raise AssertionError(
            f"{name}: {bad.sum()} / {bad.size} elements ({frac:.2e}) outside rtol={rtol} "
            f"atol={atol}; worst at {i}: actual={a[i]!r} expected={e[i]!r}")


def assert_equal(actual, expected, name=""):
    a = as_np(actual)
    e = as_np(expected)
    assert a.shape == e.shape, (name, a.shape, e.shape)
    if not np.array_equal(a, e):
        bad = np.argwhere(a != e)
        raise AssertionError(f"{name}: {len(bad)} / {a.size} differ; first at {bad[0]}: "
                             f"{a[tuple(bad[0])]} vs {e[tuple(bad[0])]}")
