"""Comparison helpers for the GPU-vs-oracle parity tests.

Every ``assert_close`` records the observed error of its comparison: the largest
absolute error, the largest error relative to the expected value, the largest
error relative to the largest expected magnitude, and the fraction of elements
outside the 1e-4 relative / 1e-5 absolute bar. With ``GSB_PARITY_LOG`` set to a
file path, one JSON line per comparison is appended there (test id included),
so a test run doubles as a report of the observed parity.
"""

import json
import os

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


def observed_error(actual, expected):
    """Observed error of ``actual`` against ``expected`` (both any array-like)."""
    a = as_np(actual).astype(np.float64)
    e = as_np(expected).astype(np.float64)
    if a.size == 0:
        return dict(n=0, max_abs=0.0, max_rel=0.0, max_scaled=0.0, frac_bar=0.0)
    err = np.abs(a - e)
    err = np.where(np.isnan(a) & np.isnan(e), 0.0, err)
    scale = float(np.nanmax(np.abs(e))) if np.isfinite(e).any() else 0.0
    nz = np.abs(e) > 0
    bar = ~(err <= 1e-5 + 1e-4 * np.abs(e))
    return dict(n=int(a.size), max_abs=float(np.nanmax(err)),
                max_rel=float(np.nanmax(err[nz] / np.abs(e[nz]))) if nz.any() else 0.0,
                max_scaled=float(np.nanmax(err) / scale) if scale > 0 else 0.0,
                frac_bar=float(bar.mean()), n_bar=int(bar.sum()))


def _log(name, rtol, atol, max_bad_frac, obs):
    path = os.environ.get("GSB_PARITY_LOG")
    if not path:
        return
    rec = dict(test=os.environ.get("PYTEST_CURRENT_TEST", "").split(" ")[0], name=name,
               rtol=float(rtol), atol=float(atol), max_bad_frac=float(max_bad_frac), **obs)
    with open(path, "a") as f:
        f.write(json.dumps(rec) + "\n")


def assert_close(actual, expected, rtol, atol, max_bad_frac=0.0, name=""):
    """Elementwise |a - e| <= atol + rtol |e| for all but ``max_bad_frac`` of the
    elements (the same criterion as torch.testing.assert_close)."""
    bad = mismatch(actual, expected, rtol, atol)
    frac = bad.mean() if bad.size else 0.0
    _log(name, rtol, atol, max_bad_frac, observed_error(actual, expected))
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


def assert_parity(actual, expected, name="", max_bad_frac=0.0, max_scaled=None):
    """The parity bar: every element within 1e-4 relative / 1e-5 absolute of the
    expected value, except at most ``max_bad_frac`` of them, and (when given) the
    largest error within ``max_scaled`` times the largest expected magnitude."""
    assert_close(actual, expected, 1e-4, 1e-5, max_bad_frac=max_bad_frac, name=name)
    if max_scaled is not None:
        obs = observed_error(actual, expected)
        assert obs["max_scaled"] <= max_scaled, (
            f"{name}: largest error {obs['max_abs']:.3e} is {obs['max_scaled']:.3e} of the largest "
            f"magnitude (bound {max_scaled:.1e})")
