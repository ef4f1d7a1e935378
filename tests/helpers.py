"""Shared test helpers: golden-fixture loading and the tolerance checks."""
import glob
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

# Output / LSE tolerance against an fp32 reference: |x - ref| <= ATOL + RTOL * |ref|.
ATOL = 2e-3
RTOL = 1e-2
# Gradient tolerance: max-abs.
GRAD_ATOL = 1e-2


def golden(name):
    return dict(np.load(os.path.join(GOLDEN, name + ".npz")))


def golden_names(prefix):
    return sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN, prefix + "*.npz")))


def assert_close(x, ref, atol=ATOL, rtol=RTOL, what="", mask=None):
    x = np.asarray(x, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    assert x.shape == ref.shape, (x.shape, ref.shape)
    both_inf = np.isinf(x) & np.isinf(ref) & (np.sign(x) == np.sign(ref))
    err = np.where(both_inf, 0.0, np.abs(x - ref))
    bound = atol + rtol * np.abs(np.where(np.isfinite(ref), ref, 0.0))
    bad = ~(err <= bound)
    if mask is not None:
        bad &= mask
    if bad.any():
        idx = np.argwhere(bad)[0]
        raise AssertionError("%s: %d/%d elements out of tolerance; first at %s: got %r want %r "
                             "(max err %.3g)" % (what, bad.sum(), bad.size, tuple(idx),
                                                 x[tuple(idx)], ref[tuple(idx)], np.nanmax(err)))


def max_abs(x, ref):
    return float(np.max(np.abs(np.asarray(x, np.float64) - np.asarray(ref, np.float64))))
