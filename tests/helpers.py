"""Shared test helpers: golden-fixture loading and the tolerance checks.

Two bars, both written here:

* The north-star bar against the fp32 oracle: outputs and LSE |x - ref| <= 2e-3 +
  1e-2 |ref| elementwise, gradients max-abs <= 1e-2.  fp16 results meet it everywhere.
* The rounding bound: |x - ref| <= 1e-4 + bound elementwise, where ``bound`` (from the
  oracle's ``unit_roundoff`` functions) is the worst case of rounding the operands every
  FlashAttention rounds to the input type -- P before P V and P^T dO, dS before dS K and
  dS^T Q -- and the output itself.  1e-4 covers fp32 accumulation order and ex2.approx.
  bf16 results are held to it (plus a mean error <= 2e-3): with an 8-bit significand one
  rounding of an output of size 4 is already 0.0156, above the absolute 1e-2 gradient
  bar, so no bf16 kernel meets the north-star bar on every element.  Measured on the
  dense test cases the kernels stay below 0.9 of the bound in both dtypes.
"""
import collections
import glob
import hashlib
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

ATOL = 2e-3        # north-star output / LSE bar: |x - ref| <= ATOL + RTOL |ref|
RTOL = 1e-2
GRAD_ATOL = 1e-2   # north-star gradient bar (max-abs)
BOUND_ATOL = 1e-4  # fp32 accumulation / ex2.approx allowance on top of the rounding bound
MEAN_ATOL = 2e-3   # mean absolute error of bf16 results


def golden(name):
    return dict(np.load(os.path.join(GOLDEN, name + ".npz")))


def golden_names(prefix):
    return sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN, prefix + "*.npz")))


def is_bf16(dtype):
    return dtype is not None and "bfloat16" in str(dtype)


def assert_close(x, ref, atol=ATOL, rtol=RTOL, what="", mask=None):
    """Elementwise |x - ref| <= atol + rtol |ref| (the north-star bar by default);
    infinities must match in sign."""
    x = np.asarray(x, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    assert x.shape == ref.shape, (x.shape, ref.shape)
    both_inf = np.isinf(x) & np.isinf(ref) & (np.sign(x) == np.sign(ref))
    with np.errstate(invalid="ignore"):
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


def assert_within_bound(x, ref, bound, what="", mean_atol=MEAN_ATOL):
    """|x - ref| <= BOUND_ATOL + bound elementwise and mean |x - ref| <= mean_atol."""
    x = np.asarray(x, np.float64)
    ref = np.asarray(ref, np.float64)
    bound = np.asarray(bound, np.float64)
    assert x.shape == ref.shape == bound.shape, (x.shape, ref.shape, bound.shape)
    err = np.abs(x - ref)
    bad = ~(err <= BOUND_ATOL + bound)
    if bad.any():
        idx = tuple(np.argwhere(bad)[0])
        raise AssertionError("%s: %d/%d elements outside the rounding bound; first at %s: got %r "
                             "want %r bound %.3g (max err / bound %.3g)"
                             % (what, bad.sum(), bad.size, idx, x[idx], ref[idx], bound[idx],
                                np.max(err / (BOUND_ATOL + bound))))
    assert err.mean() <= mean_atol, "%s: mean abs error %.3g" % (what, err.mean())


def assert_out_close(x, ref, dtype, bound=None, what=""):
    """A kernel output (attention out) in `dtype` against the fp32 oracle: fp16 must meet
    the north-star bar; bf16 must stay inside the rounding bound.  When the bound is
    given it is checked for fp16 as well."""
    if bound is not None:
        assert_within_bound(x, ref, bound, what)
    if not is_bf16(dtype):
        assert_close(x, ref, what=what)
    else:
        assert bound is not None, "bf16 outputs are checked against the rounding bound"


def assert_grad_close(got, want, dtype, what="", bound=None, want_faithful=None):
    """Gradients: fp16 max-abs <= GRAD_ATOL against the exact fp32 gradient; every dtype,
    when the bound is given, inside the rounding bound around the reference computed
    with D = rowsum(dO * O) from the output the backward was given (``want_faithful``)."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    if bound is not None:
        assert_within_bound(got, want if want_faithful is None else want_faithful, bound, what)
    if not is_bf16(dtype):
        err = np.abs(got - want)
        assert err.max() <= GRAD_ATOL, "%s max-abs %.4g" % (what, err.max())
    else:
        assert bound is not None, "bf16 gradients are checked against the rounding bound"


def max_abs(x, ref):
    return float(np.max(np.abs(np.asarray(x, np.float64) - np.asarray(ref, np.float64))))


def unit_roundoff(dtype):
    return 2.0 ** -8 if is_bf16(dtype) else 2.0 ** -11


_BWD_REFS = collections.OrderedDict()


def bwd_refs(args, o, unit_roundoff, **kw):
    """The oracle's exact gradients, its rounding-faithful gradients and their bounds for
    attention_bwd_ref(*args, **kw) with the kernel's output ``o``.

    The backward tests run each case in both backward modes on the same inputs, and the
    forward (hence ``o``) does not depend on the mode, so recent results are kept (up to
    1 GiB, oldest dropped first; the varlen tests make one entry per sequence), keyed by
    a digest of every array and option: the CPU oracle, not the GPU, dominates the long
    cases."""
    from oracle import attention_ref as R
    h = hashlib.sha1(repr((sorted(kw.items()), unit_roundoff,
                           [a if np.isscalar(a) or isinstance(a, bool) else a.shape
                            for a in args])).encode())
    for a in list(args) + [o]:
        if isinstance(a, np.ndarray):
            h.update(np.ascontiguousarray(a).tobytes())
    key = h.hexdigest()
    if key not in _BWD_REFS:
        exact = R.attention_bwd_ref(*args, **kw)
        faithful, bounds = R.attention_bwd_ref(*args, o=o, unit_roundoff=unit_roundoff, **kw)
        _BWD_REFS[key] = (exact, faithful, bounds)
        size = lambda e: sum(a.nbytes for part in e for a in part)
        while len(_BWD_REFS) > 1 and sum(size(e) for e in _BWD_REFS.values()) > 2 ** 30:
            _BWD_REFS.popitem(last=False)
    return _BWD_REFS[key]
