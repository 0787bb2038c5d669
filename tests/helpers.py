"""Comparison helpers shared by the tests."""
import json
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def golden_cases():
    with open(os.path.join(HERE, "golden", "reference_cases.json")) as f:
        return json.load(f)["cases"]


def _ordered(a):
    a = np.asarray(a)
    if a.dtype == np.float32:
        i = a.view(np.int32).astype(np.int64)
        return np.where(i < 0, -(i & 0x7FFFFFFF), i)
    i = a.astype(np.float64).view(np.int64)
    return np.where(i < 0, -(i & 0x7FFFFFFFFFFFFFFF), i)


def ulp_distance(a, b):
    """Elementwise distance in units in the last place of a's dtype."""
    a = np.asarray(a)
    b = np.asarray(b).astype(a.dtype)
    oa, ob = _ordered(a), _ordered(b)
    with np.errstate(over="ignore"):
        d = np.abs(oa - ob)
    both_nan = np.isnan(a) & np.isnan(b)
    same = (a == b) | both_nan
    return np.where(same, 0, d)


def assert_ulp(actual, expected, max_ulp, what=""):
    actual = np.asarray(actual)
    expected = np.asarray(expected)
    assert actual.shape == expected.shape, "%s: shape %s vs %s" % (what, actual.shape, expected.shape)
    d = ulp_distance(actual, expected)
    worst = float(np.max(d)) if d.size else 0.0
    assert worst <= max_ulp, "%s: %g ulp > %d (at %s: %r vs %r)" % (
        what, worst, max_ulp, np.unravel_index(int(np.argmax(d)), d.shape), actual.reshape(-1)[int(np.argmax(d))],
        expected.reshape(-1)[int(np.argmax(d))])


def assert_rel(actual, expected, rel, what="", atol=0.0):
    actual = np.asarray(actual, dtype=np.float64)
    expected = np.asarray(expected, dtype=np.float64)
    assert actual.shape == expected.shape, "%s: shape %s vs %s" % (what, actual.shape, expected.shape)
    err = np.abs(actual - expected)
    bound = rel * np.abs(expected) + atol
    bad = err > bound
    if np.any(bad):
        k = int(np.argmax(np.where(bad, err / np.maximum(bound, 1e-300), 0)))
        raise AssertionError("%s: relative error %.3g > %.1g at %d (%r vs %r)" % (
            what, err.reshape(-1)[k] / max(abs(expected.reshape(-1)[k]), 1e-300), rel, k,
            actual.reshape(-1)[k], expected.reshape(-1)[k]))


def assert_exact(actual, expected, what=""):
    actual = np.asarray(actual)
    expected = np.asarray(expected)
    assert actual.shape == expected.shape, "%s: shape %s vs %s" % (what, actual.shape, expected.shape)
    ne = actual != expected
    if np.any(ne):
        k = int(np.argmax(ne.reshape(-1)))
        raise AssertionError("%s: %d mismatches, first at %d (%r vs %r)" % (
            what, int(ne.sum()), k, actual.reshape(-1)[k], expected.reshape(-1)[k]))
