"""Full and per-axis reductions and arg-reductions: CUDA path vs the oracle.

Tolerances: relative 1e-5 (float32) / 1e-12 (float64) for sum, mean, var and
prod; exact for max, min, counts, integer sums and every index (first-index
tie rule).
"""
import itertools

import numpy as np
import pytest

import oracle
from helpers import assert_exact, assert_rel

pytestmark = pytest.mark.gpu
TOL = {"float": 1e-5, "double": 1e-12}
NP = {"float": np.float32, "double": np.float64}


def _check(op, got, exp, name, what):
    if op in ("max", "min", "count"):
        assert_exact(np.asarray(got, dtype=np.float64), np.asarray(exp, dtype=np.float64), what)
    else:
        assert_rel(got, exp, TOL[name], what, atol=1e-300)


@pytest.mark.parametrize("name", ["float", "double"])
@pytest.mark.parametrize("op", ["sum", "mean", "max", "min", "var", "prod"])
def test_full_reduction(acd, op, name):
    rng = np.random.default_rng(31)
    for n in [1, 2, 5, 255, 256, 1000, 4097, 65537, (1 << 20) + 3, 3 * (1 << 22) + 1]:
        if op == "prod":
            if n > 4097:
                continue
            x = rng.uniform(0.9, 1.1, n).astype(NP[name])
        else:
            x = (rng.normal(size=n) + 0.25).astype(NP[name])
        if op == "var" and n < 2:
            continue
        t = acd.as_tensor(x, dtype=name)
        got = getattr(acd, op)(t)
        exp = oracle.reduce(op, x)
        _check(op, np.float64(got), np.float64(exp), name, "%s n=%d" % (op, n))


@pytest.mark.parametrize("name", ["float", "double"])
def test_full_reduction_of_views(acd, name):
    rng = np.random.default_rng(12)
    x = rng.normal(size=(300, 41, 7)).astype(NP[name])
    t = acd.as_tensor(x, dtype=name)
    for perm in ([2, 1, 3], [3, 2, 1]):
        v = acd.permute_view(t, perm)
        xp = np.transpose(x, [p - 1 for p in perm])
        for op in ("sum", "var", "max"):
            _check(op, np.float64(getattr(acd, op)(v)), oracle.reduce(op, xp), name, "%s perm %s" % (op, perm))
        assert acd.which_max(v) == oracle.arg_reduce("argmax", xp)
        assert acd.which_min(v) == oracle.arg_reduce("argmin", xp)


SHAPES = [(3, 4), (1000, 7), (7, 1000), (64, 4096), (4096, 16), (17, 33, 9), (128, 64, 16), (2, 3, 4, 5),
          (1, 5000, 3), (5000, 1, 1), (3, 1 << 17)]


@pytest.mark.parametrize("name", ["float", "double"])
@pytest.mark.parametrize("op", ["sum", "mean", "max", "min", "var"])
def test_axis_reductions_every_axis_set(acd, op, name):
    rng = np.random.default_rng(17)
    for shape in SHAPES:
        x = rng.normal(size=shape).astype(NP[name])
        t = acd.as_tensor(x, dtype=name)
        nd = len(shape)
        for k in range(1, nd):
            for axes in itertools.combinations(range(1, nd + 1), k):
                got = getattr(acd, "tensor_" + op)(t, axis=list(axes)).as_array()
                exp = oracle.reduce(op, x, [a - 1 for a in axes])
                if op == "var" and np.prod([shape[a - 1] for a in axes]) < 2:
                    continue
                _check(op, got.astype(np.float64), np.asarray(exp).reshape(got.shape, order="F"), name,
                       "%s %s axes %s" % (op, shape, axes))


@pytest.mark.parametrize("name", ["float", "double"])
def test_axis_reduction_split_paths(acd, name):
    """Few long fibers: inner fibers split across CTAs, outer R split across CTAs."""
    rng = np.random.default_rng(3)
    for shape, axes in [((1 << 21, 3), [1]), ((3, 1 << 20), [2]), ((256, 8192), [2]), ((1 << 12, 1 << 10), [2]),
                        ((5, 4001, 2), [2])]:
        x = rng.normal(size=shape).astype(NP[name])
        t = acd.as_tensor(x, dtype=name)
        for op in ("sum", "var", "max"):
            got = getattr(acd, "tensor_" + op)(t, axis=axes).as_array()
            exp = oracle.reduce(op, x, [a - 1 for a in axes])
            _check(op, got.astype(np.float64), np.asarray(exp).reshape(got.shape, order="F"), name,
                   "%s %s" % (op, shape))
        for op in ("argmax", "argmin"):
            got = getattr(acd, op)(t, axis=axes[0]).as_array()
            exp = oracle.arg_reduce(op, x, axes[0] - 1)
            assert_exact(got, exp.reshape(got.shape, order="F"), "%s %s" % (op, shape))


@pytest.mark.parametrize("name", ["float", "double"])
def test_axis_reductions_on_transposed_views(acd, name):
    rng = np.random.default_rng(21)
    x = rng.normal(size=(96, 130)).astype(NP[name])
    v = acd.transpose_view(acd.as_tensor(x, dtype=name))
    for op in ("sum", "mean", "max", "var"):
        for axis in (1, 2):
            got = getattr(acd, "tensor_" + op)(v, axis=[axis]).as_array()
            exp = oracle.reduce(op, x.T, [axis - 1])
            _check(op, got.astype(np.float64), exp, name, "%s axis %d" % (op, axis))


@pytest.mark.parametrize("name", ["float", "double"])
def test_argmax_first_index_ties(acd, name):
    rng = np.random.default_rng(6)
    x = rng.integers(0, 4, size=(50, 33, 7)).astype(NP[name])  # many ties
    t = acd.as_tensor(x, dtype=name)
    assert acd.which_max(t) == oracle.arg_reduce("argmax", x)
    assert acd.which_min(t) == oracle.arg_reduce("argmin", x)
    for axis in (1, 2, 3):
        for op in ("argmax", "argmin"):
            got = getattr(acd, op)(t, axis=axis).as_array()
            exp = oracle.arg_reduce(op, x, axis - 1)
            assert_exact(got, exp, "%s axis %d" % (op, axis))
    big = np.zeros((1 << 20) + 17, dtype=NP[name])
    big[[100, 5000, (1 << 20)]] = 7.0
    assert acd.which_max(acd.as_tensor(big, dtype=name)) == 101


def test_int32_sum_bit_exact_and_bool_counts(acd):
    rng = np.random.default_rng(19)
    x = rng.integers(-1000, 1001, size=(512, 256, 16)).astype(np.int32)
    t = acd.as_tensor(x, dtype="int32")
    s = acd.tensor_sum(t)
    assert int(s.as_array()[0]) == int(x.astype(np.int64).sum())
    for axis in (1, 2, 3):
        got = acd.tensor_sum(t, axis=[axis]).as_array()
        assert_exact(got.astype(np.int64), x.astype(np.int64).sum(axis=axis - 1), "int32 sum axis %d" % axis)
    m = acd.as_tensor(rng.random((300, 77)) < 0.3, dtype="bool")
    mh = m.as_array()
    got = acd.tensor_count(m, axis=[1]).as_array()
    assert got.dtype == np.int32
    assert_exact(got, mh.sum(axis=0).astype(np.int32), "count axis 1")
    assert int(acd.tensor_sum(m).as_array()[0]) == int(mh.sum())


@pytest.mark.parametrize("name", ["float", "double"])
def test_fused_sum_var(acd, name):
    rng = np.random.default_rng(44)
    for n in [2, 1000, (1 << 22) + 7]:
        x = (rng.normal(size=n) * 3 + 10).astype(NP[name])
        s, v = acd.sum_var(acd.as_tensor(x, dtype=name))
        es, ev = oracle.sum_var(x)
        assert_rel(s, es, TOL[name], "sum n=%d" % n)
        assert_rel(v, ev, TOL[name], "var n=%d" % n)


def test_keep_dims_shapes(acd):
    x = np.arange(24, dtype=np.float64).reshape((2, 3, 4), order="F")
    t = acd.as_tensor(x, dtype="double")
    assert acd.tensor_sum(t, axis=[2], keep_dims=True).shape == (2, 1, 4)
    assert acd.tensor_sum(t, axis=[1, 3], keep_dims=True).shape == (1, 3, 1)
    assert acd.argmax(t, axis=3, keep_dims=True).shape == (2, 3, 1)


@pytest.mark.parametrize("name,dt", [("float", np.float32), ("double", np.float64), ("int32", np.int32),
                                     ("int64", np.int64), ("bool", np.bool_)])
def test_any_all_three_valued(acd, name, dt):
    """any / all with R's NA rules (NaN and INT_MIN integers are NA), over the
    whole tensor and along axes, small and multi-CTA sizes, and a view."""
    rng = np.random.default_rng(41)
    na = {np.float32: np.nan, np.float64: np.nan, np.int32: np.iinfo(np.int32).min,
          np.int64: np.iinfo(np.int64).min}.get(dt)

    def check(x, t, what):
        for op in ("any", "all"):
            got = getattr(acd, op)(t)
            exp = oracle.reduce(op, x)
            assert (got is None and np.isnan(exp)) or (got is not None and float(got) == exp), (what, op, got, exp)
            for ax in range(1, x.ndim + 1):
                r = getattr(acd, op)(t, axis=[ax]).as_array().astype(np.float64).reshape(-1)
                r[r == np.iinfo(np.int32).min] = np.nan
                e = np.asarray(oracle.reduce(op, x, [ax - 1]), dtype=np.float64).reshape(-1)
                assert np.array_equal(np.isnan(r), np.isnan(e)) and np.array_equal(r[~np.isnan(r)], e[~np.isnan(e)]), \
                    (what, op, ax)

    for shape in [(7,), (33, 40), (16, 300, 5), (2, 3000001)]:
        base = (rng.random(shape) < 0.97)
        x = base.astype(dt) if dt != np.bool_ else base
        t = acd.as_tensor(x, dtype=name)
        check(x, t, "%s mostly true" % (shape,))
        y = np.ones(shape, dtype=dt)
        if na is not None:
            y.reshape(-1)[rng.integers(0, y.size, 3)] = na
        check(y, acd.as_tensor(y, dtype=name), "%s ones with NA" % (shape,))
        z = np.zeros(shape, dtype=dt)
        check(z, acd.as_tensor(z, dtype=name), "%s zeros" % (shape,))
    m = (rng.random((64, 48)) < 0.5).astype(dt) if dt != np.bool_ else rng.random((64, 48)) < 0.5
    check(m.T, acd.transpose_view(acd.as_tensor(m, dtype=name)), "transposed view")
