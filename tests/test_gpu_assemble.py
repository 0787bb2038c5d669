"""Slices, slice and mask assignment, concat, stack, repeat and pad on the
GPU against the oracle: every dtype, views as inputs, each axis, every pad
mode.  Data movement only, so every comparison is bit-exact."""
import numpy as np
import pytest

import oracle
from helpers import assert_exact

pytestmark = pytest.mark.gpu
NAMES = {"float": np.float32, "double": np.float64, "int32": np.int32, "int64": np.int64, "bool": np.bool_}


def _rand(name, shape, rng):
    if name == "bool":
        return rng.random(shape) < 0.5
    if name in ("int32", "int64"):
        return rng.integers(-10 ** 6, 10 ** 6, shape).astype(NAMES[name])
    return rng.normal(size=shape).astype(NAMES[name])


@pytest.mark.parametrize("name", list(NAMES))
def test_concat_and_stack(acd, name):
    rng = np.random.default_rng(31)
    for axis in (1, 2, 3):
        shapes = []
        for k in (3, 1, 5):
            s = [4, 6, 5]
            s[axis - 1] = k
            shapes.append(tuple(s))
        xs = [_rand(name, s, rng) for s in shapes]
        ts = [acd.as_tensor(x, dtype=name) for x in xs]
        assert_exact(acd.concat_tensor(ts, axis=axis).as_array(), oracle.concat(xs, axis - 1), "concat %d" % axis)
    xs = [_rand(name, (7, 3, 4), rng) for _ in range(3)]
    ts = [acd.as_tensor(x, dtype=name) for x in xs]
    for axis in (1, 2, 3, 4):
        assert_exact(acd.stack_tensor(ts, axis=axis).as_array(), oracle.stack(xs, axis - 1), "stack %d" % axis)
    # views as inputs
    v = acd.transpose_view(acd.as_tensor(_rand(name, (6, 4), rng), dtype=name))
    w = acd.as_tensor(_rand(name, (4, 2), rng), dtype=name)
    assert_exact(acd.concat_tensor([v, w], axis=2).as_array(),
                 np.concatenate([v.as_array(), w.as_array()], axis=1), "concat of a transposed view")


@pytest.mark.parametrize("name", list(NAMES))
def test_repeat(acd, name):
    rng = np.random.default_rng(32)
    for shape, reps in [((2, 2), (2, 1)), ((5, 3), (1, 4)), ((4, 3, 2), (2, 3, 2)), ((300, 7), (3, 2)),
                        ((1000,), (70,)), ((2, 3, 2, 2), (1, 2, 2, 2))]:
        x = _rand(name, shape, rng)
        got = acd.repeat_tensor(acd.as_tensor(x, dtype=name), list(reps)).as_array()
        assert_exact(got, oracle.repeat(x, reps), "repeat %s %s" % (shape, reps))


@pytest.mark.parametrize("name", list(NAMES))
def test_pad_modes(acd, name):
    rng = np.random.default_rng(33)
    for shape, width in [((2, 2), ((1, 1), (1, 1))), ((5, 4, 3), ((2, 0), (0, 3), (1, 1))),
                         ((300, 200), ((3, 5), (0, 7))), ((6,), ((6, 6),)), ((3, 5), ((3, 3), (5, 5)))]:
        x = _rand(name, shape, rng)
        t = acd.as_tensor(x, dtype=name)
        b = [w[0] for w in width]
        a = [w[1] for w in width]
        for mode in ("constant", "reflect", "replicate"):
            got = acd.pad(t, np.asarray(width), mode=mode, value=-7.5).as_array()
            assert_exact(got, oracle.pad(x, b, a, mode, -7.5), "pad %s %s %s" % (shape, width, mode))
    with pytest.raises(Exception, match="reflect padding larger"):
        acd.pad(acd.as_tensor(_rand(name, (3, 2), rng), dtype=name), [[4, 0], [0, 0]], mode="reflect")


@pytest.mark.parametrize("name", list(NAMES))
def test_slices_and_assignment(acd, name):
    rng = np.random.default_rng(34)
    x = _rand(name, (9, 7, 5), rng)
    t = acd.as_tensor(x, dtype=name)
    assert_exact(acd.subset(t, [2, 3, 4], None, 5).as_array(), x[1:4, :, 4], "subset with a dropped axis")
    assert_exact(acd.subset(t, None, [7], [1, 2]).as_array(), x[:, 6:7, 0:2], "subset keeps a length-1 range")
    y = x.copy()
    acd.assign(t, [2, 3], None, [4, 5], value=3)
    y[1:3, :, 3:5] = oracle.convert(np.array([3.0]), NAMES[name])[0]
    src = _rand(name, (2, 7, 2), rng)
    acd.assign(t, [5, 6], None, [1, 2], value=acd.as_tensor(src, dtype=name))
    y[4:6, :, 0:2] = src
    assert_exact(t.as_array(), y, "slice assignment")
    m = rng.random((9, 7, 5)) < 0.3
    acd.assign(t, acd.as_tensor(m, dtype="bool"), value=1)
    y[m] = oracle.convert(np.array([1.0]), NAMES[name])[0]
    assert_exact(t.as_array(), y, "mask assignment")
    # mask assignment through a transposed view of a matrix
    z = _rand(name, (40, 30), rng)
    tz = acd.as_tensor(z, dtype=name)
    mz = rng.random((30, 40)) < 0.5
    acd.assign(acd.transpose_view(tz), acd.as_tensor(mz, dtype="bool"), value=0)
    zz = z.copy()
    zz.T[mz] = 0
    assert_exact(tz.as_array(), zz, "mask assignment on a view")


def test_assembly_errors(acd):
    a = acd.as_tensor(np.zeros((2, 3)), dtype="double")
    b = acd.as_tensor(np.zeros((2, 4)), dtype="double")
    with pytest.raises(Exception, match="Non-concat dimensions must match"):
        acd.concat_tensor([a, b], axis=1)
    with pytest.raises(Exception, match="identical shape"):
        acd.stack_tensor([a, b], axis=1)
    with pytest.raises(ValueError, match="repeat counts must be positive"):
        acd.repeat_tensor(a, [0, 1])
    with pytest.raises(ValueError, match="out of bounds"):
        acd.subset(a, 3, None)
    with pytest.raises(ValueError, match="contiguous ranges"):
        acd.subset(a, None, [1, 3])
