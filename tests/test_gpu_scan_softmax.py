"""cumsum/cumprod and softmax: CUDA path vs the oracle (relative 1e-5 for
float32, 1e-12 for float64)."""
import ctypes

import numpy as np
import pytest

import oracle
from helpers import assert_rel

pytestmark = pytest.mark.gpu
TOL = {"float": 1e-5, "double": 1e-12}
# below the smallest normal number relative error is meaningless (denormals)
ATOL = {"float": 1.2e-38, "double": 2.3e-308}
NP = {"float": np.float32, "double": np.float64}


@pytest.mark.parametrize("name", ["float", "double"])
def test_cumsum_flattened(acd, name):
    rng = np.random.default_rng(1)
    for n in [1, 2, 31, 4095, 4096, 4097, 100003, (1 << 22) + 9]:
        x = rng.uniform(0, 1, n).astype(NP[name])
        got = acd.cumsum(acd.as_tensor(x, dtype=name)).as_array()
        assert_rel(got, oracle.scan("cumsum", x), TOL[name], "cumsum n=%d" % n)


@pytest.mark.parametrize("name", ["float", "double"])
def test_cumprod_flattened(acd, name):
    rng = np.random.default_rng(2)
    for n in [1, 7, 5000, 70001]:
        x = rng.uniform(0.999, 1.001, n).astype(NP[name])
        got = acd.cumprod(acd.as_tensor(x, dtype=name)).as_array()
        assert_rel(got, oracle.scan("cumprod", x), TOL[name] * 10, "cumprod n=%d" % n)


@pytest.mark.parametrize("name", ["float", "double"])
def test_cumsum_along_axes(acd, name):
    rng = np.random.default_rng(3)
    for shape in [(64, 100000), (3, 5000), (33, 257), (1000, 6), (8, 300, 5), (1, 9000), (70, 2, 9)]:
        x = rng.uniform(0, 1, shape).astype(NP[name])
        t = acd.as_tensor(x, dtype=name)
        for axis in range(1, len(shape) + 1):
            got = acd.cumsum(t, axis=axis).as_array()
            assert_rel(got, oracle.scan("cumsum", x, axis - 1), TOL[name], "cumsum %s axis %d" % (shape, axis))
        got = acd.cumsum(t).as_array()
        assert_rel(got, oracle.scan("cumsum", x), TOL[name], "cumsum %s flat" % (shape,))


@pytest.mark.parametrize("name", ["float", "double"])
def test_cumprod_along_axes(acd, name):
    """Interleaved lanes of every lane-block width (1..33 lanes), one and many
    segments per chain, and an outer axis."""
    rng = np.random.default_rng(5)
    for shape, axis in [((2, 40000), 2), ((5, 20000), 2), ((12, 7000), 2), ((33, 3000), 2), ((40, 17, 30), 2),
                        ((3, 4, 9000), 3), ((16, 700), 2)]:
        x = rng.uniform(0.999, 1.001, shape).astype(NP[name])
        got = acd.cumprod(acd.as_tensor(x, dtype=name), axis=axis).as_array()
        assert_rel(got, oracle.scan("cumprod", x, axis - 1), TOL[name] * 10, "cumprod %s axis %d" % (shape, axis))


def test_scan_lanes_large():
    """Interleaved-lane scans of 150-260 MB (thousands of segments per chain):
    float32 and float64 sums, a ragged lane block, and a product."""
    import acediar as acd
    rng = np.random.default_rng(9)
    for shape, name, op in [((96, 400000), "float", "cumsum"), ((64, 500000), "double", "cumsum"),
                            ((40, 1000000), "float", "cumprod")]:
        lo, hi = (0.0, 1.0) if op == "cumsum" else (0.99999, 1.00001)
        x = rng.uniform(lo, hi, shape).astype(NP[name])
        got = getattr(acd, op)(acd.as_tensor(x, dtype=name), axis=2).as_array()
        tol = TOL[name] * (10 if op == "cumprod" else 1)
        assert_rel(got, oracle.scan(op, x, 1), tol, "%s %s %s" % (op, name, shape))


@pytest.mark.parametrize("name", ["float", "double"])
def test_cumsum_of_view(acd, name):
    rng = np.random.default_rng(4)
    x = rng.uniform(0, 1, (50, 70)).astype(NP[name])
    v = acd.transpose_view(acd.as_tensor(x, dtype=name))
    for axis in (1, 2):
        got = acd.cumsum(v, axis=axis).as_array()
        assert_rel(got, oracle.scan("cumsum", x.T, axis - 1), TOL[name], "cumsum transposed axis %d" % axis)


def test_scan_bounded_wait_reports_and_recovers(acd):
    """A tile that never publishes makes its successor's wait expire: the
    kernel returns, the status word is raised, and the context stays usable."""
    import acediar._lib as L
    import acediar.tensor as T
    x = np.ones(4096 * 8, dtype=np.float32)
    t = acd.as_tensor(x, dtype="float")
    lib = L.lib()
    ctx = T.context()
    acd.check_device_status()  # clean start
    L.check(lib.acd_ctx_set_scan_fault(ctx, 3, 20_000_000))  # tile 3 never publishes; 20 ms limit
    try:
        acd.cumsum(t)
        with pytest.raises(L.AcdError) as ei:
            acd.check_device_status()
        assert ei.value.status == 7
    finally:
        L.check(lib.acd_ctx_set_scan_fault(ctx, -1, 0))
    got = acd.cumsum(t).as_array()  # the context still works
    np.testing.assert_array_equal(got, np.arange(1, x.size + 1, dtype=np.float32))
    acd.check_device_status()


@pytest.mark.parametrize("name", ["float", "double"])
def test_softmax_along_axes(acd, name):
    rng = np.random.default_rng(5)
    for shape in [(65, 4096), (1000, 33), (7, 3000), (33, 64, 5), (4, 40000), (2048, 8), (8192, 600), (1030, 70)]:
        x = (rng.normal(0, 2, shape) + rng.uniform(-50, 50, (shape[0],) + (1,) * (len(shape) - 1))).astype(NP[name])
        t = acd.as_tensor(x, dtype=name)
        for axis in range(1, len(shape) + 1):
            got = acd.softmax(t, axis=axis).as_array()
            exp = oracle.softmax(x, axis - 1)
            assert_rel(got, exp, TOL[name], "softmax %s axis %d" % (shape, axis), atol=ATOL[name])


@pytest.mark.parametrize("name", ["float", "double"])
def test_softmax_rows_contiguous_lanes(acd, name):
    """Row softmax of column-major matrices (lanes contiguous): the two-pass
    wide kernels (4096+ lanes) and the single-read cluster kernel (fewer
    lanes: whole rows in a cluster's shared memory), with ragged lane blocks,
    steps past the last box, an outer axis, -inf entries and a row offset of
    +-50."""
    rng = np.random.default_rng(7)
    for shape, axis in [((4096, 2048), 2), ((2048, 700), 2), ((4100, 1200), 2), ((4096, 500, 2), 2),
                        ((8192, 96), 2), ((6000, 5000), 2), ((960, 4000), 2), ((500, 2500), 2),
                        ((600, 700, 3), 2), ((1000, 300), 2)]:
        x = (rng.normal(0, 2, shape) + rng.uniform(-50, 50, (shape[0],) + (1,) * (len(shape) - 1))).astype(NP[name])
        x.reshape(-1)[::977] = -np.inf
        t = acd.as_tensor(x, dtype=name)
        got = acd.softmax(t, axis=axis).as_array()
        exp = oracle.softmax(x, axis - 1)
        assert_rel(got, exp, TOL[name], "softmax %s axis %d" % (shape, axis), atol=ATOL[name])
    acd.check_device_status()


@pytest.mark.parametrize("name", ["float", "double"])
def test_softmax_whole_tensor(acd, name):
    rng = np.random.default_rng(6)
    for n in [1, 5, 1000, (1 << 20) + 1]:
        x = rng.normal(0, 3, n).astype(NP[name])
        got = acd.softmax(acd.as_tensor(x, dtype=name)).as_array()
        assert_rel(got, oracle.softmax(x), TOL[name], "softmax n=%d" % n, atol=ATOL[name])
        assert abs(got.astype(np.float64).sum() - 1.0) < (1e-4 if name == "float" else 1e-10)
