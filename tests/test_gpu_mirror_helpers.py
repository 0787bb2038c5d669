"""The R helpers built on the device kernels — diff, range, is.finite,
create_ones_like, tensor_pow, all.equal — against the oracle.  diff is one
subtraction per difference (bit-exact); pow is the elementwise math bar
(2 ulp)."""
import numpy as np
import pytest

import oracle
from helpers import assert_exact, assert_ulp

pytestmark = pytest.mark.gpu
NP = {"float": np.float32, "double": np.float64, "int32": np.int32}


@pytest.mark.parametrize("name", ["float", "double", "int32"])
def test_diff_sizes_lags_differences(acd, name):
    rng = np.random.default_rng(11)
    for shape in [(2,), (7,), (100003,), (1 << 21,), (33, 257), (6, 5, 4), (1000, 1000)]:
        if name == "int32":
            x = rng.integers(-1000, 1000, shape).astype(np.int32)
        else:
            x = rng.normal(0, 10, shape).astype(NP[name])
        t = acd.as_tensor(x, dtype=name)
        for lag, k in [(1, 1), (3, 1), (1, 3), (2, 2)]:
            if x.size <= lag * k:
                with pytest.raises(ValueError, match="empty result"):
                    acd.diff(t, lag=lag, differences=k)
                continue
            got = acd.diff(t, lag=lag, differences=k)
            exp = oracle.diff(x, lag, k)
            assert got.dtype == name and got.shape == exp.shape
            assert_exact(got.as_array(), exp, "diff %s %s lag=%d differences=%d" % (name, shape, lag, k))


def test_diff_of_views(acd):
    """A transposed view and an offset slice: diff runs over the logical
    column-major order."""
    rng = np.random.default_rng(12)
    x = rng.normal(0, 1, (300, 200)).astype(np.float32)
    t = acd.as_tensor(x, dtype="float")
    got = acd.diff(acd.transpose_view(t), lag=2).as_array()
    assert_exact(got, oracle.diff(x.T, 2), "diff of transpose")
    s = acd.subset(t, list(range(11, 301)), list(range(5, 201)))
    assert_exact(acd.diff(s).as_array(), oracle.diff(x[10:300, 4:200]), "diff of slice")
    import acediar.tensor as T
    v = x.reshape(-1, order="F")
    t1 = acd.as_tensor(v, dtype="float")
    w = T._slice_view(t1, [10], [50000])  # contiguous, storage offset 10
    assert_exact(acd.diff(w, differences=2).as_array(), oracle.diff(v[10:50010], 1, 2), "diff of offset view")


def test_diff_errors(acd):
    t = acd.as_tensor(np.array([1, 2, 3, 4.0]), dtype="float")
    for kw, pat in [({"lag": 0}, "lag must be positive"), ({"differences": -1}, "differences must be positive")]:
        with pytest.raises(ValueError, match=pat):
            acd.diff(t, **kw)
    with pytest.raises(ValueError, match="empty result"):
        acd.diff(acd.as_tensor(np.array([42.0]), dtype="float"))


@pytest.mark.parametrize("name", ["float", "double"])
def test_tensor_pow_broadcast(acd, name):
    rng = np.random.default_rng(13)
    for sa, sb in [((4096, 300), (4096, 300)), ((2, 3), (3,)), ((500, 70), (70,)), ((64, 32, 16), (64, 32)),
                   ((1,), (1000,)), ((1000,), (1,))]:
        a = rng.uniform(0.1, 4, sa).astype(NP[name])
        b = rng.uniform(-3, 3, sb).astype(NP[name])
        got = acd.tensor_pow(acd.as_tensor(a, dtype=name), acd.as_tensor(b, dtype=name)).as_array()
        if a.shape != b.shape and (a.size == 1 or b.size == 1):
            big = a if b.size == 1 else b
            exp = oracle.binary("pow", a if a.size > 1 else np.full(big.shape, a.reshape(-1)[0], a.dtype),
                                b if b.size > 1 else np.full(big.shape, b.reshape(-1)[0], b.dtype))
        else:
            exp = oracle.binary("pow", a, b)
        assert_ulp(got, exp, 2, "pow %s %s^%s" % (name, sa, sb))
    with pytest.raises(ValueError, match="Both arguments must be gpuTensor objects"):
        acd.tensor_pow(acd.as_tensor(np.ones(3), dtype=name), 2.0)


@pytest.mark.parametrize("name", ["float", "double", "int32"])
def test_range(acd, name):
    rng = np.random.default_rng(14)
    for n in [1, 5, 4097, 3000001]:
        x = (rng.normal(0, 100, n) if name != "int32" else rng.integers(-10 ** 6, 10 ** 6, n)).astype(NP[name])
        r = acd.range_(acd.as_tensor(x, dtype=name))
        assert r == [float(x.min()), float(x.max())], "range %s n=%d" % (name, n)


@pytest.mark.parametrize("name", ["float", "double"])
def test_is_finite(acd, name):
    rng = np.random.default_rng(15)
    x = rng.normal(0, 1, (700, 900)).astype(NP[name])
    assert acd.is_finite(acd.as_tensor(x, dtype=name)) is True
    for bad in (np.inf, -np.inf, np.nan):
        y = x.copy()
        y[699, 17] = bad
        assert acd.is_finite(acd.as_tensor(y, dtype=name)) is False
    big = np.full(5, np.finfo(NP[name]).max, dtype=NP[name])  # finite; max - max = 0
    assert acd.is_finite(acd.as_tensor(big, dtype=name)) is True
    assert acd.is_finite(acd.as_tensor(np.arange(10, dtype=np.int32), dtype="int32")) is True


@pytest.mark.parametrize("name", ["float", "double", "int32", "int64", "bool"])
def test_create_ones_like(acd, name):
    np_dt = {"float": np.float32, "double": np.float64, "int32": np.int32, "int64": np.int64, "bool": np.bool_}[name]
    for shape in [(1,), (5,), (3, 4), (64, 33, 7)]:
        t = acd.as_tensor(np.zeros(shape, dtype=np_dt), dtype=name)
        o = acd.create_ones_like(t)
        assert o.shape == t.shape and o.dtype == name
        assert_exact(o.as_array(), np.ones(shape, dtype=np_dt), "ones_like %s %s" % (name, shape))


def test_all_equal(acd):
    x = np.arange(1, 13, dtype=np.float64).reshape(3, 4, order="F")
    t = acd.as_tensor(x, dtype="double")
    assert acd.all_equal(t, x) is True
    assert acd.all_equal(t, acd.as_tensor(x * (1 + 1e-10), dtype="double")) is True
    msg = acd.all_equal(t, x + 1)
    assert isinstance(msg, str) and msg.startswith("Mean relative difference")
    assert acd.all_equal(t, np.ones(5)) == "Lengths (12, 5) differ"


def test_metadata_and_transfer_helpers(acd):
    x = np.arange(24, dtype=np.float64).reshape(2, 3, 4, order="F")
    t = acd.as_tensor(x, dtype="double")
    assert acd.size(t) == 24 and acd.dim(t) == [2, 3, 4]
    np.testing.assert_array_equal(acd.as_vector(t), np.arange(24.0))
    assert acd.as_numeric(acd.as_tensor(x, dtype="int32")).dtype == np.float64
    p = acd.permute(t, [3, 1, 2])
    assert p.shape == (4, 2, 3) and acd.shares_memory(p, t)
    np.testing.assert_array_equal(p.as_array(), np.transpose(x, (2, 0, 1)))
    with pytest.raises(ValueError, match="must match tensor dimensions"):
        acd.permute(t, [1, 2])
    info = acd.tensor_info(p)
    assert info["shape"] == [4, 2, 3] and info["size"] == 24 and info["is_contiguous"] is False
    assert not acd.shares_memory(t, acd.as_tensor(x, dtype="double"))
    import acediar.tensor as T
    v = acd.as_tensor(np.arange(100.0), dtype="double")
    assert not acd.shares_memory(T._slice_view(v, [0], [50]), T._slice_view(v, [50], [50]))
    assert acd.shares_memory(T._slice_view(v, [0], [51]), T._slice_view(v, [50], [50]))
    assert acd.tensor_to_scalar(acd.as_tensor(np.array([7.5]), dtype="float")) == 7.5
    with pytest.warns(UserWarning, match="using first element"):
        assert acd.tensor_to_scalar(v) == 0.0
    s = str(acd.as_tensor(np.ones((2, 2)), dtype="float"))
    assert s.startswith("gpuTensor with shape 2 x 2") and "Data:" in s
    assert "Use as.array() to view data" in str(acd.as_tensor(np.ones(101), dtype="float"))


def test_device_queries_and_seed(acd):
    st = acd.gpu_status()
    assert st["available"] is True and st["memory_available"] > 1e9 and st["info"].startswith("Found ")
    acd.set_random_seed(123)
    a = acd.rand_tensor((1000,), dtype="double").as_array()
    acd.set_random_seed(123)
    b = acd.rand_tensor((1000,), dtype="double").as_array()
    np.testing.assert_array_equal(a, b)


def test_legacy_vector_wrappers(acd):
    rng = np.random.default_rng(16)
    a, b = rng.normal(0, 1, 100001), rng.normal(0, 1, 100001)
    np.testing.assert_array_equal(acd.gpu_add(a, b), a + b)
    np.testing.assert_array_equal(acd.gpu_multiply(a, b), a * b)
    np.testing.assert_array_equal(acd.gpu_scale(a, 2.5), a * 2.5)
    d = acd.gpu_dot(a, b)
    assert abs(d - float(np.dot(a, b))) <= 1e-12 * float(np.abs(a * b).sum())
    assert acd.gpu_dot([], []) == 0.0 and acd.gpu_add([], []).size == 0
    with pytest.raises(ValueError, match="same length"):
        acd.gpu_add([1.0, 2.0], [1.0])
    with pytest.raises(ValueError, match="device only"):
        acd.gpu_add([1.0], [2.0], force_cpu=True)
