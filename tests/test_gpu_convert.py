"""dtype conversion on the GPU vs the oracle: every pair of the five dtypes,
edge values (NaN, +-inf, range limits, NA integers), contiguous and permuted
views.  Bit-exact, including the positions of NaN and NA."""
import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu
NAMES = {"float": np.float32, "double": np.float64, "int32": np.int32, "int64": np.int64, "bool": np.bool_}
NA_I32 = np.iinfo(np.int32).min
NA_I64 = np.iinfo(np.int64).min


def _data(name, rng, shape):
    n = int(np.prod(shape))
    if name in ("float", "double"):
        x = rng.normal(0, 3e9, n)
        edges = [np.nan, np.inf, -np.inf, 0.0, -0.0, 0.5, -0.5, 2147483647.5, 2147483648.0, -2147483648.0,
                 -2147483647.9, 9.3e18, -9.3e18, 1e300, 1.9, -1.9]
        k = min(n, len(edges))
        x[:k] = edges[:k]
        with np.errstate(over="ignore"):  # 1e300 and 9.3e18 overflow float32 to inf on purpose
            return x.astype(NAMES[name]).reshape(shape, order="F")
    if name == "int32":
        x = rng.integers(-2 ** 31 + 1, 2 ** 31 - 1, n, dtype=np.int64).astype(np.int32)
        k = min(n, 4)
        x[:k] = [NA_I32, 0, 2147483647, 16777217][:k]
        return x.reshape(shape, order="F")
    if name == "int64":
        x = rng.integers(-2 ** 62, 2 ** 62, n, dtype=np.int64)
        k = min(n, 5)
        x[:k] = [NA_I64, 0, 2 ** 53 + 1, 2147483648, -2147483647][:k]
        return x.reshape(shape, order="F")
    return (rng.random(n) < 0.5).reshape(shape, order="F")


def _same(a, b, what):
    assert a.dtype == b.dtype and a.shape == b.shape, what
    if a.dtype.kind == "f":
        assert np.array_equal(np.isnan(a), np.isnan(b)), what + ": NaN positions"
        m = ~np.isnan(a)
        assert np.array_equal(a[m].view(np.uint8), b[m].view(np.uint8)) or np.array_equal(a[m], b[m]), what
    else:
        np.testing.assert_array_equal(a, b, err_msg=what)


@pytest.mark.parametrize("src", list(NAMES))
def test_convert_all_pairs(acd, src):
    rng = np.random.default_rng(21)
    for shape in [(1,), (1000,), (37, 65), (64, 33, 5)]:
        x = _data(src, rng, shape)
        t = acd.as_tensor(x, dtype=src)
        for dst in NAMES:
            got = acd.to_dtype(t, dst).as_array()
            exp = oracle.convert(x, NAMES[dst])
            _same(np.asarray(got).astype(NAMES[dst]), exp, "%s -> %s %s" % (src, dst, shape))
        if len(shape) == 3:  # a permuted view converts in logical order
            v = acd.permute_view(t, [3, 1, 2])
            xv = np.transpose(x, (2, 0, 1))
            for dst in NAMES:
                got = acd.to_dtype(v, dst).as_array()
                _same(np.asarray(got).astype(NAMES[dst]), oracle.convert(np.ascontiguousarray(xv), NAMES[dst]),
                      "%s -> %s permuted" % (src, dst))


def test_convert_aliases_and_errors(acd):
    t = acd.as_tensor(np.array([1.5, -2.5]), dtype="double")
    assert acd.to_dtype(t, "int").dtype == "int32"
    assert acd.to_dtype(t, "float32").dtype == "float"
    assert acd.to_dtype(t, "long").dtype == "int64"
    assert acd.to_dtype(t, "half").dtype == "float16"
    assert acd.to_dtype(t, "int8").dtype == "int8"
    with pytest.raises(ValueError, match="Unsupported target dtype: uint16"):
        acd.to_dtype(t, "uint16")
