"""dtype conversion oracle (base R's as.* rules), known answers on CPU."""
import numpy as np

import oracle

NA_I32 = np.iinfo(np.int32).min
NA_I64 = np.iinfo(np.int64).min


def test_to_int32_truncates_and_marks_na():
    x = np.array([1.9, -1.9, 0.5, -0.5, 2147483647.5, 2147483648.0, -2147483648.0, -2147483647.9,
                  np.nan, np.inf, -np.inf, -0.0], dtype=np.float64)
    exp = np.array([1, -1, 0, 0, 2147483647, NA_I32, NA_I32, -2147483647, NA_I32, NA_I32, NA_I32, 0], np.int32)
    np.testing.assert_array_equal(oracle.convert(x, np.int32), exp)
    f = np.array([3.75, -2147483520.0, 2147483648.0], dtype=np.float32)
    np.testing.assert_array_equal(oracle.convert(f, np.int32), np.array([3, -2147483520, NA_I32], np.int32))
    i64 = np.array([NA_I64, 2147483647, 2147483648, -2147483647, -2147483648, 7], dtype=np.int64)
    np.testing.assert_array_equal(oracle.convert(i64, np.int32),
                                  np.array([NA_I32, 2147483647, NA_I32, -2147483647, NA_I32, 7], np.int32))


def test_to_int64_and_na_propagation():
    x = np.array([9.2e18, 9.3e18, -9.2e18, np.nan, 1e300, -0.999], dtype=np.float64)
    exp = np.array([9200000000000000000, NA_I64, -9200000000000000000, NA_I64, NA_I64, 0], np.int64)
    np.testing.assert_array_equal(oracle.convert(x, np.int64), exp)
    i = np.array([NA_I32, -5, 2147483647], dtype=np.int32)
    np.testing.assert_array_equal(oracle.convert(i, np.int64), np.array([NA_I64, -5, 2147483647], np.int64))


def test_to_float_types():
    i = np.array([NA_I32, 5, -3, 16777217], dtype=np.int32)
    d = oracle.convert(i, np.float64)
    assert np.isnan(d[0]) and list(d[1:]) == [5.0, -3.0, 16777217.0]
    f = oracle.convert(i, np.float32)
    assert np.isnan(f[0]) and f[3] == np.float32(16777216.0)  # round to nearest even
    big = np.array([2 ** 53 + 1, NA_I64], dtype=np.int64)
    d = oracle.convert(big, np.float64)
    assert d[0] == 2.0 ** 53 and np.isnan(d[1])
    x = np.array([1e300, -1e300, 0.1], dtype=np.float64)
    f = oracle.convert(x, np.float32)
    assert f[0] == np.inf and f[1] == -np.inf and f[2] == np.float32(0.1)


def test_bool_round_trip():
    x = np.array([0.0, -0.0, np.nan, 2.5, -1.0], dtype=np.float64)
    np.testing.assert_array_equal(oracle.convert(x, np.bool_), np.array([0, 0, 1, 1, 1], bool))
    b = np.array([True, False, True])
    np.testing.assert_array_equal(oracle.convert(b, np.int64), np.array([1, 0, 1], np.int64))
    np.testing.assert_array_equal(oracle.convert(b, np.float32), np.array([1, 0, 1], np.float32))


def test_strided_view_order():
    buf = np.arange(12, dtype=np.float64) + 0.5
    v = oracle.View(buf, (3, 4), (4, 1))  # a transposed view
    got = oracle.convert(v, np.int32)
    np.testing.assert_array_equal(got, np.trunc(buf.reshape(3, 4)).astype(np.int32))
