"""float16 and int8 tensors, the reference's float16 / int8 / int64 launcher
names, the contraction launchers, and log()'s domain error.

Tolerances: float16 arithmetic, comparisons, conversions and every int8 op
are bit-exact against the oracle (one rounding to binary16 per operation;
int8 wraps modulo 256).  float16 sums accumulate the exact half values in
float64: relative 1e-12.  Contractions (cuBLAS, outside the hot path) are
checked against float64 numpy products: relative 1e-5 of the row scale for
float32 and 1e-12 for float64; float16 products (float32 accumulation, one
rounding to half) within 2 half ulp of the float64 product.
"""
import ctypes

import numpy as np
import pytest
import torch

import oracle
from helpers import assert_exact, assert_rel

pytestmark = pytest.mark.gpu
SHAPES = [(1,), (7,), (4099,), (1 << 16,), (33, 17), (64, 40, 3)]


def _half_data(rng, shape):
    x = (rng.normal(0, 40, shape)).astype(np.float16)
    flat = x.reshape(-1)
    edges = np.array([0.0, -0.0, 65504, -65504, 6e-8, np.inf, -np.inf, np.nan, 1.0, 2049.0], dtype=np.float16)
    k = min(flat.size, edges.size)
    flat[:k] = edges[:k]
    return x


def _i8_data(rng, shape):
    return rng.integers(-128, 128, size=shape, dtype=np.int64).astype(np.int8)


def _bits(a):
    """Bit patterns of float16 values with every NaN mapped to one pattern
    (the payload of a NaN result is not part of the contract); other dtypes
    unchanged."""
    a = np.asarray(a)
    if a.dtype != np.float16:
        return a
    return np.where(np.isnan(a), np.uint16(0x7E00), a.view(np.uint16))


@pytest.mark.parametrize("op", ["add", "sub", "mul", "div", "max", "min", "gt", "lt", "eq", "ne", "ge", "le"])
def test_float16_binary(acd, op):
    rng = np.random.default_rng(1)
    for shape in SHAPES:
        a, b = _half_data(rng, shape), _half_data(rng, shape)
        b.reshape(-1)[-1] = 0.0  # a division by zero
        ta, tb = acd.as_tensor(a, dtype="float16"), acd.as_tensor(b, dtype="float16")
        got = getattr(ta, {"add": "__add__", "sub": "__sub__", "mul": "__mul__", "div": "__truediv__",
                           "gt": "__gt__", "lt": "__lt__", "eq": "__eq__", "ne": "__ne__", "ge": "__ge__",
                           "le": "__le__"}[op])(tb) if op not in ("max", "min") else \
            (acd.pmax if op == "max" else acd.pmin)(ta, tb)
        ref = oracle.binary(op, a, b)
        g = got.as_array()
        if g.dtype == np.bool_:
            g = g.astype(np.uint8)
        assert_exact(_bits(g), _bits(ref), "float16 %s %s" % (op, shape))


def test_float16_broadcast_and_views(acd):
    rng = np.random.default_rng(2)
    X = _half_data(rng, (48, 40))
    r = _half_data(rng, (1, 40))
    tX, tr = acd.as_tensor(X, dtype="float16"), acd.as_tensor(r, dtype="float16")
    assert_exact(_bits((tX + tr).as_array()), _bits(oracle.binary("add", X, r)), "float16 row broadcast")
    v = acd.transpose_view(tX)
    assert_exact(_bits((v * v).as_array()), _bits(oracle.binary("mul", X.T, X.T)), "float16 on a transposed view")
    assert_exact(_bits(acd.contiguous(v).as_array()), _bits(np.ascontiguousarray(X.T)), "float16 contiguous()")


@pytest.mark.parametrize("op", ["add", "sub", "mul", "div", "rsub", "rdiv"])
def test_float16_scalar(acd, op):
    rng = np.random.default_rng(3)
    x = _half_data(rng, (5000,))
    t = acd.as_tensor(x, dtype="float16")
    for s in (2.0, 0.1, -3.75, 1e-3):
        got = {"add": lambda: t + s, "sub": lambda: t - s, "mul": lambda: t * s, "div": lambda: t / s,
               "rsub": lambda: s - t, "rdiv": lambda: s / t}[op]().as_array()
        assert_exact(_bits(got), _bits(oracle.scalar(op, x, s)), "float16 %s %g" % (op, s))


@pytest.mark.parametrize("op", ["add", "sub", "mul", "max", "min", "gt", "le"])
def test_int8_binary_wraps(acd, op):
    rng = np.random.default_rng(4)
    for shape in SHAPES:
        a, b = _i8_data(rng, shape), _i8_data(rng, shape)
        ta, tb = acd.as_tensor(a, dtype="int8"), acd.as_tensor(b, dtype="int8")
        got = {"add": lambda: ta + tb, "sub": lambda: ta - tb, "mul": lambda: ta * tb,
               "max": lambda: acd.pmax(ta, tb), "min": lambda: acd.pmin(ta, tb), "gt": lambda: ta > tb,
               "le": lambda: ta <= tb}[op]().as_array()
        if got.dtype == np.bool_:
            got = got.astype(np.uint8)
        assert_exact(got, oracle.binary(op, a, b), "int8 %s %s" % (op, shape))


NARROW = {"float": np.float32, "double": np.float64, "int32": np.int32, "int64": np.int64, "bool": np.bool_,
          "float16": np.float16, "int8": np.int8}


def _conv_data(name, rng, n):
    if name in ("float", "double", "float16"):
        x = rng.normal(0, 200, n)
        edges = [np.nan, np.inf, -np.inf, 0.0, -0.0, 127.9, 128.0, -128.0, -128.9, -129.0, 65504.0, 65520.0,
                 1e9, 2.5, -2.5, 0.00006103515625]
        x[:len(edges)] = edges
        with np.errstate(over="ignore"):
            return x.astype(NARROW[name])
    if name == "int32":
        x = rng.integers(-70000, 70000, n).astype(np.int32)
        x[:4] = [np.iinfo(np.int32).min, 300, -129, 2049]
        return x
    if name == "int64":
        x = rng.integers(-70000, 70000, n).astype(np.int64)
        x[:3] = [np.iinfo(np.int64).min, 2 ** 40 + 7, -255]
        return x
    if name == "int8":
        return _i8_data(rng, (n,))
    return rng.random(n) < 0.5


@pytest.mark.parametrize("src", sorted(NARROW))
def test_conversions_with_float16_and_int8(acd, src):
    rng = np.random.default_rng(5)
    x = _conv_data(src, rng, 3001)
    t = acd.as_tensor(x, dtype=src)
    for dst in sorted(NARROW):
        if "float16" not in (src, dst) and "int8" not in (src, dst):
            continue  # the five-dtype pairs are covered by test_gpu_convert.py
        got = acd.to_dtype(t, dst).as_array()
        ref = oracle.convert(x, NARROW[dst])
        assert got.dtype == ref.dtype, (src, dst)
        if got.dtype.kind == "f":
            assert_exact(np.isnan(got), np.isnan(ref), "%s -> %s NaN positions" % (src, dst))
            assert_exact(_bits(np.where(np.isnan(got), 0, got).astype(got.dtype)),
                         _bits(np.where(np.isnan(ref), 0, ref).astype(ref.dtype)), "%s -> %s" % (src, dst))
        else:
            assert_exact(got, ref, "%s -> %s" % (src, dst))


def test_narrow_reductions(acd):
    rng = np.random.default_rng(6)
    for n in (1, 100, 4099, (1 << 20) + 7):
        h = (rng.normal(0, 30, n)).astype(np.float16)
        th = acd.as_tensor(h, dtype="float16")
        assert_rel(acd.sum(th), oracle.reduce("sum", h), 1e-12, "float16 sum n=%d" % n)
        assert_rel(acd.mean(th), oracle.reduce("mean", h), 1e-12, "float16 mean n=%d" % n)
        assert int(acd.tensor_count(th).as_array()[0]) == int(np.count_nonzero(h))
        b = _i8_data(rng, (n,))
        tb = acd.as_tensor(b, dtype="int8")
        assert int(acd.tensor_sum(tb).as_array()[0]) == int(b.astype(np.int64).sum())
        assert int(acd.tensor_max(tb).as_array()[0]) == int(b.max())
        assert int(acd.tensor_min(tb).as_array()[0]) == int(b.min())
    M = (rng.normal(0, 3, (300, 41))).astype(np.float16)
    tm = acd.as_tensor(M, dtype="float16")
    for ax in (1, 2):
        got = acd.tensor_sum(tm, axis=[ax]).as_array().astype(np.float64)
        assert_rel(got, oracle.reduce("sum", M, [ax - 1]).astype(np.float32).astype(np.float64), 1e-7,
                   "float16 axis %d sum (float result)" % ax, atol=1e-30)
    with pytest.raises(acd.AcdError):
        acd.var(tm)  # variance of float16 is not supported


# ---- reference launcher names ------------------------------------------------
class RefDesc(ctypes.Structure):
    """cuda_utils::TensorDescriptor (src/cuda_utils.h:111-118)."""
    _fields_ = [("data", ctypes.c_void_p), ("ndims", ctypes.c_int), ("shape", ctypes.c_int * 8),
                ("strides", ctypes.c_int * 8), ("offset", ctypes.c_size_t), ("total_size", ctypes.c_size_t)]


def _ref_desc(t, shape, strides):
    d = RefDesc()
    d.data = t.data_ptr()
    d.ndims = len(shape)
    for i, (s, st) in enumerate(zip(shape, strides)):
        d.shape[i] = s
        d.strides[i] = st
    d.offset = 0
    d.total_size = int(np.prod(shape))
    return d


def _dev(a):
    a = np.ascontiguousarray(a)
    if a.dtype == np.float16:
        return torch.from_numpy(a.view(np.int16)).cuda().view(torch.float16)
    return torch.from_numpy(a).cuda()


def _host(t):
    return t.cpu().numpy()


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def test_reference_float16_int8_int64_names(acd):
    lib = acd.lib()
    rng = np.random.default_rng(7)
    n = 10007
    a, b = _half_data(rng, (n,)), _half_data(rng, (n,))
    da, db = _dev(a), _dev(b)
    dr = torch.empty(n, dtype=torch.float16, device="cuda")
    N = ctypes.c_size_t(n)
    for name, op in [("add", "add"), ("sub", "sub"), ("mul", "mul"), ("div", "div")]:
        getattr(lib, "tensor_%s_float16" % name)(_p(dr), _p(da), _p(db), N)
        assert_exact(_bits(_host(dr)), _bits(oracle.binary(op, a, b)), "tensor_%s_float16" % name)
    lib.tensor_scalar_add_float16(_p(dr), _p(da), ctypes.c_float(0.3), N)
    assert_exact(_bits(_host(dr)), _bits(oracle.scalar("add", a, float(np.float32(0.3)))),
                 "tensor_scalar_add_float16")
    lib.tensor_scalar_mul_float16(_p(dr), _p(da), ctypes.c_float(-1.5), N)
    assert_exact(_bits(_host(dr)), _bits(oracle.scalar("mul", a, -1.5)), "tensor_scalar_mul_float16")
    # strided: out = a^T + b^T on 2-D views given by reference descriptors
    A, B = _half_data(rng, (30, 20)), _half_data(rng, (30, 20))
    dA, dB = _dev(A.reshape(-1, order="F")), _dev(B.reshape(-1, order="F"))
    dO = torch.empty(600, dtype=torch.float16, device="cuda")
    o, x, y = _ref_desc(dO, (20, 30), (1, 20)), _ref_desc(dA, (20, 30), (30, 1)), _ref_desc(dB, (20, 30), (30, 1))
    lib.tensor_add_strided_float16(ctypes.byref(o), ctypes.byref(x), ctypes.byref(y))
    assert_exact(_bits(_host(dO)), _bits(oracle.binary("add", A.T, B.T).reshape(-1, order="F")),
                 "tensor_add_strided_float16")
    lib.tensor_div_strided_float16(ctypes.byref(o), ctypes.byref(x), ctypes.byref(y))
    assert_exact(_bits(_host(dO)), _bits(oracle.binary("div", A.T, B.T).reshape(-1, order="F")),
                 "tensor_div_strided_float16")
    i8a, i8b = _i8_data(rng, (n,)), _i8_data(rng, (n,))
    di, dj, dk = _dev(i8a), _dev(i8b), torch.empty(n, dtype=torch.int8, device="cuda")
    lib.tensor_add_int8(_p(dk), _p(di), _p(dj), N)
    assert_exact(_host(dk), oracle.binary("add", i8a, i8b), "tensor_add_int8")
    I8 = _i8_data(rng, (30, 20))
    dI = _dev(I8.reshape(-1, order="F"))
    dK = torch.empty(600, dtype=torch.int8, device="cuda")
    oi, xi = _ref_desc(dK, (20, 30), (1, 20)), _ref_desc(dI, (20, 30), (30, 1))
    lib.tensor_add_strided_int8(ctypes.byref(oi), ctypes.byref(xi), ctypes.byref(xi))
    assert_exact(_host(dK), oracle.binary("add", I8.T, I8.T).reshape(-1, order="F"), "tensor_add_strided_int8")
    # the reference's placeholders return 0; these are the sums
    lib.tensor_sum_float16.restype = ctypes.c_float
    big = (rng.normal(0, 10, (1 << 20) + 3)).astype(np.float16)
    dbig = _dev(big)
    s = lib.tensor_sum_float16(_p(dbig), ctypes.c_size_t(big.size))
    assert s == np.float32(oracle.reduce("sum", big)), "tensor_sum_float16"
    lib.tensor_sum_int64.restype = ctypes.c_int64
    v = rng.integers(-2 ** 40, 2 ** 40, (1 << 20) + 5, dtype=np.int64)
    v[0] = 2 ** 53 + 1  # beyond float64's exact integers
    dv = _dev(v)
    assert lib.tensor_sum_int64(_p(dv), ctypes.c_size_t(v.size)) == int(v.sum())


def test_contraction_names(acd):
    lib = acd.lib()
    rng = np.random.default_rng(8)
    M, N, K = 70, 45, 33
    for dt, tol in ((np.float32, 1e-5), (np.float64, 1e-12)):
        A = rng.normal(size=(M, K)).astype(dt)
        B = rng.normal(size=(K, N)).astype(dt)
        v = rng.normal(size=K).astype(dt)
        w = rng.normal(size=M).astype(dt)
        sfx = "float32" if dt == np.float32 else "float64"
        # device copies are kept in names: a temporary's memory could be
        # reused by the next allocation before the launcher runs
        dA, dB = _dev(A.reshape(-1, order="F")), _dev(B.reshape(-1, order="F"))
        dv, dw = _dev(v), _dev(w)
        dC = torch.empty(M * N, dtype=torch.float32 if dt == np.float32 else torch.float64, device="cuda")
        getattr(lib, "tensor_matmul_" + sfx)(_p(dC), _p(dA), _p(dB), ctypes.c_size_t(M), ctypes.c_size_t(N),
                                             ctypes.c_size_t(K))
        ref = A.astype(np.float64) @ B.astype(np.float64)
        scale = np.abs(A).astype(np.float64) @ np.abs(B).astype(np.float64)
        err = np.abs(_host(dC).reshape((M, N), order="F") - ref)
        assert np.all(err <= tol * scale), "matmul " + sfx
        dr = torch.empty(M, dtype=dC.dtype, device="cuda")
        getattr(lib, "tensor_matvec_" + sfx)(_p(dr), _p(dA), _p(dv), ctypes.c_size_t(M), ctypes.c_size_t(K))
        assert np.all(np.abs(_host(dr) - A.astype(np.float64) @ v) <= tol * (np.abs(A) @ np.abs(v))), "matvec"
        dq = torch.empty(K, dtype=dC.dtype, device="cuda")
        getattr(lib, "tensor_vecmat_" + sfx)(_p(dq), _p(dw), _p(dA), ctypes.c_size_t(M), ctypes.c_size_t(K))
        assert np.all(np.abs(_host(dq) - w.astype(np.float64) @ A) <= tol * (np.abs(w) @ np.abs(A))), "vecmat"
        do = torch.empty(M * K, dtype=dC.dtype, device="cuda")
        getattr(lib, "tensor_outer_product_" + sfx)(_p(do), _p(dw), _p(dv), ctypes.c_size_t(M),
                                                    ctypes.c_size_t(K))
        assert_exact(_host(do).reshape((M, K), order="F"), np.outer(w, v).astype(dt), "outer " + sfx)
    # float16 (float32 accumulation, one rounding): within 2 half ulp of the float64 product
    A = (rng.normal(size=(M, K)) / 4).astype(np.float16)
    B = (rng.normal(size=(K, N)) / 4).astype(np.float16)
    dC = torch.empty(M * N, dtype=torch.float16, device="cuda")
    dA, dB = _dev(A.reshape(-1, order="F")), _dev(B.reshape(-1, order="F"))
    lib.tensor_matmul_float16(_p(dC), _p(dA), _p(dB), ctypes.c_size_t(M), ctypes.c_size_t(N), ctypes.c_size_t(K))
    ref = A.astype(np.float64) @ B.astype(np.float64)
    got = _host(dC).reshape((M, N), order="F").astype(np.float64)
    assert np.all(np.abs(got - ref) <= 2 * np.spacing(np.abs(ref).astype(np.float16)).astype(np.float64) + 1e-6)
    v = (rng.normal(size=K) / 4).astype(np.float16)
    dr = torch.empty(M, dtype=torch.float16, device="cuda")
    dv = _dev(v)
    lib.tensor_matvec_float16(_p(dr), _p(dA), _p(dv), ctypes.c_size_t(M), ctypes.c_size_t(K))
    ref = A.astype(np.float64) @ v.astype(np.float64)
    assert np.all(np.abs(_host(dr).astype(np.float64) - ref) <= 2 * np.spacing(np.abs(ref).astype(np.float16)) + 1e-6)


def test_log_domain_error(acd):
    """tensor_log_unified rejects non-positive input (src/TensorMath.cpp:167-174);
    NaN is not rejected, and the launcher name itself does not check."""
    x = acd.as_tensor(np.array([1.0, 2.0, 0.0, 3.0]), dtype="double")
    with pytest.raises(ValueError, match="log\\(\\) domain error: input contains non-positive values"):
        acd.log(x)
    with pytest.raises(ValueError, match="domain error"):
        acd.log(acd.as_tensor(np.array([-1e-30, 5.0], dtype=np.float32), dtype="float"))
    y = acd.log(acd.as_tensor(np.array([1.0, np.nan, 4.0]), dtype="double")).as_array()
    assert y[0] == 0.0 and np.isnan(y[1]) and abs(y[2] - np.log(4.0)) <= 2 * np.spacing(np.log(4.0))
    with pytest.raises(ValueError, match="Only natural logarithm"):
        acd.log(x, base=10)
