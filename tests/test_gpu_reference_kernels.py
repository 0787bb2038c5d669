"""Pins the oracle against the reference itself: the reference's own CUDA
launchers (acediaR src/kernels/tensor_ops.cu and tensor_kernels.cu, built
unmodified into oracle/_ref/libacediar_ref.so by oracle/ref.mk) run on small
seeded inputs, where the reference's known defects (65535-block reduction
cap, one-block argmin, placeholder axis variance) do not apply.  Each result
is compared with the oracle and with this library's CUDA path.
"""
import ctypes
import os

import numpy as np
import pytest
import torch

import oracle
from helpers import assert_exact, assert_rel, assert_ulp

pytestmark = pytest.mark.gpu
REF_SO = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref",
                      "libacediar_ref.so")


@pytest.fixture(scope="module")
def ref():
    if not os.path.exists(REF_SO):
        pytest.fail("oracle/_ref/libacediar_ref.so missing: build it with `make -C oracle -f ref.mk`")
    lib = ctypes.CDLL(REF_SO)
    for name, rt in [("tensor_sum_float64", ctypes.c_double), ("tensor_var_float64", ctypes.c_double),
                     ("tensor_sum_float32", ctypes.c_float), ("tensor_max_float64", ctypes.c_double),
                     ("tensor_argmax_float64", ctypes.c_int64), ("tensor_argmin_float32", ctypes.c_int64)]:
        getattr(lib, name).restype = rt
    return lib


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _c1_inputs(n=1 << 16):
    rng = np.random.default_rng(42)
    return rng.uniform(0, 1, n), rng.standard_normal(n)


def test_reference_elementwise_chain_f64(ref, acd):
    a, b = _c1_inputs()
    da, db = _dev(a), _dev(b)
    out = torch.empty_like(da)
    n = ctypes.c_size_t(a.size)
    ta, tb = acd.as_tensor(a, dtype="double"), acd.as_tensor(b, dtype="double")
    for name, args, ours, orc in [
            ("tensor_add_float64", (da, db), lambda: ta + tb, lambda: oracle.binary("add", a, b)),
            ("tensor_mul_float64", (da, db), lambda: ta * tb, lambda: oracle.binary("mul", a, b)),
            ("tensor_exp_float64", (da,), lambda: acd.exp(ta), lambda: oracle.unary("exp", a)),
            ("tensor_sigmoid_float64", (db,), lambda: acd.sigmoid(tb), lambda: oracle.unary("sigmoid", b)),
            ("tensor_sqrt_float64", (da,), lambda: acd.sqrt(ta), lambda: oracle.unary("sqrt", a))]:
        getattr(ref, name)(_p(out), *[_p(x) for x in args], n)
        torch.cuda.synchronize()
        r = out.cpu().numpy()
        assert_ulp(r, orc(), 2, name + ": reference vs oracle")
        assert_exact(ours().as_array(), r, name + ": this library vs reference")


def test_reference_reductions_f64(ref, acd):
    a, b = _c1_inputs()
    c = a + b
    dc = _dev(c)
    n = ctypes.c_size_t(c.size)
    assert_rel(ref.tensor_sum_float64(_p(dc), n), oracle.reduce("sum", c), 1e-12, "sum ref vs oracle")
    assert_rel(ref.tensor_var_float64(_p(dc), n), oracle.reduce("var", c), 1e-10, "var ref vs oracle")
    assert ref.tensor_max_float64(_p(dc), n) == oracle.reduce("max", c)
    assert ref.tensor_argmax_float64(_p(dc), n) == oracle.arg_reduce("argmax", c)
    tc = acd.as_tensor(c, dtype="double")
    assert acd.which_max(tc) == ref.tensor_argmax_float64(_p(dc), n)
    assert_rel(acd.sum(tc), ref.tensor_sum_float64(_p(dc), n), 1e-12, "sum ours vs ref")


def test_reference_small_f32_reductions(ref, acd):
    rng = np.random.default_rng(7)
    x = rng.normal(size=200).astype(np.float32)  # argmin scans one block: n <= 256
    x[[17, 99]] = x.min() - 1.0
    dx = _dev(x)
    n = ctypes.c_size_t(x.size)
    assert ref.tensor_argmin_float32(_p(dx), n) == oracle.arg_reduce("argmin", x) == 18
    assert_rel(ref.tensor_sum_float32(_p(dx), n), oracle.reduce("sum", x), 1e-5, "f32 sum")
    assert acd.which_min(acd.as_tensor(x, dtype="float")) == 18


def test_reference_axis_sum_and_argmax(ref, acd):
    rng = np.random.default_rng(8)
    x = rng.normal(size=(40, 30, 5)).astype(np.float32)
    x[:, 3, :] = x[:, 11, :]  # ties along axis 2
    dx = _dev(x.reshape(-1, order="F"))
    meta = lambda v: torch.tensor(v, dtype=torch.int32, device="cuda")
    st, sh, ax = meta([1, 40, 1200]), meta([40, 30, 5]), meta([1])
    ost = meta([1, 40])
    out = torch.empty(200, dtype=torch.float32, device="cuda")
    ref.tensor_axis_sum_float32(_p(out), _p(dx), _p(st), _p(sh), _p(ost), _p(ax), 1, 3, ctypes.c_size_t(200))
    r = out.cpu().numpy()
    # the reference accumulates in float32: its error is bounded by n*eps*sum|x|
    bound = 30 * np.finfo(np.float32).eps * np.abs(x).sum(axis=1).reshape(-1, order="F")
    exp = oracle.reduce("sum", x, [1]).reshape(-1, order="F")
    assert np.all(np.abs(r - exp) <= bound), "axis sum ref vs oracle"
    ours = acd.tensor_sum(acd.as_tensor(x, dtype="float"), axis=[2]).as_array().reshape(-1, order="F")
    assert_rel(ours, exp, 1e-5, "axis sum ours vs oracle", atol=1e-7)
    assert np.all(np.abs(ours - r) <= bound), "axis sum ours vs ref"
    idx = torch.empty(200, dtype=torch.int64, device="cuda")
    ref.tensor_axis_argmax_float32(_p(idx), _p(dx), _p(st), _p(sh), _p(ost), _p(ax), 1, 3, ctypes.c_size_t(200))
    ri = idx.cpu().numpy()
    assert_exact(ri, oracle.arg_reduce("argmax", x, 1, one_based=False).reshape(-1, order="F"),
                 "axis argmax ref vs oracle")
    oi = acd.argmax(acd.as_tensor(x, dtype="float"), axis=2).as_array().reshape(-1, order="F")
    assert_exact(oi - 1, ri, "axis argmax ours (1-based) vs ref (0-based)")


def test_reference_softmax_copy_compare_broadcast(ref, acd):
    rng = np.random.default_rng(9)
    x = rng.normal(size=1000)
    dx, out = _dev(x), torch.empty(1000, dtype=torch.float64, device="cuda")
    ref.tensor_softmax_float64(_p(out), _p(dx), ctypes.c_size_t(1000))
    torch.cuda.synchronize()
    r = out.cpu().numpy()
    assert_rel(r, oracle.softmax(x), 1e-12, "softmax ref vs oracle")
    assert_rel(acd.softmax(acd.as_tensor(x, dtype="double")).as_array(), r, 1e-12, "softmax ours vs ref")

    X = rng.normal(size=(64, 48)).astype(np.float32)
    dX = _dev(X.reshape(-1, order="F"))
    o = torch.empty(64 * 48, dtype=torch.float32, device="cuda")
    ints = lambda v: (ctypes.c_int * len(v))(*v)
    ref.tensor_strided_copy_float32(_p(o), _p(dX), ints([64, 1]), ints([48, 64]), 2, ctypes.c_size_t(64 * 48))
    torch.cuda.synchronize()
    assert_exact(o.cpu().numpy(), oracle.copy(oracle.View(X.reshape(-1, order="F"), (48, 64), (64, 1))).reshape(
        -1, order="F"), "strided copy ref vs oracle")

    Y = rng.normal(size=(64, 48)).astype(np.float32)
    dY = _dev(Y.reshape(-1, order="F"))
    ref.tensor_gt_float32(_p(o), _p(dX), _p(dY), ctypes.c_size_t(64 * 48))
    torch.cuda.synchronize()
    assert_exact(o.cpu().numpy(), (X > Y).astype(np.float32).reshape(-1, order="F"), "gt ref")
    r1 = rng.normal(size=(1, 48)).astype(np.float32)
    dr = _dev(r1.reshape(-1, order="F"))
    ref.tensor_add_broadcast_float32(_p(o), _p(dX), _p(dr), ints([1, 64]), ints([0, 1]), ints([48, 1]),
                                     ints([64, 48]), 2, ctypes.c_size_t(64 * 48))
    torch.cuda.synchronize()
    rb = o.cpu().numpy()
    assert_exact(rb, oracle.binary("add", X, r1).reshape(-1, order="F"), "broadcast add ref vs oracle")
    ours = (acd.as_tensor(X, dtype="float") + acd.as_tensor(r1, dtype="float")).as_array().reshape(-1, order="F")
    assert_exact(ours, rb, "broadcast add ours vs ref")
