"""The reference's launcher names (include/acediar_launchers.h) called through
ctypes on device buffers, as the reference's Rcpp modules call them."""
import ctypes

import numpy as np
import pytest
import torch

import oracle
from helpers import assert_exact, assert_rel, assert_ulp

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib(acd):
    return acd.lib()


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def test_contiguous_elementwise_names(lib):
    rng = np.random.default_rng(0)
    a = rng.normal(size=10001).astype(np.float32)
    b = rng.normal(size=10001).astype(np.float32)
    da, db, dr = _dev(a), _dev(b), torch.empty(10001, dtype=torch.float32, device="cuda")
    lib.tensor_add_float32(_p(dr), _p(da), _p(db), ctypes.c_size_t(a.size))
    assert_exact(dr.cpu().numpy(), a + b, "tensor_add_float32")
    lib.tensor_gt_float32(_p(dr), _p(da), _p(db), ctypes.c_size_t(a.size))
    assert_exact(dr.cpu().numpy(), (a > b).astype(np.float32), "tensor_gt_float32 (0/1 in input dtype)")
    lib.tensor_exp_float32(_p(dr), _p(da), ctypes.c_size_t(a.size))
    assert_ulp(dr.cpu().numpy(), oracle.unary("exp", a), 2, "tensor_exp_float32")
    lib.tensor_scalar_div_float32(_p(dr), _p(da), ctypes.c_float(3.0), ctypes.c_size_t(a.size))
    assert_exact(dr.cpu().numpy(), a / np.float32(3.0), "tensor_scalar_div_float32")


def test_reduction_names_return_host_scalars(lib):
    rng = np.random.default_rng(1)
    x = rng.normal(size=(1 << 25) + 3)  # beyond the reference's 65535*256 element cap
    dx = _dev(x)
    lib.tensor_sum_float64.restype = ctypes.c_double
    lib.tensor_var_float64.restype = ctypes.c_double
    lib.tensor_argmax_float64.restype = ctypes.c_int64
    lib.tensor_argmin_float64.restype = ctypes.c_int64
    n = ctypes.c_size_t(x.size)
    assert_rel(lib.tensor_sum_float64(_p(dx), n), oracle.reduce("sum", x), 1e-12, "sum")
    assert_rel(lib.tensor_var_float64(_p(dx), n), oracle.reduce("var", x), 1e-12, "var")
    assert lib.tensor_argmax_float64(_p(dx), n) == oracle.arg_reduce("argmax", x)
    assert lib.tensor_argmin_float64(_p(dx), n) == oracle.arg_reduce("argmin", x)


def test_axis_names_with_device_metadata(lib):
    rng = np.random.default_rng(2)
    x = rng.normal(size=(40, 30, 5)).astype(np.float32)
    dx = _dev(x.reshape(-1, order="F"))
    meta = lambda v: torch.tensor(v, dtype=torch.int32, device="cuda")
    st, sh, ax = meta([1, 40, 1200]), meta([40, 30, 5]), meta([1])
    out = torch.empty(40 * 5, dtype=torch.float32, device="cuda")
    lib.tensor_axis_sum_float32(_p(out), _p(dx), _p(st), _p(sh), _p(st), _p(ax), 1, 3, ctypes.c_size_t(200))
    assert_rel(out.cpu().numpy(), oracle.reduce("sum", x, [1]).reshape(-1, order="F"), 1e-5, "axis sum")
    lib.tensor_axis_var_float32(_p(out), _p(dx), _p(st), _p(sh), _p(st), _p(ax), 1, 3, ctypes.c_size_t(200))
    assert_rel(out.cpu().numpy(), oracle.reduce("var", x, [1]).reshape(-1, order="F"), 1e-5, "axis var")
    idx = torch.empty(200, dtype=torch.int64, device="cuda")
    lib.tensor_axis_argmax_float32(_p(idx), _p(dx), _p(st), _p(sh), _p(st), _p(ax), 1, 3, ctypes.c_size_t(200))
    assert_exact(idx.cpu().numpy(), oracle.arg_reduce("argmax", x, 1, one_based=False).reshape(-1, order="F"),
                 "axis argmax (0-based)")


def test_broadcast_and_strided_copy_names(lib):
    rng = np.random.default_rng(3)
    X = rng.normal(size=(64, 48))
    r = rng.normal(size=(1, 48))
    dX, dr = _dev(X.reshape(-1, order="F")), _dev(r.reshape(-1, order="F"))
    out = torch.empty(64 * 48, dtype=torch.float64, device="cuda")
    ints = lambda v: (ctypes.c_int * len(v))(*v)
    lib.tensor_add_broadcast_float64(_p(out), _p(dX), _p(dr), ints([1, 64]), ints([0, 1]), ints([48, 1]),
                                     ints([64, 48]), 2, ctypes.c_size_t(64 * 48))
    assert_exact(out.cpu().numpy(), (X + r).reshape(-1, order="F"), "tensor_add_broadcast_float64")
    # contiguous(transpose): strides of the 48x64 transposed view are (64, 1)
    lib.tensor_strided_copy_float64(_p(out), _p(dX), ints([64, 1]), ints([48, 64]), 2, ctypes.c_size_t(64 * 48))
    assert_exact(out.cpu().numpy(), X.T.reshape(-1, order="F"), "tensor_strided_copy_float64")


def test_softmax_name_whole_tensor(lib):
    rng = np.random.default_rng(4)
    x = rng.normal(size=5000).astype(np.float32)
    dx, out = _dev(x), torch.empty(5000, dtype=torch.float32, device="cuda")
    lib.tensor_softmax_float32(_p(out), _p(dx), ctypes.c_size_t(5000))
    assert_rel(out.cpu().numpy(), oracle.softmax(x), 1e-5, "tensor_softmax_float32")
