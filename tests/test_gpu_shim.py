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


def test_mutation_and_assembly_names(lib):
    """Slice/mask assignment and concat/stack/repeat/pad through the names
    src/TensorMutation.cpp calls, host metadata as it passes them."""
    rng = np.random.default_rng(5)
    ints = lambda v: (ctypes.c_int * len(v))(*v)
    m = np.arange(1, 21, dtype=np.float32).reshape(4, 5, order="F")
    dm = _dev(m.reshape(-1, order="F"))
    lib.tensor_slice_set_scalar_float32(_p(dm), ctypes.c_double(99.0), ints([1, 1]), ints([2, 3]), ints([1, 4]),
                                        2, ctypes.c_size_t(6))
    e = m.copy()
    e[1:3, 1:4] = 99
    lib.tensor_slice_add_scalar_float32(_p(dm), ctypes.c_double(0.5), ints([0, 0]), ints([1, 5]), ints([1, 4]),
                                        2, ctypes.c_size_t(5))
    e[0, :] += np.float32(0.5)
    assert_exact(dm.cpu().numpy(), e.reshape(-1, order="F"), "slice set / add scalar")
    src = rng.normal(size=(2, 2))
    d64 = _dev(np.zeros(20))
    dsrc = _dev(src.reshape(-1, order="F"))
    lib.tensor_slice_set_tensor_float64(_p(d64), _p(dsrc), ints([2, 3]), ints([2, 2]), ints([1, 4]), ints([1, 2]),
                                        2, ctypes.c_size_t(4))
    z = np.zeros((4, 5))
    z[2:4, 3:5] = src
    assert_exact(d64.cpu().numpy(), z.reshape(-1, order="F"), "tensor_slice_set_tensor_float64")
    mask = (rng.random(20) < 0.5).astype(np.uint8)
    dmask = _dev(mask)  # kept alive across the call
    lib.tensor_mask_set_scalar_float64(_p(d64), _p(dmask), ctypes.c_double(-1.0), ctypes.c_size_t(20))
    zz = z.reshape(-1, order="F").copy()
    zz[mask.astype(bool)] = -1
    assert_exact(d64.cpu().numpy(), zz, "tensor_mask_set_scalar_float64")

    a = rng.normal(size=(2, 3)).astype(np.float32)
    b = rng.normal(size=(3, 3)).astype(np.float32)
    da, db = _dev(a.reshape(-1, order="F")), _dev(b.reshape(-1, order="F"))
    out = torch.empty(15, dtype=torch.float32, device="cuda")
    ptrs = (ctypes.c_void_p * 2)(da.data_ptr(), db.data_ptr())
    lib.launch_concat_float32(_p(out), ptrs, ints([2, 3]), 2, ints([1, 5]), ints([1, 2, 1, 3]), ints([5, 3]), 2, 0,
                              ctypes.c_size_t(15))
    assert_exact(out.cpu().numpy(), np.concatenate([a, b], 0).reshape(-1, order="F"), "launch_concat_float32")
    c = rng.normal(size=(2, 3)).astype(np.float32)
    dc = _dev(c.reshape(-1, order="F"))
    out2 = torch.empty(12, dtype=torch.float32, device="cuda")
    ptrs = (ctypes.c_void_p * 2)(da.data_ptr(), dc.data_ptr())
    lib.launch_stack_float32(_p(out2), ptrs, 2, ints([1, 2]), ints([2, 3, 2]), 3, 2, ctypes.c_size_t(12))
    assert_exact(out2.cpu().numpy(), np.stack([a, c], 2).reshape(-1, order="F"), "launch_stack_float32")
    out3 = torch.empty(24, dtype=torch.float32, device="cuda")
    lib.launch_repeat_float32(_p(out3), _p(da), ints([1, 2]), ints([2, 2]), ints([2, 3]), ints([4, 6]), 2,
                              ctypes.c_size_t(24))
    assert_exact(out3.cpu().numpy(), oracle.repeat(a, (2, 2)).reshape(-1, order="F"), "launch_repeat_float32")
    out4 = torch.empty(4 * 7, dtype=torch.float32, device="cuda")
    for mode, name in [(0, "constant"), (1, "reflect"), (2, "replicate")]:
        lib.launch_pad_float32(_p(out4), _p(da), ints([1, 2]), ints([2, 3]), ints([1, 2]), ints([1, 2]),
                               ints([4, 7]), 2, ctypes.c_float(3.0), mode, ctypes.c_size_t(28))
        assert_exact(out4.cpu().numpy(), oracle.pad(a, [1, 2], [1, 2], name, 3.0).reshape(-1, order="F"),
                     "launch_pad_float32 " + name)
