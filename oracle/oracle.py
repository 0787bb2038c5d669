"""ctypes wrapper of the CPU oracle (oracle.c) — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module; the product never does.

Tensors are given as (buffer, shape, strides, offset) views over a 1-D numpy
buffer in column-major element strides, or as numpy arrays, which are taken
as logical R arrays (their column-major order is the storage order).  Results
are numpy arrays of the logical shape.

The broadcast rule is restated here from the reference (src/gpuTensor.h:248-340,
src/TensorArithmetic.cpp:240-292): the shorter shape is tried at every offset
from the leading side and the first fit wins.
"""
import concurrent.futures as cf
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None
_LIB_MT = None

DT = {np.dtype(np.float32): 0, np.dtype(np.float64): 1, np.dtype(np.int32): 2, np.dtype(np.int64): 3,
      np.dtype(np.uint8): 4, np.dtype(np.bool_): 4, np.dtype(np.float16): 5, np.dtype(np.int8): 6}
UNARY = {n: i for i, n in enumerate(
    ["exp", "log", "sqrt", "abs", "floor", "ceil", "round", "erf", "tanh", "sigmoid", "relu", "sin", "cos",
     "neg", "square", "copy"])}
BINARY = {n: i for i, n in enumerate(
    ["add", "sub", "mul", "div", "max", "min", "pow", "gt", "lt", "eq", "ne", "ge", "le", "rsub", "rdiv"])}
REDUCE = {n: i for i, n in enumerate(["sum", "mean", "max", "min", "prod", "var", "count", "any", "all"])}
COMPARE = {"gt", "lt", "eq", "ne", "ge", "le"}

_i64p = ctypes.POINTER(ctypes.c_int64)


def build():
    """Compiles liboracle*.so with the Makefile next to this file."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _LIB
    if _LIB is None:
        path = os.path.join(HERE, "liboracle.so")
        if not os.path.exists(path):
            build()
        _LIB = ctypes.CDLL(path)
    return _LIB


def lib_mt():
    global _LIB_MT
    if _LIB_MT is None:
        path = os.path.join(HERE, "liboracle_mt.so")
        if not os.path.exists(path):
            build()
        _LIB_MT = ctypes.CDLL(path)
    return _LIB_MT


class View:
    """A strided view over a 1-D numpy buffer (column-major element strides)."""

    def __init__(self, buf, shape, strides=None, offset=0):
        self.buf = np.ascontiguousarray(buf).reshape(-1)
        self.shape = tuple(int(s) for s in shape)
        if strides is None:
            strides, acc = [], 1
            for s in self.shape:
                strides.append(acc)
                acc *= s
        self.strides = tuple(int(s) for s in strides)
        self.offset = int(offset)

    @staticmethod
    def of(x):
        if isinstance(x, View):
            return x
        a = np.asarray(x)
        return View(a.reshape(-1, order="F") if a.ndim else a.reshape(1), a.shape if a.ndim else (1,))

    @property
    def dtype(self):
        return self.buf.dtype

    def ptr(self):
        return ctypes.c_void_p(self.buf.ctypes.data + self.offset * self.buf.itemsize)


def _arr(v):
    return (ctypes.c_int64 * max(1, len(v)))(*v)


def _shape_out(shape):
    return shape if len(shape) else (1,)


def _result(flat, shape):
    return flat.reshape(_shape_out(shape), order="F")


def broadcast_shape(a, b):
    """acediaR broadcast shape (leading-side offset sweep); raises ValueError."""
    a, b = tuple(a), tuple(b)
    if len(a) == len(b):
        offs = [(a, b, 0)]
    else:
        short, long_ = (a, b) if len(a) < len(b) else (b, a)
        offs = [(short, long_, o) for o in range(len(long_) - len(short) + 1)]
    for short, long_, off in offs:
        ok = True
        for i in range(len(long_)):
            ds = short[i - off] if off <= i < off + len(short) else 1
            if ds != long_[i] and ds != 1 and long_[i] != 1:
                ok = False
                break
        if ok:
            return tuple(max(short[i - off] if off <= i < off + len(short) else 1, long_[i])
                         for i in range(len(long_)))
    raise ValueError("Tensor shapes are not broadcastable")


def broadcast_strides(shape, strides, out_shape):
    for off in range(len(out_shape) - len(shape) + 1):
        if all(s == d or s == 1 or d == 1 for s, d in zip(shape, out_shape[off:off + len(shape)])):
            st = [0] * len(out_shape)
            for i, (s, sd) in enumerate(zip(shape, strides)):
                st[off + i] = 0 if s == 1 else sd
            return tuple(st)
    raise ValueError("Shape mismatch in broadcast stride calculation")


# ---------------------------------------------------------------------------
def _ranges(n, threads, fn):
    """Runs fn(lo, hi) over `threads` consecutive output ranges.  ctypes
    releases the GIL inside the C call, so the ranges run in parallel."""
    threads = max(1, min(int(threads), n)) if n > 0 else 1
    if threads == 1:
        fn(0, n)
        return
    bounds = [(n * k // threads, n * (k + 1) // threads) for k in range(threads)]
    with cf.ThreadPoolExecutor(threads) as ex:
        list(ex.map(lambda b: fn(*b), bounds))


def default_threads():
    return os.cpu_count() or 1


def unary(op, x, threads=1):
    v = View.of(x)
    n = int(np.prod(v.shape))
    out = np.empty(n, dtype=v.dtype)
    sh, st = _arr(v.shape), _arr(v.strides)
    _ranges(n, threads, lambda lo, hi: lib().orc_unary_range(
        UNARY[op], DT[v.dtype], v.ptr(), len(v.shape), sh, st, out.ctypes.data_as(ctypes.c_void_p),
        ctypes.c_int64(lo), ctypes.c_int64(hi)))
    return _result(out, v.shape)


def copy(x):
    return unary("copy", x)


def binary(op, a, b, out_dtype=None, threads=1):
    va, vb = View.of(a), View.of(b)
    shape = broadcast_shape(va.shape, vb.shape)
    sa = broadcast_strides(va.shape, va.strides, shape)
    sb = broadcast_strides(vb.shape, vb.strides, shape)
    odt = np.dtype(out_dtype) if out_dtype is not None else (np.dtype(np.uint8) if op in COMPARE else va.dtype)
    n = int(np.prod(shape))
    out = np.empty(n, dtype=odt)
    csa, csb, csh = _arr(sa), _arr(sb), _arr(shape)
    _ranges(n, threads, lambda lo, hi: lib().orc_binary_range(
        BINARY[op], DT[va.dtype], va.ptr(), csa, vb.ptr(), csb, len(shape), csh, DT[odt],
        out.ctypes.data_as(ctypes.c_void_p), ctypes.c_int64(lo), ctypes.c_int64(hi)))
    return _result(out, shape)


def scalar(op, x, s, out_dtype=None, threads=1):
    v = View.of(x)
    odt = np.dtype(out_dtype) if out_dtype is not None else (np.dtype(np.uint8) if op in COMPARE else v.dtype)
    n = int(np.prod(v.shape))
    out = np.empty(n, dtype=odt)
    sh, st = _arr(v.shape), _arr(v.strides)
    _ranges(n, threads, lambda lo, hi: lib().orc_scalar_range(
        BINARY[op], DT[v.dtype], v.ptr(), len(v.shape), sh, st, ctypes.c_double(s), DT[odt],
        out.ctypes.data_as(ctypes.c_void_p), ctypes.c_int64(lo), ctypes.c_int64(hi)))
    return _result(out, v.shape)


def convert(x, to_dtype):
    """as.<dtype>(x): to_dtype is a numpy dtype (float32, float64, int32, int64, bool)."""
    v = View.of(x)
    to = np.dtype(to_dtype)
    out = np.empty(int(np.prod(v.shape)), dtype=np.uint8 if to == np.bool_ else to)
    lib().orc_convert(DT[v.dtype], DT[to], v.ptr(), len(v.shape), _arr(v.shape), _arr(v.strides),
                      out.ctypes.data_as(ctypes.c_void_p))
    if to == np.bool_:
        out = out.view(np.bool_)
    return _result(out, v.shape)


def rand(n, dtype, dist, a, b, seed, offset=0):
    """Counter-based random values (Philox4x32-10): dist "uniform" on [a, b)
    or "normal" with mean a and sd b; element i uses counter offset + i."""
    dt = np.dtype(dtype)
    out = np.empty(int(n), dtype=dt)
    lib().orc_rand(DT[dt], 0 if dist == "uniform" else 1, ctypes.c_double(a), ctypes.c_double(b),
                   ctypes.c_uint64(seed), ctypes.c_uint64(offset), ctypes.c_int64(int(n)),
                   out.ctypes.data_as(ctypes.c_void_p))
    return out


# ---- assembly (pure data movement, restated with numpy on logical arrays) ----
def concat(arrays, axis):
    """concat_kernel (src/kernels/tensor_kernels.cu:298-341): the inputs in
    order along `axis` (0-based)."""
    return np.concatenate([np.asarray(a) for a in arrays], axis=axis)


def stack(arrays, axis):
    """stack_kernel (src/kernels/tensor_kernels.cu:343-379): a new axis at
    position `axis` (0-based) indexing the inputs."""
    return np.stack([np.asarray(a) for a in arrays], axis=axis)


def repeat(x, reps):
    """repeat_kernel (src/kernels/tensor_kernels.cu:381-413): out(c) =
    in(c // reps) on every axis."""
    x = np.asarray(x)
    for d, r in enumerate(reps):
        x = np.repeat(x, int(r), axis=d)
    return x


def pad(x, before, after, mode="constant", value=0.0):
    """pad_kernel (src/kernels/tensor_kernels.cu:415-466): constant, reflect
    with the edge included (numpy's "symmetric"), replicate ("edge").  The
    constant is converted to the tensor dtype as as.<dtype> would."""
    x = np.asarray(x)
    width = [(int(b), int(a)) for b, a in zip(before, after)]
    if mode == "constant":
        v = convert(np.array([value], dtype=np.float64), x.dtype if x.dtype != np.bool_ else np.bool_)[0]
        return np.pad(x, width, mode="constant", constant_values=v)
    return np.pad(x, width, mode={"reflect": "symmetric", "replicate": "edge"}[mode])


def diff(x, lag=1, differences=1):
    """diff.gpuTensor (R/gpuTensor.R:2289-2333): base R's
    diff(as.vector(x), lag, differences) on the column-major elements; for a
    tensor of two or more axes the result is recycled (rep_len) to the
    tensor's size and reshaped to its shape.  One rounding per difference."""
    x = np.asarray(x)
    if lag < 1:
        raise ValueError("lag must be positive")
    if differences < 1:
        raise ValueError("differences must be positive")
    v = x.reshape(-1, order="F")
    for _ in range(int(differences)):
        if v.size <= lag:
            raise ValueError("diff of single element tensor results in empty result - not supported by tensor system")
        v = v[lag:] - v[:-lag]
    if x.ndim <= 1:
        return v
    return np.resize(v, x.size).reshape(x.shape, order="F")


def gauss_chain(x, p=0.5, threads=1):
    """x*p + exp(-(x^2)) with one rounding per R operator."""
    a = np.ascontiguousarray(np.asarray(x).reshape(-1, order="F"))
    out = np.empty_like(a)
    if threads > 1:
        lib_mt().orc_gauss_chain_mt(DT[a.dtype], a.ctypes.data_as(ctypes.c_void_p), ctypes.c_int64(a.size),
                                    ctypes.c_double(p), out.ctypes.data_as(ctypes.c_void_p), int(threads))
    else:
        lib().orc_gauss_chain(DT[a.dtype], a.ctypes.data_as(ctypes.c_void_p), ctypes.c_int64(a.size),
                              ctypes.c_double(p), out.ctypes.data_as(ctypes.c_void_p))
    return out.reshape(np.asarray(x).shape, order="F")


def reduce(op, x, axes=None, threads=1):
    """Base-R reduction over `axes` (0-based list; None = all).  Returns float64.
    threads > 1 splits the outputs over threads (each output is computed by
    the same code)."""
    v = View.of(x)
    nd = len(v.shape)
    axes = list(range(nd)) if axes is None else list(axes)
    mask = 0
    for a in axes:
        mask |= 1 << a
    kept = [v.shape[d] for d in range(nd) if d not in axes]
    out = np.empty(max(1, int(np.prod(kept))), dtype=np.float64)
    args = (REDUCE[op], DT[v.dtype], v.ptr(), nd, _arr(v.shape), _arr(v.strides), ctypes.c_uint32(mask),
            out.ctypes.data_as(ctypes.POINTER(ctypes.c_double)))
    if threads > 1:
        lib_mt().orc_reduce_mt(*args, int(threads))
    else:
        lib().orc_reduce(*args)
    return out.reshape(kept, order="F") if kept else out[0]


def arg_reduce(op, x, axis=None, one_based=True, threads=1):
    v = View.of(x)
    nd = len(v.shape)
    kept = [v.shape[d] for d in range(nd) if axis is not None and d != axis]
    out = np.empty(max(1, int(np.prod(kept))), dtype=np.int64)
    args = (1 if op == "argmax" else 0, DT[v.dtype], v.ptr(), nd, _arr(v.shape), _arr(v.strides),
            -1 if axis is None else int(axis), 1 if one_based else 0, out.ctypes.data_as(_i64p))
    if threads > 1:
        lib_mt().orc_arg_reduce_mt(*args, int(threads))
    else:
        lib().orc_arg_reduce(*args)
    return out.reshape(kept, order="F") if axis is not None else int(out[0])


def scan(op, x, axis=None, threads=1):
    v = View.of(x)
    out = np.empty(int(np.prod(v.shape)), dtype=v.dtype)
    args = (1 if op == "cumprod" else 0, DT[v.dtype], v.ptr(), len(v.shape), _arr(v.shape), _arr(v.strides),
            -1 if axis is None else int(axis), out.ctypes.data_as(ctypes.c_void_p))
    if threads > 1:
        lib_mt().orc_scan_mt(*args, int(threads))
    else:
        lib().orc_scan(*args)
    return _result(out, v.shape)


def softmax(x, axis=None, threads=1):
    v = View.of(x)
    out = np.empty(int(np.prod(v.shape)), dtype=v.dtype)
    args = (DT[v.dtype], v.ptr(), len(v.shape), _arr(v.shape), _arr(v.strides), -1 if axis is None else int(axis),
            out.ctypes.data_as(ctypes.c_void_p))
    if threads > 1:
        lib_mt().orc_softmax_mt(*args, int(threads))
    else:
        lib().orc_softmax(*args)
    return _result(out, v.shape)


class ChunkedStats:
    """Base-R sum / mean / var / max / min / which.max / which.min of a
    contiguous array too large for reduce() (which gathers a fiber into long
    doubles first), fed in consecutive chunks and in two passes:

        st = ChunkedStats(n)
        for c in chunks: st.first(c)     # sum and the extrema
        for c in chunks: st.second(c)    # R's mean correction and the variance
        st.result()

    Sums are long double (numpy longdouble = C long double here); the mean is
    sum/n corrected by sum(x - m)/n as R does; the variance is two-pass around
    the corrected mean, divisor n - 1.  Indices are 1-based, first on ties,
    NaN never wins."""

    def __init__(self, n, threads=None):
        self.n = int(n)
        self.threads = int(threads or default_threads())
        self.acc1 = np.zeros(2, dtype=np.longdouble)
        self.acc2 = np.zeros(2, dtype=np.longdouble)
        self.zero = np.zeros(1, dtype=np.longdouble)
        self.val = np.zeros(2, dtype=np.float64)
        self.idx = np.full(2, -1, dtype=np.int64)
        self.pos = 0
        self.center = None

    def first(self, chunk):
        a = np.ascontiguousarray(chunk).reshape(-1)
        L = lib_mt()
        L.orc_moments_mt(DT[a.dtype], a.ctypes.data_as(ctypes.c_void_p), ctypes.c_int64(a.size),
                         self.zero.ctypes.data_as(ctypes.c_void_p), self.acc1.ctypes.data_as(ctypes.c_void_p),
                         self.threads)
        L.orc_extrema_mt(DT[a.dtype], a.ctypes.data_as(ctypes.c_void_p), ctypes.c_int64(a.size),
                         ctypes.c_int64(self.pos), self.val.ctypes.data_as(ctypes.c_void_p),
                         self.idx.ctypes.data_as(ctypes.c_void_p), self.threads)
        self.pos += a.size

    def second(self, chunk):
        if self.center is None:
            self.center = np.array([self.acc1[0] / np.longdouble(self.n)], dtype=np.longdouble)
        a = np.ascontiguousarray(chunk).reshape(-1)
        lib_mt().orc_moments_mt(DT[a.dtype], a.ctypes.data_as(ctypes.c_void_p), ctypes.c_int64(a.size),
                                self.center.ctypes.data_as(ctypes.c_void_p),
                                self.acc2.ctypes.data_as(ctypes.c_void_p), self.threads)

    def result(self):
        n = np.longdouble(self.n)
        s = self.acc1[0]
        m = self.center[0]
        t, q = self.acc2[0], self.acc2[1]
        mean = m + t / n
        var = (q - t * t / n) / (n - 1) if self.n > 1 else np.longdouble(np.nan)
        return {"sum": float(s), "mean": float(mean), "var": float(var), "max": float(self.val[0]),
                "min": float(self.val[1]), "which_max": int(self.idx[0]) + 1, "which_min": int(self.idx[1]) + 1}


def full_stats(x, threads=None):
    """ChunkedStats over one array (any size; column-major element order)."""
    a = np.ascontiguousarray(np.asarray(x).reshape(-1, order="F"))
    st = ChunkedStats(a.size, threads)
    st.first(a)
    st.second(a)
    return st.result()


def sum_var(x):
    a = np.ascontiguousarray(np.asarray(x).reshape(-1, order="F"))
    s, q = ctypes.c_double(), ctypes.c_double()
    lib().orc_sum_var(DT[a.dtype], a.ctypes.data_as(ctypes.c_void_p), ctypes.c_int64(a.size), ctypes.byref(s),
                      ctypes.byref(q))
    return s.value, q.value


def pipeline_views(x, threads=1):
    """The strided-views step on CPU: returns (y, z, sum, var, argmax_axis1)."""
    x = np.asarray(x, dtype=np.float32)
    n0, n1, n2 = x.shape
    xf = np.ascontiguousarray(x.reshape(-1, order="F"))
    y = np.empty(xf.size, dtype=np.float32)
    z = np.empty(xf.size, dtype=np.float32)
    idx = np.empty(n0 * n1, dtype=np.int32)
    s, v = ctypes.c_double(), ctypes.c_double()
    lib_mt().orc_pipeline_views(xf.ctypes.data_as(ctypes.c_void_p), ctypes.c_int64(n0), ctypes.c_int64(n1),
                                ctypes.c_int64(n2), y.ctypes.data_as(ctypes.c_void_p),
                                z.ctypes.data_as(ctypes.c_void_p), ctypes.byref(s), ctypes.byref(v),
                                idx.ctypes.data_as(ctypes.c_void_p), ctypes.c_int(threads))
    return (y.reshape((n2, n0, n1), order="F"), z.reshape((n2, n0, n1), order="F"), s.value, v.value,
            idx.reshape((n0, n1), order="F"))


def pipeline_views_raw(xf, n0, n1, n2, y, z, idx, threads):
    """Same as pipeline_views on preallocated flat buffers (for timing)."""
    s, v = ctypes.c_double(), ctypes.c_double()
    lib_mt().orc_pipeline_views(xf.ctypes.data_as(ctypes.c_void_p), ctypes.c_int64(n0), ctypes.c_int64(n1),
                                ctypes.c_int64(n2), y.ctypes.data_as(ctypes.c_void_p),
                                z.ctypes.data_as(ctypes.c_void_p), ctypes.byref(s), ctypes.byref(v),
                                idx.ctypes.data_as(ctypes.c_void_p), ctypes.c_int(threads))
    return s.value, v.value
