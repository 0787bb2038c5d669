"""Python mirror of acediaR's gpuTensor S3 API (R/gpuTensor.R) over the C ABI.

Names, argument meanings and error messages follow the R functions they
mirror; axes are 1-based as in R, storage is column-major as in R, and
keep.dims is spelled keep_dims.  Device memory comes from torch's caching
allocator (plumbing only): every computation is a call into
libacediar_b200.so on the current torch stream.

Reference semantics kept on purpose:
  - comparisons return 0/1 (R/gpuTensor.R:1872-1930); here they are stored as
    bool tensors (one byte) unless dtype_out="same" asks for the input dtype;
  - softmax() / cumsum() without an axis act on the whole tensor in
    column-major order (R/gpuTensor.R:1718, 2234-2277); axis= gives the row
    softmax / per-axis scan;
  - which.max / argmax indices are 1-based with the first-index tie rule.
"""
import builtins
import ctypes
import numbers

import numpy as np
import torch

from . import _lib as L

_TORCH = {"float": torch.float32, "double": torch.float64, "int32": torch.int32, "int64": torch.int64,
          "bool": torch.uint8}
_NUMPY = {"float": np.float32, "double": np.float64, "int32": np.int32, "int64": np.int64, "bool": np.bool_}
_ALIASES = {"float32": "float", "float64": "double", "float": "float", "double": "double", "int32": "int32",
            "int64": "int64", "bool": "bool", "logical": "bool"}

_ctx = {}


def _norm_dtype(dtype):
    try:
        return _ALIASES[dtype]
    except KeyError:
        raise ValueError("Unknown dtype string: %s" % dtype)


def context(device=None):
    """Per-device acd context (workspace + status word), created on first use."""
    if device is None:
        device = torch.cuda.current_device()
    c = _ctx.get(device)
    if c is None:
        p = ctypes.c_void_p()
        L.check(L.lib().acd_ctx_create(int(device), ctypes.byref(p)), "acd_ctx_create")
        c = p
        _ctx[device] = c
    return c


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def col_major_strides(shape):
    st, acc = [], 1
    for s in shape:
        st.append(acc)
        acc *= s
    return tuple(st)


class gpuTensor:
    """A strided column-major view over device storage."""

    __slots__ = ("storage", "shape", "strides", "offset", "dtype")

    def __init__(self, storage, shape, dtype, strides=None, offset=0):
        self.storage = storage  # 1-D torch tensor on a CUDA device
        self.shape = tuple(int(s) for s in shape)
        self.dtype = dtype
        self.strides = tuple(int(s) for s in (strides if strides is not None else col_major_strides(self.shape)))
        self.offset = int(offset)

    # ---- metadata
    @property
    def size(self):
        return int(np.prod(self.shape)) if self.shape else 1

    @property
    def ndims(self):
        return len(self.shape)

    @property
    def device(self):
        return self.storage.device

    def desc(self):
        return L.make_desc(self.storage.data_ptr(), L.DTYPE_CODES[self.dtype], self.shape, self.strides,
                           self.offset)

    def is_contiguous(self):
        return _is_contig(self.shape, self.strides)

    def __repr__(self):
        return "gpuTensor(shape=%s, dtype=%s%s)" % (self.shape, self.dtype,
                                                     "" if self.is_contiguous() else ", view")

    # ---- transfer
    def as_array(self):
        """Host numpy array with R's column-major layout."""
        t = contiguous(self) if not self.is_contiguous() or self.offset else self
        n = t.size
        host = t.storage[:n].cpu().numpy()
        if self.dtype == "bool":
            host = host.astype(np.bool_)
        return host.reshape(self.shape if self.shape else (1,), order="F")

    # ---- operators (R Ops group)
    def __add__(self, o): return _arith("add", self, o)
    def __radd__(self, o): return _arith("add", self, o)
    def __sub__(self, o): return _arith("sub", self, o)
    def __rsub__(self, o): return _arith("rsub", self, o)
    def __mul__(self, o): return _arith("mul", self, o)
    def __rmul__(self, o): return _arith("mul", self, o)
    def __truediv__(self, o): return _arith("div", self, o)
    def __rtruediv__(self, o): return _arith("rdiv", self, o)
    def __pow__(self, o): return _arith("pow", self, o)
    def __neg__(self): return _unary("neg", self)
    def __gt__(self, o): return _arith("gt", self, o)
    def __lt__(self, o): return _arith("lt", self, o)
    def __ge__(self, o): return _arith("ge", self, o)
    def __le__(self, o): return _arith("le", self, o)
    def __eq__(self, o): return _arith("eq", self, o)
    def __ne__(self, o): return _arith("ne", self, o)
    __hash__ = object.__hash__


def _is_contig(shape, strides):
    exp = 1
    for s, st in zip(shape, strides):
        if s != 1 and st != exp:
            return False
        exp *= s
    return True


def _alloc(shape, dtype, device=None):
    n = int(np.prod(shape)) if len(shape) else 1
    dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
    storage = torch.empty(builtins.max(n, 1), dtype=_TORCH[dtype], device=dev)
    return gpuTensor(storage, shape, dtype)


def empty_tensor(shape, dtype="double"):
    return _alloc(tuple(int(s) for s in shape), _norm_dtype(dtype))


def as_tensor(data, dtype="double", shape=None):
    """R's as_tensor: host data (column-major) -> device tensor."""
    dtype = _norm_dtype(dtype)
    a = np.asarray(data)
    if shape is None:
        shape = a.shape if a.ndim else (1,)
    shape = tuple(int(s) for s in shape)
    flat = np.ascontiguousarray(a.reshape(-1, order="F"), dtype=_NUMPY[dtype])
    if flat.size != (int(np.prod(shape)) if shape else 1):
        raise ValueError("Data size doesn't match shape size")
    t = _alloc(shape, dtype)
    host = torch.from_numpy(flat.view(np.uint8) if dtype == "bool" else flat)
    t.storage[:flat.size].copy_(host, non_blocking=False)
    return t


gpu_tensor = as_tensor


def from_torch(x, shape, dtype):
    """Wraps an existing flat device buffer (no copy)."""
    return gpuTensor(x.reshape(-1), shape, _norm_dtype(dtype))


def as_array(x):
    return x.as_array() if isinstance(x, gpuTensor) else np.asarray(x)


def shape(x):
    return x.shape


def dtype(x):
    return x.dtype


def synchronize():
    torch.cuda.current_stream().synchronize()


def check_device_status():
    """Raises AcdError when a kernel raised the context status word."""
    code = ctypes.c_int32()
    L.check(L.lib().acd_ctx_check(context(), _stream(), ctypes.byref(code)), "device status")


# ---------------------------------------------------------------------------
# elementwise
# ---------------------------------------------------------------------------
def _unary(op, x):
    out = _alloc(x.shape, x.dtype, x.device)
    L.check(L.lib().acd_unary(context(), L.UNARY[op], ctypes.byref(out.desc()), ctypes.byref(x.desc()), _stream()),
            op)
    return out


def _scalar_value(t):
    """Host value of a one-element tensor (the reference's scalar path copies
    it to the host, src/TensorArithmetic.cpp:812-826)."""
    return float(t.as_array().reshape(-1)[0])


_COMPARE = {"gt", "lt", "eq", "ne", "ge", "le"}


def _arith(op, a, b, dtype_out=None):
    cmp = op in _COMPARE
    if isinstance(b, numbers.Number) or (isinstance(b, np.ndarray) and b.size == 1):
        s = float(b)
        odt = ("bool" if dtype_out is None else a.dtype) if cmp else a.dtype
        out = _alloc(a.shape, odt, a.device)
        L.check(L.lib().acd_scalar(context(), L.BINARY[op], ctypes.byref(out.desc()), ctypes.byref(a.desc()),
                                   ctypes.c_double(s), _stream()), op)
        return out
    if not isinstance(b, gpuTensor):
        raise TypeError("unsupported operand type: %s" % type(b).__name__)
    if op == "rsub":
        return _arith("sub", b, a, dtype_out)
    if op == "rdiv":
        return _arith("div", b, a, dtype_out)
    if a.dtype != b.dtype:
        raise ValueError("Cannot combine tensors with different dtypes")
    # a one-element operand follows the reference's scalar path (result keeps
    # the other operand's shape)
    if a.shape != b.shape and (a.size == 1 or b.size == 1):
        big, one = (a, b) if b.size == 1 else (b, a)
        one_b = gpuTensor(one.storage, big.shape, one.dtype, (0,) * len(big.shape), one.offset)
        a, b = (big, one_b) if b.size == 1 else (one_b, big)
    if a.shape == b.shape:
        shp = a.shape
    else:
        try:
            shp = L.broadcast_shape(a.shape, b.shape)
        except L.AcdError:
            raise ValueError("Tensor shapes are not broadcastable")
    odt = ("bool" if dtype_out is None else a.dtype) if cmp else a.dtype
    out = _alloc(shp, odt, a.device)
    L.check(L.lib().acd_binary(context(), L.BINARY[op], ctypes.byref(out.desc()), ctypes.byref(a.desc()),
                               ctypes.byref(b.desc()), _stream()), op)
    return out


def compare(op, a, b, dtype_out=None):
    """`>`, `<`, ... with dtype_out="same" giving the reference's 0/1 in the input dtype."""
    return _arith(op, a, b, dtype_out=None if dtype_out is None else "same")


def exp(x): return _unary("exp", x)
def log(x): return _unary("log", x)
def sqrt(x): return _unary("sqrt", x)
def abs(x): return _unary("abs", x)
def floor(x): return _unary("floor", x)
def ceiling(x): return _unary("ceil", x)
def round(x): return _unary("round", x)
def erf(x): return _unary("erf", x)
def tanh(x): return _unary("tanh", x)
def sigmoid(x): return _unary("sigmoid", x)
def relu(x): return _unary("relu", x)
def sin(x): return _unary("sin", x)
def cos(x): return _unary("cos", x)


def pmax(a, b): return _arith("max", a, b)
def pmin(a, b): return _arith("min", a, b)


def fused(op, a, b=None, p0=0.0):
    """Fused chains (see acd_fused_op): bit-identical to the operator sequence."""
    if op == "add_relu":
        shp = L.broadcast_shape(a.shape, b.shape)
    else:
        shp = a.shape
    out = _alloc(shp, a.dtype, a.device)
    L.check(L.lib().acd_fused(context(), L.FUSED[op], ctypes.byref(out.desc()), ctypes.byref(a.desc()),
                              ctypes.byref(b.desc()) if b is not None else None, ctypes.c_double(p0), _stream()),
            op)
    return out


# ---------------------------------------------------------------------------
# views
# ---------------------------------------------------------------------------
def permute_view(x, dims):
    """Zero-copy permutation (R/gpuTensor.R:1544-1556); dims are 1-based."""
    dims = [int(d) - 1 for d in dims]
    if sorted(dims) != list(range(x.ndims)):
        raise ValueError("Invalid permutation dimensions")
    return gpuTensor(x.storage, [x.shape[d] for d in dims], x.dtype, [x.strides[d] for d in dims], x.offset)


def transpose_view(x):
    if x.ndims != 2:
        raise ValueError("Transpose currently supports 2D tensors only")
    return permute_view(x, [2, 1])


transpose = transpose_view


def contiguous(x):
    """Materialises a view in column-major order (tensor_strided_copy)."""
    if x.is_contiguous() and x.offset == 0:
        return x
    out = _alloc(x.shape, x.dtype, x.device)
    L.check(L.lib().acd_copy(context(), ctypes.byref(out.desc()), ctypes.byref(x.desc()), _stream()), "contiguous")
    return out


def is_contiguous(x):
    return x.is_contiguous()


_DTYPE_ALIASES = {"float32": "float", "float": "float", "float64": "double", "double": "double",
                  "int32": "int32", "int": "int32", "int64": "int64", "long": "int64", "bool": "bool",
                  "logical": "bool"}


def to_dtype(x, target_dtype):
    """tensor_to_dtype_unified (src/TensorDataAccess.cpp:152-190): a new tensor
    of `target_dtype` holding as.<dtype>(x) (truncation toward zero and NA for
    NaN or out-of-range values when converting to an integer type)."""
    dt = _DTYPE_ALIASES.get(target_dtype)
    if dt is None:
        raise ValueError("Error converting tensor dtype: Unsupported target dtype: %s" % target_dtype)
    out = _alloc(x.shape, dt, x.device)
    L.check(L.lib().acd_convert(context(), ctypes.byref(out.desc()), ctypes.byref(x.desc()), _stream()),
            "to_dtype")
    return out


def view(x, shape):
    shape = tuple(int(s) for s in shape)
    if int(np.prod(shape)) != x.size:
        raise ValueError("View shape size must match original size")
    base = contiguous(x)
    return gpuTensor(base.storage, shape, base.dtype, None, base.offset)


reshape = view


# ---------------------------------------------------------------------------
# reductions
# ---------------------------------------------------------------------------
def _axes_mask(x, axis):
    axes = [axis] if isinstance(axis, numbers.Number) else list(axis)
    for a in axes:
        if not isinstance(a, numbers.Number) or a != int(a) or a < 1 or a > x.ndims:
            raise ValueError("axis must be a vector of positive integers")
    mask = 0
    for a in axes:
        mask |= 1 << (int(a) - 1)
    return mask, sorted(set(int(a) - 1 for a in axes))


def _reduce(op, x, axis=None, keep_dims=False, out_dtype=None):
    if axis is None:
        mask, axes = (1 << x.ndims) - 1 if x.ndims else 0, list(range(x.ndims))
    else:
        mask, axes = _axes_mask(x, axis)
    kept = [x.shape[d] for d in range(x.ndims) if d not in axes]
    if keep_dims:
        oshape = [1 if d in axes else x.shape[d] for d in range(x.ndims)]
    else:
        oshape = kept if kept else [1]
    if out_dtype is None:
        if op == "count":
            out_dtype = "int32"
        elif x.dtype == "bool":
            out_dtype = "int32"
        elif x.dtype in ("int32", "int64") and op in ("mean", "var", "prod"):
            out_dtype = "double"
        else:
            out_dtype = x.dtype
    out = _alloc(tuple(oshape), out_dtype, x.device)
    L.check(L.lib().acd_reduce(context(), L.REDUCE[op], ctypes.byref(out.desc()), ctypes.byref(x.desc()),
                               ctypes.c_uint32(mask), _stream()), op)
    return out


def _scalar_result(t):
    v = t.as_array().reshape(-1)[0]
    return int(v) if t.dtype in ("int32", "int64") else float(v)


def tensor_sum(x, axis=None, keep_dims=False): return _reduce("sum", x, axis, keep_dims)
def tensor_mean(x, axis=None, keep_dims=False): return _reduce("mean", x, axis, keep_dims)
def tensor_max(x, axis=None, keep_dims=False): return _reduce("max", x, axis, keep_dims)
def tensor_min(x, axis=None, keep_dims=False): return _reduce("min", x, axis, keep_dims)
def tensor_prod(x, axis=None, keep_dims=False): return _reduce("prod", x, axis, keep_dims)
def tensor_var(x, axis=None, keep_dims=False): return _reduce("var", x, axis, keep_dims)
def tensor_count(x, axis=None, keep_dims=False): return _reduce("count", x, axis, keep_dims)


def _r_reduce(op):
    def f(x, axis=None, keep_dims=False):
        t = _reduce(op, x, axis, keep_dims, out_dtype="double" if axis is None and x.dtype in ("float", "double")
                    else None)
        return _scalar_result(t) if axis is None else t
    f.__name__ = op
    f.__doc__ = "R's %s.gpuTensor: a number without axis, a gpuTensor with axis (1-based)." % op
    return f


sum = _r_reduce("sum")
mean = _r_reduce("mean")
max = _r_reduce("max")
min = _r_reduce("min")
prod = _r_reduce("prod")
var = _r_reduce("var")


def sum_var(x):
    """Fused single pass: (sum, var) as Python floats."""
    s = _alloc((1,), "double", x.device)
    v = _alloc((1,), "double", x.device)
    L.check(L.lib().acd_sum_var(context(), ctypes.byref(s.desc()), ctypes.byref(v.desc()), ctypes.byref(x.desc()),
                                _stream()), "sum_var")
    return float(s.as_array()[0]), float(v.as_array()[0])


def _arg(op, x, axis=None, keep_dims=False, one_based=True, index_dtype=None):
    if axis is None:
        idt = index_dtype or ("int32" if x.size < 2 ** 31 else "int64")
        out = _alloc((1,), idt, x.device)
        L.check(L.lib().acd_arg_reduce(context(), L.ARG[op], ctypes.byref(out.desc()), None, ctypes.byref(x.desc()),
                                       -1, 1 if one_based else 0, _stream()), op)
        return out
    if not isinstance(axis, numbers.Number) or axis != int(axis) or axis < 1 or axis > x.ndims:
        raise ValueError("axis must be a single positive integer within tensor dimensions")
    a = int(axis) - 1
    kept = [x.shape[d] for d in range(x.ndims) if d != a]
    oshape = [1 if d == a else x.shape[d] for d in range(x.ndims)] if keep_dims else (kept if kept else [1])
    out = _alloc(tuple(oshape), index_dtype or "int64", x.device)
    L.check(L.lib().acd_arg_reduce(context(), L.ARG[op], ctypes.byref(out.desc()), None, ctypes.byref(x.desc()), a,
                                   1 if one_based else 0, _stream()), op)
    return out


def argmax(x, axis=None, keep_dims=False):
    """R's argmax(): 1-based; a number without axis, an int64 gpuTensor with axis."""
    t = _arg("argmax", x, axis, keep_dims)
    return _scalar_result(t) if axis is None else t


def argmin(x, axis=None, keep_dims=False):
    t = _arg("argmin", x, axis, keep_dims)
    return _scalar_result(t) if axis is None else t


def which_max(x):
    return _scalar_result(_arg("argmax", x))


def which_min(x):
    return _scalar_result(_arg("argmin", x))


# ---------------------------------------------------------------------------
# scans and softmax
# ---------------------------------------------------------------------------
def _scan(op, x, axis=None):
    if axis is not None:
        if not isinstance(axis, numbers.Number) or axis != int(axis) or axis < 1 or axis > x.ndims:
            raise ValueError("axis must be a single positive integer within tensor dimensions")
        a = int(axis) - 1
    else:
        a = -1
        if not x.is_contiguous() or x.offset:
            x = contiguous(x)
    out = _alloc(x.shape, x.dtype, x.device)
    st = L.lib().acd_scan(context(), L.SCAN[op], ctypes.byref(out.desc()), ctypes.byref(x.desc()), a, _stream())
    if st == 8:  # view not collapsible around the axis: materialise first
        x = contiguous(x)
        st = L.lib().acd_scan(context(), L.SCAN[op], ctypes.byref(out.desc()), ctypes.byref(x.desc()), a, _stream())
    L.check(st, op)
    return out


def cumsum(x, axis=None): return _scan("cumsum", x, axis)
def cumprod(x, axis=None): return _scan("cumprod", x, axis)


def softmax(x, axis=None):
    """Whole-tensor softmax (reference semantics) or, with axis, along that axis."""
    if axis is not None:
        if not isinstance(axis, numbers.Number) or axis != int(axis) or axis < 1 or axis > x.ndims:
            raise ValueError("axis must be a single positive integer within tensor dimensions")
        a = int(axis) - 1
    else:
        a = -1
        if not x.is_contiguous() or x.offset:
            x = contiguous(x)
    out = _alloc(x.shape, x.dtype, x.device)
    st = L.lib().acd_softmax(context(), ctypes.byref(out.desc()), ctypes.byref(x.desc()), a, _stream())
    if st == 8:
        x = contiguous(x)
        st = L.lib().acd_softmax(context(), ctypes.byref(out.desc()), ctypes.byref(x.desc()), a, _stream())
    L.check(st, "softmax")
    return out
