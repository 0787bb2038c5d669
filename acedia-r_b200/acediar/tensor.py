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
import os

import numpy as np
import torch

from . import _lib as L

_TORCH = {"float": torch.float32, "double": torch.float64, "int32": torch.int32, "int64": torch.int64,
          "bool": torch.uint8, "float16": torch.float16, "int8": torch.int8}
_NUMPY = {"float": np.float32, "double": np.float64, "int32": np.int32, "int64": np.int64, "bool": np.bool_,
          "float16": np.float16, "int8": np.int8}
_ALIASES = {"float32": "float", "float64": "double", "float": "float", "double": "double", "int32": "int32",
            "int64": "int64", "bool": "bool", "logical": "bool", "float16": "float16", "half": "float16",
            "int8": "int8"}

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

    def __str__(self):
        """print.gpuTensor (R/gpuTensor.R:295-311): shape, device, dtype,
        size, and the values when there are at most 100."""
        lines = ["gpuTensor with shape %s " % " x ".join(str(s) for s in self.shape), "Device: CUDA",
                 "DType: %s " % self.dtype, "Size: %d elements" % self.size]
        if self.size <= 100:
            lines += ["Data:", str(self.as_array())]
        else:
            lines.append("Use as.array() to view data")
        return "\n".join(lines)

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


def log(x, base=np.e):
    """log.gpuTensor (R/gpuTensor.R:873-883) over tensor_log_unified
    (src/TensorMath.cpp:167-174): natural logarithm only, and an input with a
    value <= 0 is an error (NaN is not).  The check runs on the device (one
    comparison and count) where the reference copies the tensor to the host."""
    if base != np.e:
        raise ValueError("Only natural logarithm (base e) is currently supported")
    if x.dtype in ("float", "double") and tensor_count(_arith("le", x, 0.0)).as_array().reshape(-1)[0] > 0:
        raise ValueError("log() domain error: input contains non-positive values")
    return _unary("log", x)
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


# ---- slicing, assignment and assembly (src/TensorMutation.cpp) -------------
def _ranges(x, idx, what):
    """R index arguments -> (start0, count, keep) per axis.  None selects the
    whole axis, an int (1-based) one element (the axis is dropped), a
    sequence of 1-based ints a contiguous range (R/gpuTensor.R:719-811)."""
    if len(idx) > x.ndims:
        raise ValueError("Too many indices for tensor with %d dimensions" % x.ndims)
    starts, counts, keep = [], [], []
    for d in range(x.ndims):
        i = idx[d] if d < len(idx) else None
        n = x.shape[d]
        if i is None:
            starts.append(0), counts.append(n), keep.append(True)
            continue
        v = [int(i)] if isinstance(i, numbers.Number) else [int(k) for k in i]
        if builtins.any(k <= 0 for k in v):
            raise ValueError("Only positive indices are supported in this implementation" if what == "[" else
                             "Negative or zero indices not supported in slice assignment")
        if builtins.any(k > n for k in v):
            raise ValueError("Index %d is out of bounds for dimension %d with size %d" % (builtins.max(v), d + 1, n)
                             if what == "[" else "Index out of bounds in slice assignment")
        if builtins.any(b - a != 1 for a, b in zip(v, v[1:])):
            raise ValueError("Only contiguous ranges are supported in this basic implementation" if what == "[" else
                             "Only contiguous ranges supported in slice assignment")
        starts.append(v[0] - 1), counts.append(len(v)), keep.append(len(v) > 1 or not isinstance(i, numbers.Number))
    return starts, counts, keep


def _slice_view(x, starts, counts):
    st = (ctypes.c_int64 * builtins.max(x.ndims, 1))(*starts)
    ct = (ctypes.c_int64 * builtins.max(x.ndims, 1))(*counts)
    d = L.Desc()
    L.check(L.lib().acd_slice_desc(ctypes.byref(x.desc()), st, ct, ctypes.byref(d)), "slice")
    return gpuTensor(x.storage, tuple(counts), x.dtype, x.strides, d.offset)


def subset(x, *idx):
    """`[.gpuTensor`: x[i, j, ...] with R's 1-based contiguous ranges; a
    single index drops its axis, and a result with no axes left is a
    number (R/gpuTensor.R:719-811)."""
    if not idx:
        return x
    starts, counts, keep = _ranges(x, idx, "[")
    v = contiguous(_slice_view(x, starts, counts))
    new_shape = [c for c, k in zip(counts, keep) if k]
    if not new_shape:
        return _scalar_result(v)
    return gpuTensor(v.storage, tuple(new_shape), v.dtype, col_major_strides(new_shape), v.offset)


def assign(x, *idx, value):
    """`[<-.gpuTensor`, in place: x[mask] <- scalar (mask a bool tensor or a
    logical array of x's length), x[ranges] <- scalar, x[ranges] <- tensor or
    vector of the slice's shape (src/TensorMutation.cpp:439-623)."""
    if len(idx) == 1 and (isinstance(idx[0], gpuTensor) and idx[0].dtype == "bool" or
                          isinstance(idx[0], np.ndarray) and idx[0].dtype == np.bool_):
        m = idx[0]
        if isinstance(m, np.ndarray):
            if m.size != x.size:
                raise ValueError("Logical mask must have same length as tensor")
            m = as_tensor(m.reshape(x.shape if x.shape else (1,), order="F"), dtype="bool")
        if not isinstance(value, numbers.Number):
            raise ValueError("Currently only scalar assignment to boolean mask is supported")
        L.check(L.lib().acd_mask_fill(context(), ctypes.byref(x.desc()), ctypes.byref(m.desc()),
                                      ctypes.c_double(float(value)), _stream()), "mask assignment")
        return x
    starts, counts, _ = _ranges(x, idx, "[<-")
    v = _slice_view(x, starts, counts)
    if isinstance(value, numbers.Number):
        L.check(L.lib().acd_fill(context(), ctypes.byref(v.desc()), ctypes.c_double(float(value)), _stream()),
                "slice assignment")
        return x
    if not isinstance(value, gpuTensor):
        value = as_tensor(np.asarray(value).reshape(counts, order="F"), dtype=x.dtype)
    if value.dtype != x.dtype:
        value = to_dtype(value, x.dtype)
    if value.size != v.size:
        raise ValueError("Source tensor shape must match slice shape")
    src = value if tuple(value.shape) == tuple(counts) else gpuTensor(
        contiguous(value).storage, tuple(counts), value.dtype)
    L.check(L.lib().acd_copy(context(), ctypes.byref(v.desc()), ctypes.byref(src.desc()), _stream()),
            "slice assignment")
    return x


def _desc_array(tensors):
    descs = [t.desc() for t in tensors]
    arr = (ctypes.POINTER(L.Desc) * len(descs))(*[ctypes.pointer(d) for d in descs])
    return arr, descs


def concat_tensor(lst, axis=1):
    """tensor_concat_unified (src/TensorMutation.cpp:167-273): concatenation
    along `axis` (1-based)."""
    if len(lst) < 2:
        raise ValueError("Need at least two tensors to concatenate")
    a = int(axis) - 1
    base = lst[0]
    if a < 0 or a >= base.ndims:
        raise ValueError("axis out of range")
    shape = list(base.shape)
    shape[a] = builtins.sum(t.shape[a] for t in lst) if builtins.all(t.ndims == base.ndims for t in lst) else -1
    if shape[a] < 0:
        raise ValueError("All tensors must have same number of dims")
    out = _alloc(tuple(shape), base.dtype, base.device)
    arr, keep = _desc_array(lst)
    L.check(L.lib().acd_concat(context(), ctypes.byref(out.desc()), arr, len(lst), a, _stream()), "concat")
    return out


def stack_tensor(lst, axis=1):
    """tensor_stack_unified (src/TensorMutation.cpp:275-331): equal-shaped
    tensors stacked along a new axis at position `axis` (1-based)."""
    if len(lst) < 2:
        raise ValueError("Need at least two tensors to stack")
    a = int(axis) - 1
    base = lst[0]
    if a < 0 or a > base.ndims:
        raise ValueError("axis out of range")
    shape = list(base.shape)
    shape.insert(a, len(lst))
    out = _alloc(tuple(shape), base.dtype, base.device)
    arr, keep = _desc_array(lst)
    L.check(L.lib().acd_stack(context(), ctypes.byref(out.desc()), arr, len(lst), a, _stream()), "stack")
    return out


def repeat_tensor(x, reps):
    """tensor_repeat_unified (src/TensorMutation.cpp:333-385): each element
    repeated reps[d] times along axis d."""
    reps = [int(r) for r in (reps if not isinstance(reps, numbers.Number) else [reps])]
    if len(reps) != x.ndims:
        raise ValueError("repeats length must match tensor dims")
    if builtins.any(r <= 0 for r in reps):
        raise ValueError("repeat counts must be positive")
    out = _alloc(tuple(s * r for s, r in zip(x.shape, reps)), x.dtype, x.device)
    rp = (ctypes.c_int64 * len(reps))(*reps)
    L.check(L.lib().acd_repeat(context(), ctypes.byref(out.desc()), ctypes.byref(x.desc()), rp, _stream()), "repeat")
    return out


_PAD_MODES = {"constant": 0, "reflect": 1, "replicate": 2}


def pad(x, pad_width, mode="constant", value=0):
    """tensor_pad_unified (src/TensorMutation.cpp:387-437): pad_width is an
    ndims x 2 matrix of (before, after) counts."""
    if mode not in _PAD_MODES:
        raise ValueError("Unsupported pad mode")
    pw = np.asarray(pad_width, dtype=np.int64).reshape(-1, 2)
    if pw.shape[0] != x.ndims:
        raise ValueError("pad_width must be matrix of ndims x 2")
    if (pw < 0).any():
        raise ValueError("padding must be non-negative")
    out = _alloc(tuple(int(s + b + a) for s, (b, a) in zip(x.shape, pw)), x.dtype, x.device)
    bp = (ctypes.c_int64 * x.ndims)(*[int(b) for b in pw[:, 0]])
    L.check(L.lib().acd_pad(context(), ctypes.byref(out.desc()), ctypes.byref(x.desc()), bp, _PAD_MODES[mode],
                            ctypes.c_double(float(value)), _stream()), "pad")
    return out


def pad_tensor(x, pad_width, mode="constant", value=0):
    """pad_tensor (R/gpuTensor.R:1816-1831): pad_width = c(before1, after1,
    before2, after2, ...)."""
    if len(pad_width) != x.ndims * 2:
        raise ValueError("pad_width must have length ndims * 2")
    return pad(x, np.asarray(pad_width).reshape(x.ndims, 2), mode, value)


concat = concat_tensor
stack = stack_tensor


def _flat_view(x, start, count):
    """Elements start .. start+count-1 of a contiguous tensor, as a 1-D view."""
    return gpuTensor(x.storage, (count,), x.dtype, (1,), x.offset + start)


def diff(x, lag=1, differences=1):
    """diff.gpuTensor (R/gpuTensor.R:2289-2333) on the device: base R's
    diff(as.vector(x), lag, differences), each round one subtraction of two
    offset views; a result of a multi-dimensional tensor is recycled to the
    tensor's size and shape, as the reference does."""
    if lag < 1:
        raise ValueError("lag must be positive")
    if differences < 1:
        raise ValueError("differences must be positive")
    d = contiguous(x) if not (x.is_contiguous()) else x
    n = d.size
    for _ in range(int(differences)):
        m = n - int(lag)
        if m <= 0:
            raise ValueError("diff of single element tensor results in empty result - not supported by tensor system")
        out = _alloc((m,), d.dtype, d.device)
        L.check(L.lib().acd_binary(context(), L.BINARY["sub"], ctypes.byref(out.desc()),
                                   ctypes.byref(_flat_view(d, int(lag), m).desc()),
                                   ctypes.byref(_flat_view(d, 0, m).desc()), _stream()), "diff")
        d, n = out, m
    if x.ndims <= 1:
        return d
    full = _alloc(x.shape, x.dtype, x.device)  # rep_len(result, prod(shape))
    pos, total = 0, x.size
    while pos < total:
        k = builtins.min(n, total - pos)
        L.check(L.lib().acd_copy(context(), ctypes.byref(_flat_view(full, pos, k).desc()),
                                 ctypes.byref(_flat_view(d, 0, k).desc()), _stream()), "diff")
        pos += k
    return full


def range_(x):
    """range.gpuTensor (R/gpuTensor.R:2216-2226): [min, max]."""
    return [float(tensor_min(x).as_array().reshape(-1)[0]), float(tensor_max(x).as_array().reshape(-1)[0])]


def is_finite(x):
    """is.finite.gpuTensor (R/gpuTensor.R:1594-1596): TRUE when every element
    is finite.  x - x is 0 exactly for finite x and NaN for +-Inf and NaN."""
    if x.dtype in ("int32", "int64", "bool"):
        return True
    return bool(all((x - x) == 0))


def all_equal(target, current, tolerance=1.5e-8):
    """all.equal.gpuTensor (R/gpuTensor.R:1587-1591): base R's all.equal on
    the host arrays — True, or a message naming the difference (mismatched
    lengths, NA positions, or the mean relative / absolute difference above
    `tolerance`)."""
    t = np.asarray(target.as_array() if isinstance(target, gpuTensor) else target, dtype=np.float64)
    c = np.asarray(current.as_array() if isinstance(current, gpuTensor) else current, dtype=np.float64)
    if t.size != c.size:
        return "Lengths (%d, %d) differ" % (t.size, c.size)
    t, c = t.reshape(-1, order="F"), c.reshape(-1, order="F")
    na_t, na_c = np.isnan(t), np.isnan(c)
    if (na_t != na_c).any():
        return "'is.NA' value mismatch: %d in current %d in target" % (na_c.sum(), na_t.sum())
    t, c = t[~na_t], c[~na_t]
    if t.size == 0:
        return True
    xy = np.abs(t - c).mean()
    xn = np.abs(t).mean()
    what = "absolute"
    if np.isfinite(xn) and xn > tolerance:
        xy, what = xy / xn, "relative"
    if np.isnan(xy) or xy > tolerance:
        return "Mean %s difference: %.7g" % (what, xy)
    return True


def create_ones_like(t):
    """create_ones_like (R/gpuTensor.R:238-257): ones of t's shape and dtype,
    filled on the device (the reference copies a host vector)."""
    out = _alloc(t.shape, t.dtype, t.device)
    L.check(L.lib().acd_fill(context(), ctypes.byref(out.desc()), ctypes.c_double(1.0), _stream()), "ones_like")
    return out


def tensor_pow(a, b):
    """tensor_pow (R/gpuTensor.R:2123-2130): a^b elementwise with broadcasting."""
    if not isinstance(a, gpuTensor) or not isinstance(b, gpuTensor):
        raise ValueError("Both arguments must be gpuTensor objects")
    return _arith("pow", a, b)


# ---- random tensors (src/TensorRandom.cpp, R/gpuTensor.R:2342-2524) ---------
# A counter-based stream: (seed, position).  Every call takes the next n
# positions (rounded up to a multiple of 4).  set_seed makes runs repeatable;
# the initial seed comes from the OS, as the reference seeds from the clock.
_rng = {"seed": int.from_bytes(os.urandom(8), "little"), "pos": 0}


def set_seed(seed):
    """Seeds the tensor random stream (position 0 of seed `seed`)."""
    _rng["seed"] = int(seed) & (2 ** 64 - 1)
    _rng["pos"] = 0


def _rand(shape, dtype, dist, a, b):
    shape = tuple(int(s) for s in (shape if not isinstance(shape, numbers.Number) else [shape]))
    if builtins.any(s <= 0 for s in shape):
        raise ValueError("All shape dimensions must be positive")
    dt = _ALIASES.get(dtype, dtype)
    if dt not in ("float", "double"):
        raise ValueError("Unsupported dtype for random tensor. Use 'float' or 'double'")
    out = _alloc(shape, dt)
    pos = _rng["pos"]
    _rng["pos"] = pos + (out.size + 3) // 4 * 4
    L.check(L.lib().acd_rand(context(), ctypes.byref(out.desc()), dist, ctypes.c_double(a), ctypes.c_double(b),
                             ctypes.c_uint64(_rng["seed"]), ctypes.c_uint64(pos), _stream()), "rand_tensor")
    return out


def rand_tensor(shape, dtype="float"):
    """rand_tensor (src/TensorRandom.cpp:42-110): uniform on [0, 1)."""
    return _rand(shape, dtype, 0, 0.0, 1.0)


def rnorm_tensor(shape, mean=0.0, sd=1.0, dtype="float"):
    """rnorm_tensor (src/TensorRandom.cpp:120-224): normal(mean, sd)."""
    return _rand(shape, dtype, 1, float(mean), float(sd))


def rand_tensor_uniform(shape, dtype="float", min=0.0, max=1.0):
    """rand_tensor_uniform (R/gpuTensor.R): uniform on [min, max)."""
    if not (min < max):
        raise ValueError("min must be less than max")
    return _rand(shape, dtype, 0, float(min), float(max))


def rand_tensor_normal(shape, mean=0.0, sd=1.0, dtype="float"):
    """rand_tensor_normal (R/gpuTensor.R): normal(mean, sd)."""
    if not sd > 0:
        raise ValueError("sd must be positive")
    return _rand(shape, dtype, 1, float(mean), float(sd))


def runif(x, min=0.0, max=1.0):
    """runif.gpuTensor: a new tensor of x's shape and dtype, uniform on [min, max)."""
    if not isinstance(x, gpuTensor):
        raise ValueError("runif method requires a gpuTensor object or numeric count")
    return rand_tensor_uniform(x.shape, x.dtype, min, max)


def rnorm(x, mean=0.0, sd=1.0):
    """rnorm.gpuTensor: a new tensor of x's shape and dtype, normal(mean, sd)."""
    if not isinstance(x, gpuTensor):
        raise ValueError("rnorm method requires a gpuTensor object or numeric count")
    return rand_tensor_normal(x.shape, mean, sd, x.dtype)


_DTYPE_ALIASES = {"float32": "float", "float": "float", "float64": "double", "double": "double",
                  "int32": "int32", "int": "int32", "int64": "int64", "long": "int64", "bool": "bool",
                  "logical": "bool", "float16": "float16", "half": "float16", "int8": "int8"}


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
        elif x.dtype in ("bool", "int8"):
            out_dtype = "double" if op == "mean" else "int32"
        elif x.dtype in ("int32", "int64") and op in ("mean", "var", "prod"):
            out_dtype = "double"
        elif x.dtype == "float16":
            out_dtype = "float"  # the reference's float16 sum returns float (src/TensorReduction.cpp:12)
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


def _logical(op, x, axis):
    r = _reduce(op, x, axis, False, out_dtype="int32")
    if axis is not None:
        return r
    v = int(r.as_array().reshape(-1)[0])
    return None if v == np.iinfo(np.int32).min else bool(v)


def any(x, axis=None):
    """any.gpuTensor (R/gpuTensor.R:2178-2187), on the device: TRUE if an
    element is non-zero, else NA (None) if an element is NaN, else FALSE.
    With `axis`, an int32 tensor of 1 / 0 / NA (INT32_MIN)."""
    return _logical("any", x, axis)


def all(x, axis=None):
    """all.gpuTensor (R/gpuTensor.R:2197-2206), on the device: FALSE if an
    element is zero, else NA (None) if an element is NaN, else TRUE."""
    return _logical("all", x, axis)


def _r_reduce(op):
    def f(x, axis=None, keep_dims=False):
        t = _reduce(op, x, axis, keep_dims,
                    out_dtype="double" if axis is None and x.dtype in ("float", "double", "float16") else None)
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


def chain5_stats(a, b):
    """The elementwise chain + reduction configuration in one kernel
    (acd_chain5_stats): for float64 tensors a and b of one size, the tensors
    a + b, a * b, exp(a), sigmoid(b), sqrt(a) (each bit-identical to the
    operator), a float64[15] device tensor of their (sum, mean, var) and an
    int64[1] device tensor holding which.max(a + b)."""
    if a.dtype != "double" or b.dtype != "double" or a.size != b.size:
        raise ValueError("chain5_stats: float64 tensors of one size required")
    a = contiguous(a) if not a.is_contiguous() or a.offset else a
    b = contiguous(b) if not b.is_contiguous() or b.offset else b
    outs = [_alloc(a.shape, "double", a.device) for _ in range(5)]
    stats = torch.empty(15, dtype=torch.float64, device=a.device)
    which = torch.empty(1, dtype=torch.int64, device=a.device)
    descs = [o.desc() for o in outs]
    arr = (ctypes.POINTER(L.Desc) * 5)(*[ctypes.pointer(d) for d in descs])
    L.check(L.lib().acd_chain5_stats(context(), ctypes.byref(a.desc()), ctypes.byref(b.desc()), arr,
                                     ctypes.c_void_p(stats.data_ptr()), ctypes.c_void_p(which.data_ptr()), _stream()),
            "chain5_stats")
    return outs, stats, which


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


# ---------------------------------------------------------------------------
# host-side helpers of the R API (metadata, transfers, device queries)
# ---------------------------------------------------------------------------
def permute(tensor, dims):
    """permute (R/gpuTensor.R:619-633): a zero-copy view with the axes in
    `dims` order (1-based)."""
    if len(dims) != tensor.ndims:
        raise ValueError("Number of dimensions in 'dims' must match tensor dimensions")
    return permute_view(tensor, dims)


def size(tensor):
    """size (R/gpuTensor.R:274-279): the number of elements."""
    return tensor.size


def dim(x):
    """dim.gpuTensor (R/gpuTensor.R:844-846): the shape as integers."""
    return [int(s) for s in x.shape]


def as_vector(x):
    """as.vector.gpuTensor (R/gpuTensor.R:187-190): the elements in
    column-major order, in the tensor's dtype."""
    return x.as_array().reshape(-1, order="F")


def as_numeric(x):
    """as.numeric.gpuTensor (R/gpuTensor.R:193-198): the elements in
    column-major order as float64."""
    return as_vector(x).astype(np.float64)


def to_numeric(x):
    """to_numeric (R/gpuTensor.R:202-208)."""
    return as_numeric(x) if isinstance(x, gpuTensor) else np.asarray(x, dtype=np.float64).reshape(-1)


def tensor_to_scalar(x):
    """tensor_to_scalar (R/gpuTensor.R:218-230): the first element as a
    number, with a warning when the tensor holds more than one."""
    if not isinstance(x, gpuTensor):
        raise ValueError("x must be a gpuTensor")
    if x.size != 1:
        import warnings
        warnings.warn("Converting multi-element tensor to scalar, using first element")
    first = gpuTensor(x.storage, (1,), x.dtype, (1,), x.offset)
    return float(first.as_array().reshape(-1)[0])


def shares_memory(tensor1, tensor2):
    """shares_memory (R/gpuTensor.R:1524-1534).  The reference answers FALSE
    always; here True when the two views address overlapping bytes of the
    same device allocation (the span from each view's lowest to highest
    element)."""
    if not isinstance(tensor1, gpuTensor) or not isinstance(tensor2, gpuTensor):
        raise ValueError("Both objects must be gpuTensors")
    if tensor1.storage.untyped_storage().data_ptr() != tensor2.storage.untyped_storage().data_ptr():
        return False

    def span(t):
        es = t.storage.element_size()
        lo = hi = t.offset
        for n, s in zip(t.shape, t.strides):
            if n == 0:
                return None
            if s < 0:
                lo += (n - 1) * s
            else:
                hi += (n - 1) * s
        base = t.storage.data_ptr()
        return base + lo * es, base + (hi + 1) * es

    a, b = span(tensor1), span(tensor2)
    return a is not None and b is not None and a[0] < b[1] and b[0] < a[1]


def tensor_info(tensor):
    """tensor_info (R/gpuTensor.R:1566-1577): shape, size, strides,
    contiguity and dtype."""
    if not isinstance(tensor, gpuTensor):
        raise ValueError("Object is not a gpuTensor")
    return {"shape": list(tensor.shape), "size": tensor.size, "strides": list(tensor.strides),
            "is_contiguous": tensor.is_contiguous(), "dtype": tensor.dtype}


def set_random_seed(seed):
    """set_random_seed (src/TensorRandom.cpp:221-231): reseeds the random
    stream used by rand_tensor / rnorm_tensor / runif / rnorm."""
    set_seed(int(seed))


def gpu_available():
    """gpu_available (src/RcppInterface.cpp:7-9)."""
    return bool(L.lib().acd_gpu_available())


def gpu_info():
    """gpu_info (src/RcppInterface.cpp:12-14): the device list as text."""
    n = L.lib().acd_gpu_info(None, 0)
    buf = ctypes.create_string_buffer(int(n) + 1)
    L.lib().acd_gpu_info(buf, len(buf))
    return buf.value.decode()


def gpu_memory_available():
    """gpu_memory_available (src/RcppInterface.cpp:17-20): free bytes."""
    return float(L.lib().acd_gpu_memory_available())


def gpu_status():
    """gpu_status (R/gpu-utils.R:74-82)."""
    free = gpu_memory_available()
    ok = gpu_available()
    return {"available": ok, "info": gpu_info(), "memory_available": free, "memory_gb": free / 1e9,
            "recommended_use": ok and free > 1e9}


def _vector_pair(a, b):
    a = np.asarray(a, dtype=np.float64).reshape(-1)
    b = np.asarray(b, dtype=np.float64).reshape(-1)
    if a.size != b.size:
        raise ValueError("Input vectors must have the same length")
    return a, b


def _device_only(force_cpu):
    if force_cpu:
        raise ValueError("force_cpu is not supported: this library computes on the device only")


def gpu_add(a, b, force_cpu=False, warn_fallback=True):
    """gpu_add (R/gpu_add.R:51-89): a + b of two numeric vectors through
    float64 tensors.  The reference falls back to the CPU on error; here an
    error propagates."""
    _device_only(force_cpu)
    a, b = _vector_pair(a, b)
    if a.size == 0:
        return np.zeros(0)
    return as_vector(as_tensor(a) + as_tensor(b))


def gpu_multiply(a, b, force_cpu=False, warn_fallback=True):
    """gpu_multiply (R/gpu_multiply.R:51-88): a * b elementwise."""
    _device_only(force_cpu)
    a, b = _vector_pair(a, b)
    if a.size == 0:
        return np.zeros(0)
    return as_vector(as_tensor(a) * as_tensor(b))


def gpu_scale(x, scalar, force_cpu=False, warn_fallback=True):
    """gpu_scale (R/gpu_multiply.R:127-163): x * scalar."""
    _device_only(force_cpu)
    if np.ndim(scalar) != 0 and np.size(scalar) != 1:
        raise ValueError("scalar must be a single numeric value")
    x = np.asarray(x, dtype=np.float64).reshape(-1)
    if x.size == 0:
        return np.zeros(0)
    return as_vector(as_tensor(x) * float(np.asarray(scalar).reshape(-1)[0]))


def gpu_dot(a, b, force_cpu=False, warn_fallback=True):
    """gpu_dot (R/gpu_multiply.R:201-238): tensor_sum(a * b)."""
    _device_only(force_cpu)
    a, b = _vector_pair(a, b)
    if a.size == 0:
        return 0.0
    return float(tensor_sum(as_tensor(a) * as_tensor(b)).as_array().reshape(-1)[0])
