"""ctypes binding of libacediar_b200.so (the C ABI declared in include/acd.h).

The library is the product: there is no fallback.  Importing this module
without the built library raises ImportError with the build command.
"""
import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
LIB_PATH = os.path.join(PKG, "lib", "libacediar_b200.so")

MAX_DIMS = 8

FLOAT32, FLOAT64, INT32, INT64, BOOL, FLOAT16, INT8 = 0, 1, 2, 3, 4, 5, 6
DTYPE_CODES = {"float": FLOAT32, "double": FLOAT64, "int32": INT32, "int64": INT64, "bool": BOOL,
               "float16": FLOAT16, "int8": INT8}
DTYPE_NAMES = {v: k for k, v in DTYPE_CODES.items()}
DTYPE_SIZES = {FLOAT32: 4, FLOAT64: 8, INT32: 4, INT64: 8, BOOL: 1, FLOAT16: 2, INT8: 1}

UNARY = {n: i for i, n in enumerate(
    ["exp", "log", "sqrt", "abs", "floor", "ceil", "round", "erf", "tanh", "sigmoid", "relu", "sin", "cos",
     "neg", "square", "copy"])}
BINARY = {n: i for i, n in enumerate(
    ["add", "sub", "mul", "div", "max", "min", "pow", "gt", "lt", "eq", "ne", "ge", "le", "rsub", "rdiv"])}
FUSED = {"scale_add_exp_neg_square": 0, "add_relu": 1, "tanh_scale": 2}
REDUCE = {n: i for i, n in enumerate(["sum", "mean", "max", "min", "prod", "var", "count", "any", "all"])}
ARG = {"argmax": 0, "argmin": 1}
SCAN = {"cumsum": 0, "cumprod": 1}

STATUS = {0: "ok", 1: "invalid argument", 2: "shape mismatch", 3: "unsupported dtype", 4: "axis out of range",
          5: "allocation failed", 6: "CUDA error", 7: "device error", 8: "unsupported"}


class AcdError(RuntimeError):
    """A non-OK status from the C ABI; .status holds the code."""

    def __init__(self, status, message):
        super().__init__(message)
        self.status = status


class Desc(ctypes.Structure):
    _fields_ = [
        ("data", ctypes.c_void_p),
        ("offset", ctypes.c_int64),
        ("shape", ctypes.c_int64 * MAX_DIMS),
        ("stride", ctypes.c_int64 * MAX_DIMS),
        ("ndim", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
    ]


def make_desc(ptr, dtype_code, shape, strides, offset=0):
    d = Desc()
    d.data = ptr
    d.offset = offset
    d.ndim = len(shape)
    d.dtype = dtype_code
    for i, (s, st) in enumerate(zip(shape, strides)):
        d.shape[i] = s
        d.stride[i] = st
    return d


_lib = None


def _bind(lib):
    P = ctypes.POINTER
    dp = P(Desc)
    vp = ctypes.c_void_p
    i32, i64, u32, f64 = ctypes.c_int32, ctypes.c_int64, ctypes.c_uint32, ctypes.c_double
    sigs = {
        "acd_version": ([], ctypes.c_char_p),
        "acd_last_error": ([], ctypes.c_char_p),
        "acd_gpu_available": ([], i32),
        "acd_gpu_info": ([ctypes.c_char_p, i64], i64),
        "acd_gpu_memory_available": ([], f64),
        "acd_ctx_create": ([ctypes.c_int, P(vp)], i32),
        "acd_ctx_destroy": ([vp], i32),
        "acd_ctx_set_allocator": ([vp, vp, vp, vp], i32),
        "acd_ctx_check": ([vp, vp, P(i32)], i32),
        "acd_ctx_set_scan_fault": ([vp, i64, i64], i32),
        "acd_broadcast_shape": ([i32, P(i64), i32, P(i64), P(i32), P(i64)], i32),
        "acd_broadcast_strides": ([i32, P(i64), P(i64), i32, P(i64), P(i64)], i32),
        "acd_unary": ([vp, i32, dp, dp, vp], i32),
        "acd_binary": ([vp, i32, dp, dp, dp, vp], i32),
        "acd_scalar": ([vp, i32, dp, dp, f64, vp], i32),
        "acd_fused": ([vp, i32, dp, dp, dp, f64, vp], i32),
        "acd_copy": ([vp, dp, dp, vp], i32),
        "acd_convert": ([vp, dp, dp, vp], i32),
        "acd_slice_desc": ([dp, P(i64), P(i64), dp], i32),
        "acd_fill": ([vp, dp, ctypes.c_double, vp], i32),
        "acd_mask_fill": ([vp, dp, dp, ctypes.c_double, vp], i32),
        "acd_concat": ([vp, dp, ctypes.POINTER(dp), i32, i32, vp], i32),
        "acd_stack": ([vp, dp, ctypes.POINTER(dp), i32, i32, vp], i32),
        "acd_repeat": ([vp, dp, dp, P(i64), vp], i32),
        "acd_pad": ([vp, dp, dp, P(i64), i32, ctypes.c_double, vp], i32),
        "acd_rand": ([vp, dp, i32, ctypes.c_double, ctypes.c_double, ctypes.c_uint64, ctypes.c_uint64, vp], i32),
        "acd_reduce": ([vp, i32, dp, dp, u32, vp], i32),
        "acd_sum_var": ([vp, dp, dp, dp, vp], i32),
        "acd_arg_reduce": ([vp, i32, dp, dp, dp, i32, i32, vp], i32),
        "acd_scan": ([vp, i32, dp, dp, i32, vp], i32),
        "acd_softmax": ([vp, dp, dp, i32, vp], i32),
        "acd_stats_partial": ([vp, vp, dp, vp], i32),
        "acd_argmax_keys": ([vp, vp, dp, i32, i64, vp], i32),
        "acd_argmax_keys_decode": ([vp, dp, vp, i32, vp], i32),
        "acd_shard_exchange_init": ([vp, vp, i64, i32, vp], i32),
        "acd_chain5_stats": ([vp, dp, dp, ctypes.POINTER(dp), vp, vp, vp], i32),
        "acd_shard_finish": ([vp, vp, i64, i32, dp, vp, i32, vp], i32),
        "acd_fused_stats_keys": ([vp, dp, dp, f64, vp, vp, i64, vp], i32),
        "acd_permute_fused_stats_keys": ([vp, dp, dp, dp, f64, vp, vp, i64, vp], i32),
        "acd_copy_fanout": ([vp, vp, vp, vp, i64, vp], i32),
        "acd_selftest_fastdiv": ([u32, u32, P(u32)], i32),
        "acd_selftest_collapse": ([dp, dp, P(i64), P(i64), P(i64)], i32),
    }
    for name, (args, res) in sigs.items():
        f = getattr(lib, name)
        f.argtypes = args
        f.restype = res


def lib():
    """Loads the library once; raises ImportError when it is not built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError("libacediar_b200.so not built: run `python acedia-r_b200/build.py` "
                              "(expected at %s)" % LIB_PATH)
        l = ctypes.CDLL(LIB_PATH)
        _bind(l)
        _lib = l
    return _lib


def check(status, what=""):
    if status != 0:
        msg = lib().acd_last_error().decode(errors="replace")
        raise AcdError(status, "%s%s (%s)" % (what + ": " if what else "", msg, STATUS.get(status, status)))


def broadcast_shape(a, b):
    """The C ABI's broadcast rule (host only, needs no GPU)."""
    L = lib()
    A = (ctypes.c_int64 * max(1, len(a)))(*a)
    B = (ctypes.c_int64 * max(1, len(b)))(*b)
    nd = ctypes.c_int32()
    out = (ctypes.c_int64 * MAX_DIMS)()
    check(L.acd_broadcast_shape(len(a), A, len(b), B, ctypes.byref(nd), out), "broadcast")
    return tuple(out[i] for i in range(nd.value))


def broadcast_strides(shape, strides, out_shape):
    L = lib()
    S = (ctypes.c_int64 * max(1, len(shape)))(*shape)
    T = (ctypes.c_int64 * max(1, len(strides)))(*strides)
    O = (ctypes.c_int64 * max(1, len(out_shape)))(*out_shape)
    R = (ctypes.c_int64 * max(1, len(out_shape)))()
    check(L.acd_broadcast_strides(len(shape), S, T, len(out_shape), O, R), "broadcast")
    return tuple(R[i] for i in range(len(out_shape)))
