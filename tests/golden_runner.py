"""Runs one golden case (tests/golden/reference_cases.json) through either
the CPU oracle or the CUDA path (the acediar mirror of the R API)."""
import numpy as np

import oracle

_OPS = {"+": "add", "-": "sub", "*": "mul", "/": "div", "==": "eq", "!=": "ne", "<": "lt", "<=": "le", ">": "gt",
        ">=": "ge"}
_NP = {"float": np.float32, "double": np.float64}


def _host(inp):
    return np.asarray(inp["data"], dtype=_NP[inp["dtype"]]).reshape(inp["shape"], order="F")


def _transposed_view(a):
    """The transpose view of a 2-D column-major array (strides swapped)."""
    v = oracle.View.of(a)
    return oracle.View(v.buf, (v.shape[1], v.shape[0]), (v.strides[1], v.strides[0]))


def run_oracle(case):
    op, args = case["op"], case["args"]
    xs = [_host(i) for i in case["inputs"]]
    if op in ("sum", "mean", "max", "min", "prod", "var"):
        x = _transposed_view(xs[0]) if args.get("transpose") else oracle.View.of(xs[0])
        axis = args.get("axis")
        for a in axis or []:
            if not (isinstance(a, int) and 1 <= a <= len(x.shape)):
                raise ValueError("axis must be a vector of positive integers")
        r = oracle.reduce(op, x, None if axis is None else [a - 1 for a in axis])
        return np.asarray(r)
    if op in ("which.max", "which.min"):
        x = _transposed_view(xs[0]) if args.get("transpose") else oracle.View.of(xs[0])
        return oracle.arg_reduce("argmax" if op == "which.max" else "argmin", x, None, True)
    if op in ("any", "all"):
        x = _transposed_view(xs[0]) if args.get("transpose") else oracle.View.of(xs[0])
        return np.asarray(oracle.reduce(op, x))
    if op in ("cumsum", "cumprod"):
        return oracle.scan(op, xs[0])
    if op in _OPS:
        if "scalar" in args:
            return oracle.scalar(_OPS[op], xs[0], args["scalar"])
        a = _transposed_view(xs[0]) if args.get("transpose_first") else xs[0]
        return oracle.binary(_OPS[op], a, xs[1])
    if op in ("tanh", "sigmoid", "relu"):
        return oracle.unary(op, xs[0])
    if op == "softmax":
        return oracle.softmax(xs[0])
    if op == "permute":
        v = oracle.View.of(xs[0])
        perm = [p - 1 for p in args["perm"]]
        return oracle.copy(oracle.View(v.buf, [v.shape[p] for p in perm], [v.strides[p] for p in perm]))
    if op == "concat":
        return oracle.concat(xs, args["axis"] - 1)
    if op == "stack":
        return oracle.stack(xs, args["axis"] - 1)
    if op == "repeat":
        return oracle.repeat(xs[0], args["reps"])
    if op == "pad":
        pw = np.asarray(args["pad_width"]).reshape(-1, 2)
        return oracle.pad(xs[0], pw[:, 0], pw[:, 1])
    if op in ("subset", "assign"):
        sl = tuple(slice(None) if i is None else (i - 1 if isinstance(i, int) else slice(i[0] - 1, i[-1]))
                   for i in args["index"])
        if op == "subset":
            return xs[0][sl]
        y = xs[0].copy()
        if "value" in args:
            y[sl] = args["value"]
        elif "vector" in args:
            y[sl] = np.asarray(args["vector"]).reshape(y[sl].shape, order="F")
        else:
            y[sl] = xs[1]
        return y
    if op == "diff":
        return oracle.diff(xs[0], args.get("lag", 1), args.get("differences", 1))
    if op == "range":
        v = oracle.View.of(xs[0])
        return np.asarray([oracle.reduce("min", v), oracle.reduce("max", v)], dtype=np.float64)
    if op == "tensor_pow":
        return oracle.binary("pow", xs[0], xs[1])
    if op == "mask_assign":
        y = xs[0].copy()
        m = np.asarray(args["mask"], dtype=bool).reshape(y.shape, order="F")
        y[m] = args["value"]
        return y
    raise KeyError(op)


def run_gpu(acd, case):
    op, args = case["op"], case["args"]
    dts = [i["dtype"] for i in case["inputs"]]
    xs = [acd.as_tensor(_host(i), dtype=d) for i, d in zip(case["inputs"], dts)]
    if op in ("sum", "mean", "max", "min", "prod", "var"):
        x = acd.transpose_view(xs[0]) if args.get("transpose") else xs[0]
        f = getattr(acd, op)
        axis = args.get("axis")
        r = f(x, axis=axis, keep_dims=args.get("keep_dims", False))
        return np.asarray(r.as_array() if hasattr(r, "as_array") else r)
    if op in ("which.max", "which.min"):
        x = acd.transpose_view(xs[0]) if args.get("transpose") else xs[0]
        return acd.which_max(x) if op == "which.max" else acd.which_min(x)
    if op in ("any", "all"):
        x = acd.transpose_view(xs[0]) if args.get("transpose") else xs[0]
        r = getattr(acd, op)(x)
        return np.float64(np.nan if r is None else float(r))
    if op in ("cumsum", "cumprod"):
        return getattr(acd, op)(xs[0]).as_array()
    if op in _OPS:
        a = acd.transpose_view(xs[0]) if args.get("transpose_first") else xs[0]
        b = args["scalar"] if "scalar" in args else xs[1]
        r = {"+": lambda: a + b, "-": lambda: a - b, "*": lambda: a * b, "/": lambda: a / b,
             "==": lambda: a == b, "!=": lambda: a != b, "<": lambda: a < b, "<=": lambda: a <= b,
             ">": lambda: a > b, ">=": lambda: a >= b}[op]()
        return r.as_array()
    if op in ("tanh", "sigmoid", "relu"):
        return getattr(acd, op)(xs[0]).as_array()
    if op == "softmax":
        return acd.softmax(xs[0]).as_array()
    if op == "permute":
        return acd.contiguous(acd.permute_view(xs[0], args["perm"])).as_array()
    if op == "concat":
        return acd.concat_tensor(xs, axis=args["axis"]).as_array()
    if op == "stack":
        return acd.stack_tensor(xs, axis=args["axis"]).as_array()
    if op == "repeat":
        return acd.repeat_tensor(xs[0], args["reps"]).as_array()
    if op == "pad":
        return acd.pad_tensor(xs[0], args["pad_width"]).as_array()
    if op == "subset":
        r = acd.subset(xs[0], *[None if i is None else i for i in args["index"]])
        return np.asarray(r.as_array() if hasattr(r, "as_array") else r)
    if op == "assign":
        if "value" in args:
            v = args["value"]
        elif "vector" in args:
            v = np.asarray(args["vector"], dtype=np.float64)
        else:
            v = xs[1]
        return acd.assign(xs[0], *args["index"], value=v).as_array()
    if op == "diff":
        return acd.diff(xs[0], lag=args.get("lag", 1), differences=args.get("differences", 1)).as_array()
    if op == "range":
        return np.asarray(acd.range_(xs[0]), dtype=np.float64)
    if op == "tensor_pow":
        return acd.tensor_pow(xs[0], xs[1]).as_array()
    if op == "mask_assign":
        return acd.assign(xs[0], np.asarray(args["mask"], dtype=bool), value=args["value"]).as_array()
    raise KeyError(op)


def expected_of(case):
    e = case["expected"]
    return np.asarray(e["data"], dtype=np.float64).reshape(e["shape"], order="F")
