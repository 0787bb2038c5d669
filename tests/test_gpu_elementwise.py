"""Elementwise, broadcast and strided ops: CUDA path vs the oracle.

Tolerances (per the parity contract): bit-exact for + - * / (both sides
correctly rounded), max/min, abs/floor/ceil/round/relu/neg, comparisons and
every integer op; <= 2 ulp for exp/log/sqrt/tanh/sigmoid/erf/sin/cos/pow.
"""
import numpy as np
import torch
import pytest

import oracle
from helpers import assert_exact, assert_ulp

pytestmark = pytest.mark.gpu

EXACT_UNARY = {"abs", "floor", "ceil", "round", "relu", "neg", "square", "copy", "sqrt"}
SIZES = [1, 3, 7, 1000, 4099, 1 << 16, (1 << 20) + 5]


def _data(op, n, dt, rng):
    if op in ("log", "sqrt"):
        return rng.uniform(1e-3, 50.0, n).astype(dt)
    if op in ("exp",):
        return rng.uniform(-60.0, 60.0, n).astype(dt)
    return rng.normal(0.0, 3.0, n).astype(dt)


@pytest.mark.parametrize("dt", [np.float32, np.float64])
@pytest.mark.parametrize("op", ["exp", "log", "sqrt", "abs", "floor", "ceil", "round", "erf", "tanh", "sigmoid",
                                "relu", "sin", "cos"])
def test_unary_contiguous(acd, op, dt):
    rng = np.random.default_rng(11)
    for n in SIZES:
        x = _data(op, n, dt, rng)
        t = acd.as_tensor(x, dtype="float" if dt == np.float32 else "double")
        got = getattr(acd, {"ceil": "ceiling"}.get(op, op))(t).as_array()
        exp = oracle.unary(op, x)
        if op in EXACT_UNARY:
            assert_exact(got, exp, "%s n=%d" % (op, n))
        else:
            assert_ulp(got, exp, 2, "%s n=%d" % (op, n))


@pytest.mark.parametrize("dt,name", [(np.float32, "float"), (np.float64, "double")])
def test_unary_on_views(acd, dt, name):
    rng = np.random.default_rng(5)
    x = rng.normal(size=(37, 21, 5)).astype(dt)
    t = acd.as_tensor(x, dtype=name)
    for perm in ([2, 1, 3], [3, 1, 2], [3, 2, 1], [1, 3, 2]):
        v = acd.permute_view(t, perm)
        got = acd.exp(v).as_array()
        exp = oracle.unary("exp", np.transpose(x, [p - 1 for p in perm]))
        assert_ulp(got, exp, 2, "exp perm %s" % perm)
        got = acd.abs(v).as_array()
        assert_exact(got, np.abs(np.transpose(x, [p - 1 for p in perm])), "abs perm %s" % perm)


def _mk(acd, a, name):
    return acd.as_tensor(a, dtype=name)


OPS = {"add": lambda a, b: a + b, "sub": lambda a, b: a - b, "mul": lambda a, b: a * b,
       "div": lambda a, b: a / b, "max": None, "min": None, "pow": lambda a, b: a ** b,
       "gt": lambda a, b: a > b, "lt": lambda a, b: a < b, "eq": lambda a, b: a == b,
       "ne": lambda a, b: a != b, "ge": lambda a, b: a >= b, "le": lambda a, b: a <= b}
SHAPE_PAIRS = [((1000,), (1000,)), ((64, 33), (64, 33)), ((8192, 8), (1, 8)), ((64, 96), (64, 1)), ((5, 6, 7), (5, 6)),
               ((2, 1, 3), (1, 4, 1)), ((128, 256), (256,)), ((4099, 3), (1, 3)), ((33, 17), (1,))]


def _bin(acd, op, ta, tb):
    if op == "max":
        return acd.pmax(ta, tb)
    if op == "min":
        return acd.pmin(ta, tb)
    return OPS[op](ta, tb)


@pytest.mark.parametrize("dt,name", [(np.float32, "float"), (np.float64, "double")])
@pytest.mark.parametrize("op", list(OPS))
def test_binary_broadcast(acd, op, dt, name):
    rng = np.random.default_rng(23)
    for sa, sb in SHAPE_PAIRS:
        a = rng.normal(size=sa).astype(dt)
        b = rng.normal(size=sb).astype(dt)
        if op == "pow":
            a = np.abs(a) + np.asarray(0.5, dt)
        if op in ("eq", "ne", "ge", "le"):
            b = np.where(rng.random(sb) < 0.5, b, np.asarray(a.reshape(-1, order="F")[:b.size].reshape(sb, order="F")))
        got = _bin(acd, op, _mk(acd, a, name), _mk(acd, b, name)).as_array()
        exp = oracle.binary(op, a, b)
        if op in ("gt", "lt", "eq", "ne", "ge", "le"):
            assert got.dtype == np.bool_
            assert_exact(got.astype(np.uint8), exp, "%s %s %s" % (op, sa, sb))
        elif op == "pow":
            assert_ulp(got, exp, 2, "%s %s %s" % (op, sa, sb))
        else:
            assert_exact(got, exp, "%s %s %s" % (op, sa, sb))


@pytest.mark.parametrize("dt,name", [(np.int32, "int32"), (np.int64, "int64")])
def test_integer_ops_exact(acd, dt, name):
    rng = np.random.default_rng(2)
    a = rng.integers(-1000, 1000, size=(300, 7)).astype(dt)
    b = rng.integers(-1000, 1000, size=(1, 7)).astype(dt)
    ta, tb = _mk(acd, a, name), _mk(acd, b, name)
    assert_exact((ta + tb).as_array(), a + b, "add")
    assert_exact((ta - tb).as_array(), a - b, "sub")
    assert_exact((ta * tb).as_array(), a * b, "mul")
    assert_exact((ta > tb).as_array(), a > b, "gt")
    assert_exact(acd.pmax(ta, tb).as_array(), np.maximum(a, b), "max")


@pytest.mark.parametrize("dt,name", [(np.float32, "float"), (np.float64, "double")])
def test_scalar_ops(acd, dt, name):
    rng = np.random.default_rng(9)
    x = rng.normal(size=(4097,)).astype(dt)
    t = _mk(acd, x, name)
    for op, fn in [("add", lambda: t + 0.3), ("sub", lambda: t - 0.3), ("mul", lambda: t * 0.5),
                   ("div", lambda: t / 3.0), ("rsub", lambda: 2.0 - t), ("rdiv", lambda: 2.0 / t)]:
        assert_exact(fn().as_array(), oracle.scalar(op, x, {"rsub": 2.0, "rdiv": 2.0, "add": 0.3, "sub": 0.3,
                                                             "mul": 0.5, "div": 3.0}[op]), op)
    # x^2 is x*x (bit-exact), unary minus is exact
    assert_exact((t ** 2).as_array(), (x * x).astype(dt), "x^2")
    assert_exact((-t).as_array(), -x, "neg")
    assert_ulp((acd.abs(t) ** 0.75).as_array(), oracle.scalar("pow", np.abs(x), 0.75), 2, "x^0.75")
    for op in ("gt", "lt", "eq", "ne", "ge", "le"):
        got = {"gt": t > 0.1, "lt": t < 0.1, "eq": t == float(x[5]), "ne": t != float(x[5]), "ge": t >= 0.1,
               "le": t <= 0.1}[op].as_array()
        s = float(x[5]) if op in ("eq", "ne") else 0.1
        assert_exact(got.astype(np.uint8), oracle.scalar(op, x, s), op)


@pytest.mark.parametrize("dt,name", [(np.float32, "float"), (np.float64, "double")])
def test_misaligned_views(acd, dt, name):
    """Views starting at odd element offsets take the scalar head/tail path."""
    import acediar.tensor as T
    rng = np.random.default_rng(4)
    x = rng.normal(size=10007).astype(dt)
    base = _mk(acd, x, name)
    for off in (1, 2, 3, 5):
        n = 10007 - off - 3
        v = T.gpuTensor(base.storage, (n,), name, (1,), off)
        assert_ulp(acd.exp(v).as_array(), oracle.unary("exp", x[off:off + n]), 2, "exp off=%d" % off)
        w = T.gpuTensor(base.storage, (n,), name, (1,), off + 1)
        assert_exact((v + w).as_array(), x[off:off + n] + x[off + 1:off + 1 + n], "add off=%d" % off)


@pytest.mark.parametrize("dt,name", [(np.float32, "float"), (np.float64, "double")])
def test_fused_chains_bit_identical(acd, dt, name):
    rng = np.random.default_rng(8)
    x = rng.normal(size=(333, 65)).astype(dt)
    t = _mk(acd, x, name)
    fused = acd.fused("scale_add_exp_neg_square", t, p0=0.5).as_array()
    stepwise = (t * 0.5 + acd.exp(-(t ** 2))).as_array()
    assert_exact(fused, stepwise, "fused vs op-by-op")
    # exp is within 2 ulp of the oracle's; the final add can cancel, so the
    # bound is 2 ulp of the larger addend plus one rounding of the result
    ref = oracle.gauss_chain(x, 0.5)
    bound = 2 * np.spacing(np.maximum(np.abs(x * dt(0.5)), np.exp(-(x * x)).astype(dt))) + np.spacing(np.abs(ref))
    assert np.all(np.abs(fused.astype(np.float64) - ref) <= bound), "fused vs oracle" 
    r = rng.uniform(-1, 1, size=(1, 65)).astype(dt)
    tr = _mk(acd, r, name)
    assert_exact(acd.fused("add_relu", t, tr).as_array(), acd.relu(t + tr).as_array(), "add_relu")
    assert_exact(acd.fused("tanh_scale", t, p0=2.0).as_array(), (acd.tanh(t) * 2.0).as_array(), "tanh_scale")


@pytest.mark.parametrize("name,dt", [("float", np.float32), ("int32", np.int32)])
def test_copy_transpose_tma_shapes(acd, name, dt):
    """4-byte transposes whose strides suit the TMA path: full and ragged
    64x64 tiles, a batch axis, the strided-views permutation at reduced size,
    and extents just past a tile edge (boxes wholly outside the tensor)."""
    rng = np.random.default_rng(11)
    cases = [((64, 64), (2, 1)), ((256, 132), (2, 1)), ((1000, 2052), (2, 1)), ((68, 100, 3), (2, 1, 3)),
             ((64, 72, 5), (2, 1, 3)), ((72, 5, 64), (3, 2, 1)), ((256, 512, 64), (3, 1, 2)),
             ((96, 4, 260), (3, 2, 1)), ((100, 68), (2, 1)), ((260, 68), (2, 1))]
    for shape, perm in cases:
        x = (rng.normal(size=shape) * 1000).astype(dt)
        t = acd.as_tensor(x, dtype=name)
        got = acd.contiguous(acd.permute_view(t, list(perm))).as_array()
        assert_exact(got, np.transpose(x, [p - 1 for p in perm]), "%s perm %s" % (shape, perm))
    # status word clean: no pipeline wait expired
    acd.check_device_status()


@pytest.mark.parametrize("name,dt", [("float", np.float32), ("double", np.float64), ("int32", np.int32),
                                     ("int64", np.int64), ("bool", np.bool_)])
def test_copy_permutations_bit_exact(acd, name, dt):
    rng = np.random.default_rng(1)
    for shape in [(3, 4), (37, 65), (64, 64), (130, 67), (5, 6, 7), (33, 64, 3), (16, 8, 4, 2)]:
        x = (rng.normal(size=shape) * 100).astype(dt) if dt != np.bool_ else rng.random(shape) < 0.5
        t = acd.as_tensor(x, dtype=name)
        import itertools
        for perm in itertools.permutations(range(1, len(shape) + 1)):
            got = acd.contiguous(acd.permute_view(t, list(perm))).as_array()
            assert_exact(got, np.transpose(x, [p - 1 for p in perm]), "%s perm %s" % (shape, perm))


def test_copy_fanout(acd):
    """acd_copy_fanout: one source into one or two destinations, bit for bit;
    misaligned buffers and sizes are refused before any launch."""
    import ctypes
    import acediar._lib as L
    from acediar.tensor import context
    src = torch.randint(-2 ** 31, 2 ** 31 - 1, (1 << 20,), dtype=torch.int32, device="cuda")
    d0 = torch.zeros_like(src)
    d1 = torch.zeros_like(src)
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    lib = L.lib()
    assert lib.acd_copy_fanout(context(), ctypes.c_void_p(d0.data_ptr()), ctypes.c_void_p(d1.data_ptr()),
                               ctypes.c_void_p(src.data_ptr()), src.numel() * 4, s) == 0
    assert torch.equal(d0, src) and torch.equal(d1, src)
    d2 = torch.zeros_like(src)
    assert lib.acd_copy_fanout(context(), ctypes.c_void_p(d2.data_ptr()), None, ctypes.c_void_p(src.data_ptr()),
                               4096 * 4, s) == 0
    assert torch.equal(d2[:4096], src[:4096]) and int(d2[4096:].abs().sum()) == 0
    assert lib.acd_copy_fanout(context(), ctypes.c_void_p(d2.data_ptr() + 4), None, ctypes.c_void_p(src.data_ptr()),
                               64, s) != 0
    assert lib.acd_copy_fanout(context(), ctypes.c_void_p(d2.data_ptr()), None, ctypes.c_void_p(src.data_ptr()),
                               40, s) != 0
