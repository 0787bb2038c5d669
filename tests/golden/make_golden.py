"""Generates tests/golden/reference_cases.json.

The cases are the known-answer tests of the reference's testthat suite
(tests/testthat/*.R of acediaR), transcribed as inputs plus the base-R
expression each test compares against.  The expected values are computed
here with numpy on the logical (column-major) arrays, following the R
expression named in each case — independently of the C oracle and of the
CUDA library, which are both checked against this file.

Run:  python tests/golden/make_golden.py
"""
import json
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def col(a):
    """Flat column-major list of a logical array."""
    return np.asarray(a).reshape(-1, order="F").tolist()


def rmatrix(data, nrow, ncol):
    return np.asarray(data, dtype=np.float64).reshape((nrow, ncol), order="F")


def rarray(data, dims):
    return np.asarray(data, dtype=np.float64).reshape(dims, order="F")


def t_in(a, dtype="float"):
    a = np.asarray(a, dtype=np.float64)
    return {"data": col(a), "shape": list(a.shape) if a.ndim else [1], "dtype": dtype}


def r_sweep(x, margin, stats, fn):
    """R's sweep(x, MARGIN, STATS, FUN) for the margins used by the tests."""
    x = np.asarray(x)
    stats = np.asarray(stats)
    shape = [1] * x.ndim
    for i, m in enumerate(margin):
        shape[m - 1] = x.shape[m - 1]
    s = stats.reshape([x.shape[m - 1] for m in margin], order="F")
    # place the stats on the margin axes, singleton elsewhere
    full = np.empty(x.shape)
    it = np.nditer(x, flags=["multi_index"])
    for _ in it:
        idx = it.multi_index
        full[idx] = s[tuple(idx[m - 1] for m in margin)]
    return fn(x, full)


cases = []


def case(cid, source, op, inputs, expected, **args):
    e = np.asarray(expected)
    cases.append({
        "id": cid, "source": source, "op": op, "inputs": inputs, "args": args,
        "expected": {"data": col(e) if e.ndim else [e.item()], "shape": list(e.shape) if e.ndim else [1]},
    })


def case_error(cid, source, op, inputs, pattern, **args):
    cases.append({"id": cid, "source": source, "op": op, "inputs": inputs, "args": args, "error": pattern})


AX = "tests/testthat/test-axis-aware-reductions.R"
m12 = rmatrix(np.arange(1, 13), 3, 4)
a24 = rarray(np.arange(1, 25), (2, 3, 4))
mext = rmatrix([3, 1, 4, 1, 5, 9, 2, 6, 5, 3, 5, 8], 3, 4)
mprod = rmatrix([1, 2, 1, 2, 1, 2, 1, 2, 1, 2, 1, 2], 3, 4)

case("sum_axis1", AX + ":21-36", "sum", [t_in(m12)], m12.sum(axis=0), axis=[1])           # colSums
case("sum_axis2", AX + ":38-42", "sum", [t_in(m12)], m12.sum(axis=1), axis=[2])           # rowSums
case("sum_axis1_keep", AX + ":44-47", "sum", [t_in(m12)], m12.sum(axis=0, keepdims=True), axis=[1], keep_dims=True)
case("sum_axis2_keep", AX + ":49-51", "sum", [t_in(m12)], m12.sum(axis=1, keepdims=True), axis=[2], keep_dims=True)
case("sum_axes12", AX + ":54-62", "sum", [t_in(a24)], a24.sum(axis=(0, 1)), axis=[1, 2])  # apply(x, 3, sum)
case("sum_axes12_keep", AX + ":64-67", "sum", [t_in(a24)], a24.sum(axis=(0, 1), keepdims=True), axis=[1, 2],
     keep_dims=True)
case("sum_global", AX + ":70-78", "sum", [t_in(m12)], m12.sum())
case("mean_axis1", AX + ":84-93", "mean", [t_in(m12)], m12.mean(axis=0), axis=[1])       # colMeans
case("mean_axis2", AX + ":95-99", "mean", [t_in(m12)], m12.mean(axis=1), axis=[2])       # rowMeans
case("max_axis1", AX + ":107-116", "max", [t_in(mext)], mext.max(axis=0), axis=[1])
case("max_axis2", AX + ":118-122", "max", [t_in(mext)], mext.max(axis=1), axis=[2])
case("min_axis1", AX + ":125-133", "min", [t_in(mext)], mext.min(axis=0), axis=[1])
case("min_axis2", AX + ":135-139", "min", [t_in(mext)], mext.min(axis=1), axis=[2])
case("prod_axis1", AX + ":145-155", "prod", [t_in(mprod)], mprod.prod(axis=0), axis=[1])
case("prod_axis2", AX + ":157-161", "prod", [t_in(mprod)], mprod.prod(axis=1), axis=[2])
v = col(mext)
case("argmax_global", AX + ":167-176", "which.max", [t_in(mext)], int(np.argmax(v)) + 1)
case("argmin_global", AX + ":167-176", "which.min", [t_in(mext)], int(np.argmin(v)) + 1)
case("sum_transposed_axis1", AX + ":215-224", "sum", [t_in(m12)], m12.T.sum(axis=0), axis=[1], transpose=True)
case("sum_transposed_axis2", AX + ":226-228", "sum", [t_in(m12)], m12.T.sum(axis=1), axis=[2], transpose=True)
case("sum_double", AX + ":244-248", "sum", [t_in(m12, "double")], m12.sum(axis=0), axis=[1])
case("sum_1d_axis", AX + ":254-261", "sum", [t_in([1, 2, 3, 4, 5])], np.float64(15), axis=[1])
case("sum_single_axis", AX + ":263-266", "sum", [t_in([42])], np.float64(42), axis=[1])
case("var_axis1", AX + ":273-279", "var", [t_in(m12)], m12.var(axis=0, ddof=1), axis=[1])
case("var_axis2", AX + ":281-282", "var", [t_in(m12)], m12.var(axis=1, ddof=1), axis=[2])
for a in (5, 0, -1, 1.5):
    case_error("axis_invalid_%s" % str(a).replace(".", "_").replace("-", "m"), AX + ":192-207", "sum",
               [t_in(m12)], "axis must be a vector of positive integers", axis=[a])

EX = "tests/testthat/test-range-extrema-helpers.R"
for cid, data, dt, line in [("wmax_1d", [3, 1, 4, 1, 5, 9, 2, 6], "float", "118-128"),
                            ("wmax_f32", [1.5, 4.9, 2.7, 0.3, 1.1], "float", "130-145"),
                            ("wmax_f64", [1.5, 4.9, 2.7, 0.3, 1.1], "double", "130-145"),
                            ("wmax_single", [42], "float", "158-162"),
                            ("wmax_ties", [5, 2, 5, 1, 5, 3], "float", "164-169"),
                            ("wmax_negative", [-5, -1, -10, -3, -7], "float", "171-175"),
                            ("wmax_all_same", [3.14] * 5, "float", "177-181")]:
    case(cid, EX + ":" + line, "which.max", [t_in(data, dt)], int(np.argmax(data)) + 1)
case("wmax_matrix", EX + ":147-155", "which.max", [t_in(mext)], int(np.argmax(col(mext))) + 1)
m33 = rmatrix([1, 8, 3, 2, 9, 4, 5, 1, 6], 3, 3)
case("wmax_transposed", EX + ":185-195", "which.max", [t_in(m33)], int(np.argmax(col(m33.T))) + 1, transpose=True)
for cid, data, dt, line in [("wmin_1d", [3, 1, 4, 1, 5, 9, 2, 6], "float", "203-212"),
                            ("wmin_f32", [1.5, 0.3, 2.7, 4.9, 1.1], "float", "214-229"),
                            ("wmin_f64", [1.5, 0.3, 2.7, 4.9, 1.1], "double", "214-229"),
                            ("wmin_ties", [5, 2, 5, 2, 3, 2], "float", "248-254")]:
    case(cid, EX + ":" + line, "which.min", [t_in(data, dt)], int(np.argmin(data)) + 1)
case("wmin_matrix", EX + ":231-240", "which.min", [t_in(mext)], int(np.argmin(col(mext))) + 1)

CU = "tests/testthat/test-cumulative-operations.R"
case("cumsum_1d", CU + ":25-37", "cumsum", [t_in([1, 2, 3, 4, 5])], np.cumsum([1, 2, 3, 4, 5.0]))
case("cumsum_f32", CU + ":39-48", "cumsum", [t_in([1.5, 2.7, 3.1, 4.9])], np.cumsum([1.5, 2.7, 3.1, 4.9]))
case("cumsum_f64", CU + ":50-55", "cumsum", [t_in([1.5, 2.7, 3.1, 4.9], "double")],
     np.cumsum([1.5, 2.7, 3.1, 4.9]))
case("cumsum_matrix", CU + ":58-69", "cumsum", [t_in(m12)],
     np.cumsum(col(m12)).reshape((3, 4), order="F"))
case("cumsum_single", CU + ":71-75", "cumsum", [t_in([42])], np.array([42.0]))
case("cumsum_negative", CU + ":88-96", "cumsum", [t_in([-1, 2, -3, 4, -5])], np.cumsum([-1, 2, -3, 4, -5.0]))
case("cumprod_1d", CU + ":99-111", "cumprod", [t_in([1, 2, 1.5, 1.2, 1.1])], np.cumprod([1, 2, 1.5, 1.2, 1.1]))
case("cumprod_f32", CU + ":113-122", "cumprod", [t_in([1.1, 1.2, 1.05, 0.9])], np.cumprod([1.1, 1.2, 1.05, 0.9]))
case("cumprod_f64", CU + ":124-129", "cumprod", [t_in([1.1, 1.2, 1.05, 0.9], "double")],
     np.cumprod([1.1, 1.2, 1.05, 0.9]))
mcp = rmatrix([1, 1.1, 1.2, 0.9, 1.05, 1.15], 2, 3)
case("cumprod_matrix", CU + ":132-143", "cumprod", [t_in(mcp)], np.cumprod(col(mcp)).reshape((2, 3), order="F"))
case("cumprod_single", CU + ":145-150", "cumprod", [t_in([3.14])], np.array([3.14]))

CO = "tests/testthat/test-comparison-operators.R"
a5, b5 = np.array([1, 2, 3, 2, 1.0]), np.array([1, 3, 3, 2, 2.0])
for op, f in [("==", np.equal), ("!=", np.not_equal), ("<", np.less), ("<=", np.less_equal), (">", np.greater),
              (">=", np.greater_equal)]:
    case("cmp_%s" % {"==": "eq", "!=": "ne", "<": "lt", "<=": "le", ">": "gt", ">=": "ge"}[op], CO + ":25-250", op,
         [t_in(a5), t_in(b5)], f(a5, b5).astype(np.float64))
    case("cmp_scalar_%s" % {"==": "eq", "!=": "ne", "<": "lt", "<=": "le", ">": "gt", ">=": "ge"}[op],
         CO + ":40-250", op, [t_in(a5)], f(a5, 2.0).astype(np.float64), scalar=2.0)
d27 = np.array([1.5, 2.7, 3.1, 2.7])
case("cmp_eq_f32_2_7", CO + ":51-59", "==", [t_in(d27)], (np.float32(d27) == np.float32(2.7)).astype(float),
     scalar=2.7)
case("cmp_eq_f64_2_7", CO + ":61-65", "==", [t_in(d27, "double")], (d27 == 2.7).astype(float), scalar=2.7)
m6 = rmatrix([1, 2, 3, 4, 5, 6], 2, 3)
v3 = np.array([2, 3, 4.0])
case("cmp_bcast_gt", CO + ":273-285", ">", [t_in(m6), t_in(v3)], r_sweep(m6, [2], v3, np.greater).astype(float))
case("cmp_bcast_eq", CO + ":287-292", "==", [t_in(m6), t_in(v3)], r_sweep(m6, [2], v3, np.equal).astype(float))

BR = "tests/testthat/test-comprehensive-broadcasting.R"
v10 = np.array([10, 20, 30.0])
case("bcast_mat_vec", BR + ":25-37", "+", [t_in(m6), t_in(v10)], r_sweep(m6, [2], v10, np.add))
case("bcast_vec_mat", BR + ":39-41", "+", [t_in(v10), t_in(m6)], r_sweep(m6, [2], v10, np.add))
case("bcast_3d_mat", BR + ":43-55", "+", [t_in(a24), t_in(m6)], r_sweep(a24, [1, 2], m6, np.add))
m6b = rmatrix([10, 20, 30, 40, 50, 60], 2, 3)
case("bcast_sub", BR + ":57-76", "-", [t_in(m6b), t_in([1, 2, 3])], r_sweep(m6b, [2], np.array([1, 2, 3.0]),
                                                                           np.subtract))
ta = rarray([1, 2, 3, 4, 5, 6], (2, 1, 3))
tb = rarray([10, 20, 30, 40], (1, 4, 1))
case("bcast_multi", BR + ":264-286", "+", [t_in(ta), t_in(tb)], ta + tb)
sa = rarray([1, 2, 3, 4, 5, 6], (3, 1, 2))
sb = rarray([2, 3, 4, 5], (1, 4, 1))
case("bcast_singleton_mul", BR + ":288-306", "*", [t_in(sa), t_in(sb)], sa * sb)
r13 = rmatrix([1, 2, 3], 1, 3)
m23 = rmatrix([10, 20, 30, 40, 50, 60], 2, 3)
case("bcast_row", BR + ":308-320", "+", [t_in(r13), t_in(m23)], r13 + m23)
c31 = rmatrix([1, 2, 3], 3, 1)
m34 = rmatrix(np.arange(10, 130, 10), 3, 4)
case("bcast_col", BR + ":322-335", "+", [t_in(c31), t_in(m34)], c31 + m34)
case("bcast_transposed", BR + ":370-387", "+", [t_in(m6), t_in([10, 20])],
     r_sweep(m6.T, [2], np.array([10, 20.0]), np.add), transpose_first=True)
case_error("bcast_error_2d", BR + ":392-405", "+", [t_in(rmatrix(np.arange(1, 7), 2, 3)),
                                                     t_in(rmatrix(np.arange(1, 9), 2, 4))], "shape|dimension|broadcast")
case_error("bcast_error_3d", BR + ":406-411", "+", [t_in(rarray(np.arange(1, 13), (2, 2, 3))),
                                                     t_in(rmatrix(np.arange(1, 9), 4, 2))], "shape|dimension|broadcast")

CC = "tests/testthat/test-consolidated-core.R"
d5 = np.array([-2, -1, 0, 1, 2.0])
case("act_tanh", CC + ":369-377", "tanh", [t_in(d5)], np.tanh(d5))
case("act_sigmoid", CC + ":379-383", "sigmoid", [t_in(d5)], 1 / (1 + np.exp(-d5)))
dr = np.array([-3, -1, 0, 1, 3.0])
case("act_relu", CC + ":385-390", "relu", [t_in(dr)], np.maximum(dr, 0))
e = np.exp(d5 - d5.max())
case("softmax_1d", CC + ":392-404", "softmax", [t_in(d5)], e / e.sum())
d15 = np.array([1, 2, 3, 4, 5.0])
case("prod_global", CC + ":555-558", "prod", [t_in(d15)], np.float64(120))
case("var_global", CC + ":560-563", "var", [t_in(d15)], np.float64(d15.var(ddof=1)))

VM = "tests/testthat/test-consolidated-views-memory.R"
case("permute_231", VM + ":80-93", "permute", [t_in(a24)], np.transpose(a24, (1, 2, 0)), perm=[2, 3, 1])
case("permute_312", VM + ":98-101", "permute", [t_in(a24)], np.transpose(a24, (2, 0, 1)), perm=[3, 1, 2])
case("permute_132", VM + ":103-104", "permute", [t_in(a24)], np.transpose(a24, (0, 2, 1)), perm=[1, 3, 2])
case("permute_identity", VM + ":107-108", "permute", [t_in(a24)], a24, perm=[1, 2, 3])
m34v = rmatrix(np.arange(1, 13), 3, 4)
case("contiguous_transposed", VM + ":128-146", "permute", [t_in(m34v)], m34v.T, perm=[2, 1])

# assembly and mutation (tests/testthat/test-consolidated-core.R:497-547 and
# test-consolidated-views-memory.R:270-345).  Where a test checks only the
# shape, the expected values follow the reference kernel's definition.
a23 = rmatrix(np.arange(1, 7), 2, 3)
b23 = rmatrix(np.arange(7, 13), 2, 3)
case("concat_rbind", CC + ":497-515", "concat", [t_in(a23), t_in(b23)], np.concatenate([a23, b23], axis=0), axis=1)
case("stack_axis3", CC + ":517-520", "stack", [t_in(a23), t_in(b23)], np.stack([a23, b23], axis=2), axis=3)
m22 = rmatrix(np.arange(1, 5), 2, 2)
# repeat_kernel (src/kernels/tensor_kernels.cu:381-413): out(c) = in(c %/% reps)
case("repeat_2_1", CC + ":522-533", "repeat", [t_in(m22)], np.repeat(m22, 2, axis=0), reps=[2, 1])
# pad_tensor(t, c(1,1,1,1)): one element of 0 on every side (R/gpuTensor.R:1816-1831)
case("pad_1111", CC + ":535-541", "pad", [t_in(m22)], np.pad(m22, 1), pad_width=[1, 1, 1, 1])
m45 = rmatrix(np.arange(1, 21), 4, 5)
case("slice_row", VM + ":275-279", "subset", [t_in(m45)], m45[1, :], index=[2, None])
case("slice_col", VM + ":281-284", "subset", [t_in(m45)], m45[:, 2], index=[None, 3])
case("slice_block", VM + ":286-288", "subset", [t_in(m45)], m45[0:2, 1:4], index=[[1, 2], [2, 3, 4]])
e1 = m45.copy()
e1[1:3, 1:4] = 99
case("assign_scalar", VM + ":293-302", "assign", [t_in(m45)], e1, index=[[2, 3], [2, 3, 4]], value=99)
rep = rmatrix([101, 102, 103, 104, 105, 106], 2, 3)
e2 = m45.copy()
e2[1:3, 1:4] = rep
case("assign_tensor", VM + ":304-311", "assign", [t_in(m45), t_in(rep)], e2, index=[[2, 3], [2, 3, 4]])
e3 = m45.copy()
e3[1:3, 1:4] = rmatrix([201, 202, 203, 204, 205, 206], 2, 3)
case("assign_vector", VM + ":313-319", "assign", [t_in(m45)], e3, index=[[2, 3], [2, 3, 4]],
     vector=[201, 202, 203, 204, 205, 206])
v6 = np.array([1, 2, 3, 4, 5, 6.0])
mk = np.array([True, False, True, False, True, False])
e4 = v6.copy()
e4[mk] = 99
case("mask_vector", VM + ":323-334", "mask_assign", [t_in(v6)], e4, mask=mk.tolist(), value=99)
m34m = rmatrix(np.arange(1, 13), 3, 4)
e5 = m34m.copy()
e5[m34m > 6] = -1
case("mask_matrix", VM + ":336-344", "mask_assign", [t_in(m34m)], e5, mask=col(m34m > 6), value=-1)

# any / all (tests/testthat/test-logical-reductions.R): R's any(x != 0) / all(x != 0)
LR = "tests/testthat/test-logical-reductions.R"
for cid, lines, op, data, dtype in [
        ("any_1d_true", "25-39", "any", [0, 0, 1, 0], "float"), ("any_1d_false", "40-47", "any", [0, 0, 0, 0], "float"),
        ("any_1d_ones", "48-53", "any", [1, 1, 1, 1], "float"), ("any_f32_half", "55-64", "any", [0, 0, 0.5, 0], "float"),
        ("any_f64_zero", "66-72", "any", [0, 0, 0, 0], "double"), ("any_negative", "118-121", "any", [0, -1, 0, 0], "float"),
        ("any_small", "123-126", "any", [0, 0, 1e-10, 0], "float"),
        ("all_1d_true", "144-152", "all", [1, 2, 3, 4], "float"), ("all_1d_some_zero", "154-159", "all", [1, 0, 3, 4], "float"),
        ("all_1d_zeros", "161-166", "all", [0, 0, 0, 0], "float"), ("all_f32", "174-180", "all", [1.5, 2.7, 0.1, 3.9], "float"),
        ("all_f64_zero", "182-187", "all", [1.5, 0, 2.7, 3.9], "double"), ("all_negative", "248-251", "all", [-1, -2, -3, -4], "float"),
        ("all_mixed_zero", "253-256", "all", [-1, 2, 0, -4], "float"), ("all_small", "258-261", "all", [1e-10, 2e-10, 3e-10, 4e-10], "float")]:
    d = np.asarray(data, dtype=np.float64)
    case(cid, LR + ":" + lines, op, [t_in(d, dtype)], np.float64((d != 0).any() if op == "any" else (d != 0).all()))
mz = rmatrix([0, 0, 1, 0, 0, 0], 2, 3)
case("any_2d", LR + ":75-83", "any", [t_in(mz)], np.float64((mz != 0).any()))
az = rarray([0, 0, 0, 1, 0, 0, 0, 0], (2, 2, 2))
case("any_3d", LR + ":93-101", "any", [t_in(az)], np.float64((az != 0).any()))
mt = rmatrix([0, 1, 0, 0, 0, 0], 2, 3)
case("any_transposed", LR + ":128-141", "any", [t_in(mt)], np.float64((mt.T != 0).any()), transpose=True)
m6 = rmatrix([1, 0, 3, 4, 5, 6], 2, 3)
case("all_transposed_zero", LR + ":264-288", "all", [t_in(m6)], np.float64((m6.T != 0).all()), transpose=True)
a8 = rarray([1, 2, 0, 4, 5, 6, 7, 8], (2, 2, 2))
case("all_3d_zero", LR + ":214-232", "all", [t_in(a8)], np.float64((a8 != 0).all()))

# diff (tests/testthat/test-cumulative-operations.R): base R's diff(as.vector(x), lag, differences);
# a matrix result is recycled to the matrix's shape (array(expected_vec, dim = dim(x)))
CO = "tests/testthat/test-cumulative-operations.R"


def r_diff(v, lag=1, differences=1):
    v = np.asarray(v, dtype=np.float64).reshape(-1, order="F")
    for _ in range(differences):
        v = v[lag:] - v[:-lag]
    return v


d5 = [1, 4, 6, 8, 12]
case("diff_1d", CO + ":168-180", "diff", [t_in(d5)], r_diff(d5))
d6 = [1, 3, 6, 10, 15, 21]
for lag, lines in [(1, "186-189"), (2, "191-194"), (3, "196-199")]:
    case("diff_lag%d" % lag, CO + ":" + lines, "diff", [t_in(d6)], r_diff(d6, lag), lag=lag)
d7 = [1, 2, 4, 7, 11, 16, 22]
for k, lines in [(1, "206-209"), (2, "211-214"), (3, "216-219")]:
    case("diff_differences%d" % k, CO + ":" + lines, "diff", [t_in(d7)], r_diff(d7, 1, k), differences=k)
dd = [1.5, 3.2, 5.1, 7.8, 10.9]
case("diff_f32", CO + ":222-231", "diff", [t_in(dd, "float")], r_diff(dd))
case("diff_f64", CO + ":233-238", "diff", [t_in(dd, "double")], r_diff(dd))
mdiff = rmatrix([1, 2, 4, 7, 11, 16], 2, 3)
case("diff_matrix_recycled", CO + ":241-250", "diff", [t_in(mdiff)],
     np.resize(r_diff(mdiff), mdiff.size).reshape(mdiff.shape, order="F"))
case("diff_two", CO + ":253-256", "diff", [t_in([5, 8])], [3.0])
case_error("diff_single", CO + ":258-263 (the reference's diff.gpuTensor stops: R/gpuTensor.R:2307-2312)", "diff",
           [t_in([42])], "empty result")
case("diff_negative", CO + ":265-269", "diff", [t_in([10, 7, 5, 8, 3])], r_diff([10, 7, 5, 8, 3]))
for cid, lines, kw, pat in [("diff_lag0", "276", {"lag": 0}, "lag must be positive"),
                            ("diff_lag_neg", "277", {"lag": -1}, "lag must be positive"),
                            ("diff_differences0", "280", {"differences": 0}, "differences must be positive"),
                            ("diff_differences_neg", "281", {"differences": -1}, "differences must be positive")]:
    case_error(cid, CO + ":" + lines, "diff", [t_in([1, 2, 3, 4])], pat, **kw)

# range (tests/testthat/test-range-extrema-helpers.R): c(min(x), max(x))
RG = "tests/testthat/test-range-extrema-helpers.R"
for cid, lines, data, dtype in [("range_1d", "25-36", [3, 1, 4, 1, 5, 9, 2, 6], "float"),
                                ("range_f32", "38-46", [1.5, 2.7, 0.3, 4.9, 1.1], "float"),
                                ("range_f64", "48-52", [1.5, 2.7, 0.3, 4.9, 1.1], "double"),
                                ("range_single", "78-81", [42], "float"),
                                ("range_same", "83-87", [3.14] * 5, "float"),
                                ("range_negative", "89-93", [-5, -1, -10, -3, -7], "float"),
                                ("range_mixed", "95-99", [-2, 5, -8, 3, 0, -1, 7], "float")]:
    d = np.asarray(data, dtype=np.float64)
    if dtype == "float":
        d32 = d.astype(np.float32).astype(np.float64)  # the tensor holds float32 values
        case(cid, RG + ":" + lines, "range", [t_in(d, dtype)], [d32.min(), d32.max()])
    else:
        case(cid, RG + ":" + lines, "range", [t_in(d, dtype)], [d.min(), d.max()])
mr = rmatrix([3, 1, 4, 1, 5, 9, 2, 6, 5, 3, 5, 8], 3, 4)
case("range_2d", RG + ":55-64", "range", [t_in(mr)], [mr.min(), mr.max()])

# tensor_pow: sweep(base, 2, exp, "^") (test-comprehensive-broadcasting.R) and data_base ^ data_exp
# (test-consolidated-core.R)
pb = rmatrix([2, 3, 2, 3, 2, 3], 2, 3)
pe = np.asarray([1.0, 2.0, 3.0])
case("pow_broadcast_sweep", "tests/testthat/test-comprehensive-broadcasting.R:201-212", "tensor_pow",
     [t_in(pb), t_in(pe)], r_sweep(pb, [2], pe, lambda a, b: a ** b))
case("pow_elementwise", "tests/testthat/test-consolidated-core.R:356-366", "tensor_pow",
     [t_in([2, 3, 4, 2, 3]), t_in([1, 2, 1, 3, 1])], np.asarray([2, 3, 4, 2, 3.0]) ** np.asarray([1, 2, 1, 3, 1.0]))


def main():
    out = {"generator": "tests/golden/make_golden.py",
           "note": "inputs and base-R expressions transcribed from the reference testthat suite; expected values "
                   "computed with numpy on column-major logical arrays",
           "cases": cases}
    with open(os.path.join(HERE, "reference_cases.json"), "w") as f:
        json.dump(out, f, indent=1)
    print("wrote %d cases" % len(cases))


if __name__ == "__main__":
    main()
