"""The five workloads at their stated sizes, CUDA path vs the oracle on the
same input buffers (the inputs are generated on the device and copied back).

Tolerances (written per check below):
  * bit-exact: integer and bool outputs, comparisons, max/min values and
    every index (first-index tie rule);
  * elementwise: + - * / and sqrt are correctly rounded on both sides, so
    exact; exp, tanh and sigmoid within 2 ulp;
  * sums, means, variances and softmax: relative 1e-5 (float32 data) and
    1e-12 (float64 data).

Workloads:
  C1  float64 a ~ U(0,1), b ~ N(0,1), n = 2^20: c=a+b, d=a*b, e=exp(a),
      f=sigmoid(b), g=sqrt(a); sum/mean/var of each; which.max(c).
  C2  float32 X ~ N(0,1) 8192x8192, r ~ U(-1,1) 1x8192: relu(X+r), X>r as
      bool, pmax(X,r), tanh(X)*2, colSums(relu(X+r)), count(X>r) per column.
  C3  float32 T ~ N(0,1) 4096x4096x16: sum/mean/var/max/which.max of the whole
      tensor and sum/mean/var/max/argmax along each axis; int32 U[-1000,1000]
      of the same shape summed exactly; cumsum along axis 2 of float32
      64x1048576 ~ U(0,1).
  C4  row softmax of float32 65536x4096 ~ N(0, sd 2) plus a row offset
      ~ U(-50,50), and of float64 1024x32768 ~ N(0,1); rows sum to 1.
  C5  float32 256x512x32768 (2^32 elements) ~ N(0,1): the strided-views step
      (permute -> contiguous, x*0.5 + exp(-x^2), global sum/var, argmax along
      the permuted axis 1), all 131072 argmax fibers and the global sum/var
      against the oracle run slab by slab on the host.

The oracle's large-array forms split its per-output loops over the host's
threads (oracle_mt.c); each output is computed by the same code as the
single-threaded oracle.
"""
import numpy as np
import pytest
import torch

import oracle
from helpers import assert_exact, assert_rel, assert_ulp

pytestmark = pytest.mark.gpu
THREADS = oracle.default_threads()
F32, F64 = 1e-5, 1e-12


def _release():
    torch.cuda.synchronize()
    torch.cuda.empty_cache()


def _host(t):
    return t.as_array()


# ---------------------------------------------------------------------------
def test_c1_chain_and_statistics(acd):
    n = 1 << 20
    acd.set_seed(42)
    a = acd.rand_tensor((n,), dtype="double")
    b = acd.rnorm_tensor((n,), dtype="double")
    ah, bh = _host(a), _host(b)
    got = {"c": a + b, "d": a * b, "e": acd.exp(a), "f": acd.sigmoid(b), "g": acd.sqrt(a)}
    ref = {"c": oracle.binary("add", ah, bh), "d": oracle.binary("mul", ah, bh), "e": oracle.unary("exp", ah),
           "f": oracle.unary("sigmoid", bh), "g": oracle.unary("sqrt", ah)}
    for k in "cdg":  # correctly rounded on both sides
        assert_exact(_host(got[k]), ref[k], "C1 %s" % k)
    for k in "ef":  # exp / sigmoid: within 2 ulp
        assert_ulp(_host(got[k]), ref[k], 2, "C1 %s" % k)
    # the 15 statistics of the device's own c..g (identical buffers on both sides)
    for k, t in got.items():
        h = _host(t)
        assert_rel(acd.sum(t), oracle.reduce("sum", h), F64, "C1 sum(%s)" % k)
        assert_rel(acd.mean(t), oracle.reduce("mean", h), F64, "C1 mean(%s)" % k)
        assert_rel(acd.var(t), oracle.reduce("var", h), F64, "C1 var(%s)" % k)
    assert acd.which_max(got["c"]) == oracle.arg_reduce("argmax", _host(got["c"]))
    # the whole configuration as one kernel: the same five tensors bit for bit,
    # the 15 statistics against the oracle, which.max exact
    import acediar.tensor as Tm
    outs, stats, which = Tm.chain5_stats(a, b)
    st = stats.cpu().numpy()
    for k, o in zip("cdefg", outs):
        assert_exact(_host(o), _host(got[k]), "C1 fused %s vs the operator" % k)
        h = _host(o)
        assert_rel(st["cdefg".index(k) * 3], oracle.reduce("sum", h), F64, "C1 fused sum(%s)" % k)
        assert_rel(st["cdefg".index(k) * 3 + 1], oracle.reduce("mean", h), F64, "C1 fused mean(%s)" % k)
        assert_rel(st["cdefg".index(k) * 3 + 2], oracle.reduce("var", h), F64, "C1 fused var(%s)" % k)
    assert int(which.item()) == oracle.arg_reduce("argmax", _host(got["c"]))


# ---------------------------------------------------------------------------
def test_c2_broadcast_compare_and_column_reductions(acd):
    R = C = 8192
    acd.set_seed(42)
    X = acd.rnorm_tensor((R, C), dtype="float")
    r = acd.rand_tensor_uniform((1, C), dtype="float", min=-1.0, max=1.0)
    Xh, rh = _host(X), _host(r)
    # Y[i, j] = relu(X[i, j] + r[j]): the operator sequence and the fused kernel
    Y = acd.relu(X + r)
    Yf = acd.fused("add_relu", X, r)
    Yref = oracle.unary("relu", oracle.binary("add", Xh, rh, threads=THREADS), threads=THREADS)
    Yh = _host(Y)
    assert_exact(Yh, Yref, "C2 relu(X+r)")
    assert_exact(_host(Yf), Yref, "C2 fused relu(X+r)")
    M = X > r
    assert M.dtype == "bool"
    Mh = _host(M)
    assert_exact(Mh.astype(np.uint8), oracle.binary("gt", Xh, rh, threads=THREADS), "C2 X>r")
    assert_exact(_host(acd.pmax(X, r)), oracle.binary("max", Xh, rh, threads=THREADS), "C2 pmax(X,r)")
    T2ref = oracle.scalar("mul", oracle.unary("tanh", Xh, threads=THREADS), 2.0, threads=THREADS)
    T2 = _host(acd.tanh(X) * 2)
    assert_ulp(T2, T2ref, 2, "C2 tanh(X)*2")
    assert_exact(_host(acd.fused("tanh_scale", X, p0=2.0)), T2, "C2 fused tanh(X)*2 vs the operator sequence")
    del X, r, Yf, T2
    # per-column sum of Y (float32 data: relative 1e-5) and count of M (int32, exact)
    cs = _host(acd.tensor_sum(Y, axis=[1]))
    assert_rel(cs, oracle.reduce("sum", Yh, [0], threads=THREADS), F32, "C2 colSums(Y)", atol=1e-300)
    cnt = acd.tensor_count(M, axis=[1])
    assert cnt.dtype == "int32"
    assert_exact(_host(cnt), oracle.reduce("count", Mh, [0], threads=THREADS).astype(np.int32),
                 "C2 count(M) per column")
    del Y, M
    _release()


# ---------------------------------------------------------------------------
def test_c3_full_and_axis_reductions(acd):
    shp = (4096, 4096, 16)
    acd.set_seed(42)
    T = acd.rnorm_tensor(shp, dtype="float")
    Th = _host(T)
    full = oracle.full_stats(Th, THREADS)
    assert_rel(acd.sum(T), full["sum"], F32, "C3 sum(T)")
    assert_rel(acd.mean(T), full["mean"], F32, "C3 mean(T)")
    assert_rel(acd.var(T), full["var"], F32, "C3 var(T)")
    assert acd.max(T) == full["max"], "C3 max(T)"
    assert acd.which_max(T) == full["which_max"], "C3 which.max(T)"
    s, v = acd.sum_var(T)  # the fused single pass
    assert_rel(s, full["sum"], F32, "C3 fused sum")
    assert_rel(v, full["var"], F32, "C3 fused var")
    for ax in (1, 2, 3):
        for op in ("sum", "mean", "var"):
            got = _host(getattr(acd, "tensor_" + op)(T, axis=[ax])).astype(np.float64)
            ref = oracle.reduce(op, Th, [ax - 1], threads=THREADS)
            assert_rel(got, np.asarray(ref).reshape(got.shape, order="F"), F32, "C3 %s axis %d" % (op, ax),
                       atol=1e-300)
        got = _host(acd.tensor_max(T, axis=[ax]))
        ref = oracle.reduce("max", Th, [ax - 1], threads=THREADS)
        assert_exact(got.astype(np.float64), np.asarray(ref).reshape(got.shape, order="F"), "C3 max axis %d" % ax)
        got = _host(acd.argmax(T, axis=ax))
        ref = oracle.arg_reduce("argmax", Th, ax - 1, threads=THREADS)
        assert_exact(got, np.asarray(ref).reshape(got.shape, order="F"), "C3 argmax axis %d" % ax)
    del T, Th
    _release()
    # int32 U[-1000, 1000], same shape: exact int64 accumulation, int32 result
    rng = np.random.default_rng(42)
    Ih = rng.integers(-1000, 1001, size=shp[0] * shp[1] * shp[2], dtype=np.int32)
    I = acd.as_tensor(Ih, dtype="int32", shape=shp)
    got = acd.tensor_sum(I)
    assert got.dtype == "int32"
    assert int(_host(got).reshape(-1)[0]) == int(oracle.full_stats(Ih, THREADS)["sum"]) == int(Ih.sum(dtype=np.int64))
    del I, Ih
    _release()
    # cumsum along axis 2 of 64 x 1048576 (interleaved lanes)
    acd.set_seed(43)
    U = acd.rand_tensor((64, 1048576), dtype="float")
    Uh = _host(U)
    assert_rel(_host(acd.cumsum(U, axis=2)), oracle.scan("cumsum", Uh, 1, threads=THREADS), F32, "C3 cumsum axis 2")
    del U
    _release()


# ---------------------------------------------------------------------------
def test_c4_row_softmax(acd):
    R, C = 65536, 4096
    acd.set_seed(42)
    X = acd.rnorm_tensor((R, C), sd=2.0, dtype="float")
    off = acd.rand_tensor_uniform((R, 1), dtype="float", min=-50.0, max=50.0)
    Xo = X + off  # logits[i, j] = X[i, j] + off[i]
    del X
    Xh = _host(Xo)
    sm = acd.softmax(Xo, axis=2)
    ref = oracle.softmax(Xh, 1, threads=THREADS)
    assert_rel(_host(sm), ref, F32, "C4 softmax float32 65536x4096 along axis 2", atol=1e-300)
    rows = _host(acd.tensor_sum(sm, axis=[2])).astype(np.float64)
    assert_rel(rows, np.ones(R), F32, "C4 float32 row sums")
    del Xo, off, sm, ref, Xh
    _release()
    R2, C2 = 1024, 32768
    Xd = acd.rnorm_tensor((R2, C2), dtype="double")
    Xdh = _host(Xd)
    smd = acd.softmax(Xd, axis=2)
    assert_rel(_host(smd), oracle.softmax(Xdh, 1, threads=THREADS), F64, "C4 softmax float64 1024x32768 along axis 2",
               atol=1e-300)
    assert_rel(_host(acd.tensor_sum(smd, axis=[2])), np.ones(R2), F64, "C4 float64 row sums")
    del Xd, smd
    _release()


# ---------------------------------------------------------------------------
def test_c5_views_step_at_full_size(acd):
    """The bench step's call at 2^32 elements (the one-kernel step) against
    the oracle run slab by slab from the same x: global sum and var (relative
    1e-5) and every one of the 256x512 argmax fibers (exact); y and z
    bit-identical to contiguous() and the fused chain.  The separate R-level
    ops on z are checked too (sum, var, argmax along axis 1)."""
    import ctypes

    import acediar._lib as L
    import acediar.sharded as SH
    from acediar.tensor import _alloc, _stream, context

    n0, n1, n2 = 256, 512, 32768
    n = n0 * n1 * n2
    x = _alloc((n0, n1, n2), "float")
    # as the bench: normal(0, 1) from Philox seed 42, counter = global index
    L.check(L.lib().acd_rand(context(), ctypes.byref(x.desc()), 1, ctypes.c_double(0.0), ctypes.c_double(1.0),
                             ctypes.c_uint64(42), ctypes.c_uint64(0), _stream()), "rand")
    # the bench's step: one kernel (acd_permute_fused_stats_keys)
    xv = acd.permute_view(x, [3, 1, 2])
    y, z, stats, keys = SH.permute_chain_stats_keys(xv, 0.5, 0)
    y_ref = acd.contiguous(xv)
    assert torch.equal(y.storage[:n], y_ref.storage[:n]), "C5 y = contiguous(permute(x)), bit for bit"
    del y_ref
    z_ref = acd.fused("scale_add_exp_neg_square", y, p0=0.5)
    assert torch.equal(z.storage[:n], z_ref.storage[:n]), "C5 z = y*0.5 + exp(-y^2), bit for bit"
    del y, z_ref
    tot, var = (float(t.item()) for t in SH.merge_stats_torch(stats.view(1, -1)))
    idx = SH.decode_keys(keys, (n0, n1), one_based=True, dtype="int32").as_array()
    s_op, v_op = acd.sum(z), acd.var(z)
    am_op = acd.argmax(z, axis=1).as_array()
    del z, keys, stats
    _release()

    # oracle: z = x*0.5 + exp(-x^2) per slab of x along its axis 3; the
    # permuted fiber (a, b) of z is x[a, b, :], so a slab holds a piece of
    # every fiber: keep the running first maximum per fiber
    slab = 1024
    st = oracle.ChunkedStats(n, THREADS)
    best = np.full(n0 * n1, -np.inf, dtype=np.float32)
    arg = np.zeros(n0 * n1, dtype=np.int64)
    per = n0 * n1 * slab

    def zslab(c0):
        xs = x.storage[c0 * n0 * n1:c0 * n0 * n1 + per].cpu().numpy()
        return oracle.gauss_chain(xs, 0.5, threads=THREADS)

    for c0 in range(0, n2, slab):
        zs = zslab(c0)
        st.first(zs)
        z2 = zs.reshape(slab, n0 * n1)
        m = z2.max(axis=0)
        a = z2.argmax(axis=0)  # first index of the maximum within the slab
        upd = m > best  # strict: an earlier slab keeps a tie
        best[upd] = m[upd]
        arg[upd] = c0 + a[upd]
    for c0 in range(0, n2, slab):
        st.second(zslab(c0))
    ref = st.result()
    ref_idx = (arg + 1).reshape((n0, n1), order="F")
    assert_rel(tot, ref["sum"], F32, "C5 sum (step kernel)")
    assert_rel(var, ref["var"], F32, "C5 var (step kernel)")
    assert_exact(idx.astype(np.int64), ref_idx, "C5 argmax along axis 1, all 131072 fibers (step kernel keys)")
    assert_rel(s_op, ref["sum"], F32, "C5 sum(z)")
    assert_rel(v_op, ref["var"], F32, "C5 var(z)")
    assert_exact(am_op.astype(np.int64), ref_idx, "C5 argmax(z, axis=1)")
    print("C5 oracle: sum %.10g var %.10g argmax checksum %d; device: sum %.10g var %.10g" % (
        ref["sum"], ref["var"], int(ref_idx.sum()), tot, var))
    del x
    _release()
