"""The one-pass forms of the strided-views step against the separate calls
they replace.  acd_fused_stats_keys (the elementwise chain with its
statistics row and argmax keys) and acd_permute_fused_stats_keys (the
permute -> contiguous copy followed by that): y and z
bit-identical, keys identical to acd_argmax_keys, the statistics row's n and
shift identical and its moments within 1e-12 relative, and the merged
sum/var within the float32 contract of the oracle."""
import numpy as np
import pytest
import torch

import oracle
from helpers import assert_exact

pytestmark = pytest.mark.gpu


def _merged(stats):
    import acediar.sharded as SH
    tot, var = SH.merge_stats_torch(stats.view(1, -1))
    return float(tot.item()), float(var.item())


def _check_stats(st, st_ref, z_ref):
    assert st[0] == st_ref[0] and st[1] == st_ref[1], (st, st_ref)
    scale = np.abs(z_ref.astype(np.float64) - st_ref[1])
    assert abs(st[2] - st_ref[2]) <= 1e-12 * max(1.0, scale.sum())
    assert abs(st[3] - st_ref[3]) <= 1e-12 * max(1.0, (scale ** 2).sum())


@pytest.mark.parametrize("shape,base", [((4096, 16, 8), 0), ((32768, 3, 5), 7), ((8, 1000), 0), ((4, 1), 12345),
                                        ((1024, 700), 2 ** 31), ((6, 10), 0), ((4100, 33), 5)])
def test_fused_stats_keys_matches_separate_calls(acd, shape, base):
    import acediar.sharded as SH
    rng = np.random.default_rng(sum(shape) + base)
    x = (np.round(rng.normal(0, 1, shape) * 4) / 4).astype(np.float32)  # quarters: ties inside fibers
    y = acd.as_tensor(x, dtype="float")
    z, stats, keys = SH.chain_stats_keys(y, 0.5, base)
    z_ref = acd.fused("scale_add_exp_neg_square", y, p0=0.5)
    assert_exact(z.as_array(), z_ref.as_array(), "z")
    keys_ref, _ = SH.argmax_keys(z_ref, 0, base)
    assert torch.equal(keys.cpu(), keys_ref.cpu()), "argmax keys"
    zz = z_ref.as_array()
    _check_stats(stats.cpu().numpy(), SH.stats_partial(z_ref).cpu().numpy(), zz)
    tot, var = _merged(stats)
    e_tot = float(oracle.reduce("sum", oracle.View.of(zz)))
    e_var = float(oracle.reduce("var", oracle.View.of(zz)))
    assert abs(tot - e_tot) <= 1e-5 * max(1.0, np.abs(zz.astype(np.float64)).sum())
    if zz.size > 1:
        assert abs(var - e_var) <= 1e-5 * abs(e_var)
    idx = SH.decode_keys(keys, shape[1:] if len(shape) > 1 else (1,), one_based=True, dtype="int64").as_array()
    exp_idx = np.argmax(zz, axis=0) + 1 + base
    assert_exact(idx, exp_idx.astype(np.int64).reshape(idx.shape), "decoded argmax")


def test_fused_stats_keys_view_falls_back(acd):
    """A permuted (non-contiguous) input runs the three separate passes."""
    import acediar.sharded as SH
    x = np.random.default_rng(3).normal(size=(64, 48)).astype(np.float32)
    v = acd.transpose_view(acd.as_tensor(x, dtype="float"))
    z, stats, keys = SH.chain_stats_keys(v, 0.5, 0)
    zc = acd.fused("scale_add_exp_neg_square", acd.contiguous(v), p0=0.5)
    assert_exact(z.as_array(), zc.as_array(), "z of a view")
    keys_ref, _ = SH.argmax_keys(zc, 0, 0)
    assert torch.equal(keys.cpu(), keys_ref.cpu())


@pytest.mark.parametrize("xshape,base", [((64, 32, 256), 0), ((128, 64, 4096), 9), ((100, 3, 72), 0),
                                         ((256, 5, 1000), 3 * 2 ** 30), ((64, 64, 130), 0), ((8, 8, 16), 0),
                                         ((96, 1, 64), 1)])
def test_permute_fused_stats_keys_matches_separate_calls(acd, xshape, base):
    """Transposes the TMA copy takes (tile-aligned and ragged) and ones it
    does not (an extent not a multiple of 4, or below one 64 x 64 tile), with
    and without the chain kernel's one-pass form; two calls in a row, since
    the statistics counter must start clean each call."""
    import acediar.sharded as SH
    rng = np.random.default_rng(sum(xshape) + base)
    x = (np.round(rng.normal(0, 1, xshape) * 8) / 8).astype(np.float32)  # eighths: ties inside fibers
    xv = acd.permute_view(acd.as_tensor(x, dtype="float"), [3, 1, 2])
    for rep in range(2):
        y, z, stats, keys = SH.permute_chain_stats_keys(xv, 0.5, base)
        y_ref = acd.contiguous(xv)
        assert_exact(y.as_array(), y_ref.as_array(), "y")
        z_ref = acd.fused("scale_add_exp_neg_square", y_ref, p0=0.5)
        assert_exact(z.as_array(), z_ref.as_array(), "z")
        keys_ref, _ = SH.argmax_keys(z_ref, 0, base)
        assert torch.equal(keys.cpu(), keys_ref.cpu()), ("keys", rep)
        _check_stats(stats.cpu().numpy(), SH.stats_partial(z_ref).cpu().numpy(), z_ref.as_array())
    acd.check_device_status()


@pytest.mark.parametrize("xshape,perm,base", [((64, 300, 192), [3, 1, 2], 0), ((256, 160, 256), [3, 1, 2], 5),
                                              ((64, 5, 128), [3, 2, 1], 0), ((68, 7, 200), [3, 2, 1], 11),
                                              ((64, 2, 64), [3, 1, 2], 0), ((640, 1, 68), [3, 1, 2], 2 ** 31)])
def test_permute_one_kernel_shapes(acd, xshape, perm, base):
    """The one-kernel form (the view is a TMA-eligible transpose): sequences
    of 1 to 4 tiles, more sequences than CTAs, a batch axis between the two
    transposed ones (fiber keys at a stride), and edges ragged along either
    transposed axis."""
    import acediar.sharded as SH
    rng = np.random.default_rng(sum(xshape) + base)
    x = (np.round(rng.normal(0, 1, xshape) * 8) / 8).astype(np.float32)
    xv = acd.permute_view(acd.as_tensor(x, dtype="float"), perm)
    y, z, stats, keys = SH.permute_chain_stats_keys(xv, 0.5, base)
    y_ref = acd.contiguous(xv)
    assert_exact(y.as_array(), y_ref.as_array(), "y")
    z_ref = acd.fused("scale_add_exp_neg_square", y_ref, p0=0.5)
    assert_exact(z.as_array(), z_ref.as_array(), "z")
    keys_ref, _ = SH.argmax_keys(z_ref, 0, base)
    assert torch.equal(keys.cpu(), keys_ref.cpu()), "keys"
    zz = z_ref.as_array()
    _check_stats(stats.cpu().numpy(), SH.stats_partial(z_ref).cpu().numpy(), zz)
    xt = np.ascontiguousarray(np.transpose(x, [p - 1 for p in perm]))
    zo = oracle.gauss_chain(xt, 0.5)
    bound = 2 * np.spacing(np.maximum(np.abs(xt * np.float32(0.5)), np.exp(-(xt * xt)).astype(np.float32))) + \
        np.spacing(np.abs(zo))
    assert np.all(np.abs(zz.astype(np.float64) - zo) <= bound), "z vs the oracle"
    # the argmax rule of the oracle (first of equal values) on this z
    idx = SH.decode_keys(keys, zz.shape[1:], one_based=True, dtype="int64").as_array()
    assert_exact(idx, oracle.arg_reduce("argmax", zz, axis=0, one_based=True) + base, "decoded argmax vs the oracle")
    acd.check_device_status()


def test_permute_one_kernel_infinities_nan_and_signed_zeros(acd):
    """The one-kernel form with fibers all -inf, all NaN, NaN among values,
    +inf, and -0/+0 ties (both map to z = 1; the smaller index wins), keys
    identical to acd_argmax_keys on the separately computed z."""
    import acediar.sharded as SH
    x = np.random.default_rng(8).normal(size=(64, 4, 256)).astype(np.float32)
    x[3, 0, :] = -np.inf
    x[4, 0, :] = np.nan
    x[5, 1, 17] = np.nan
    x[6, 1, 100] = np.inf
    x[7, 2, :] = 5.0
    x[7, 2, 90] = -0.0
    x[7, 2, 30] = 0.0
    x[8, 3, :] = 5.0
    x[8, 3, 200] = 0.0
    x[8, 3, 10] = -0.0
    xv = acd.permute_view(acd.as_tensor(x, dtype="float"), [3, 1, 2])
    y, z, stats, keys = SH.permute_chain_stats_keys(xv, 0.5, 3)
    z_ref = acd.fused("scale_add_exp_neg_square", acd.contiguous(xv), p0=0.5)
    np.testing.assert_array_equal(z.as_array(), z_ref.as_array())
    keys_ref, _ = SH.argmax_keys(z_ref, 0, 3)
    assert torch.equal(keys.cpu(), keys_ref.cpu()), (keys.cpu(), keys_ref.cpu())
    assert np.isnan(stats.cpu().numpy()[2]) and np.isnan(SH.stats_partial(z_ref).cpu().numpy()[2])
    acd.check_device_status()


def test_fused_stats_keys_infinities_and_nan(acd):
    """Fibers that are all -inf (the first element wins, as in the argmax
    reduction), a fiber with NaN (NaN never wins; the moments turn NaN, as in
    acd_stats_partial), and +inf."""
    import acediar.sharded as SH
    x = np.random.default_rng(4).normal(size=(64, 6)).astype(np.float32)
    x[:, 0] = -np.inf
    x[5, 1] = np.nan
    x[7, 2] = np.inf
    x[:, 3] = -np.inf
    x[9, 3] = 2.0
    y = acd.as_tensor(x, dtype="float")
    z, stats, keys = SH.chain_stats_keys(y, 0.5, 3)
    z_ref = acd.fused("scale_add_exp_neg_square", y, p0=0.5)
    np.testing.assert_array_equal(z.as_array(), z_ref.as_array())  # NaN in the same place counts as equal
    keys_ref, _ = SH.argmax_keys(z_ref, 0, 3)
    assert torch.equal(keys.cpu(), keys_ref.cpu()), (keys.cpu(), keys_ref.cpu())
    assert np.isnan(stats.cpu().numpy()[2]) and np.isnan(SH.stats_partial(z_ref).cpu().numpy()[2])


@pytest.mark.parametrize("world", [1, 3])
def test_shard_exchange_on_one_gpu(acd, world):
    """The one-collective exchange with `world` shards emulated on one GPU:
    each shard's one-pass chain kernel writes its keys and its statistics row
    into its own exchange buffer, torch.maximum over the buffers stands in for
    the MAX all-reduce, and acd_shard_finish gives the argmax along the
    permuted axis (exact, ties across shards included) and the global sum and
    var (float32 contract) of the whole tensor; the rows are reset after."""
    import ctypes

    import acediar._lib as L
    import acediar.sharded as SH
    from acediar.tensor import _alloc, _stream, context

    rng = np.random.default_rng(40 + world)
    n0, n1, n2 = 64, 48, 96
    x = (np.round(rng.normal(0, 1, (n0, n1, n2)) * 4) / 4).astype(np.float32)  # ties, across shards too
    nkeys = n0 * n1
    bufs = []
    for r in range(world):
        lo, hi = SH.shard_bounds(n2, r, world)
        xs = acd.as_tensor(np.ascontiguousarray(x[:, :, lo:hi]), dtype="float")
        y = acd.contiguous(acd.permute_view(xs, [3, 1, 2]))
        buf = SH.exchange_buffer(nkeys, world, y.storage.device)
        z = _alloc(y.shape, "float")
        L.check(L.lib().acd_fused_stats_keys(context(), ctypes.byref(z.desc()), ctypes.byref(y.desc()),
                                             ctypes.c_double(0.5), SH.row_slot(buf, nkeys, r),
                                             ctypes.c_void_p(buf.data_ptr()), lo, _stream()), "fused_stats_keys")
        bufs.append(buf)
    red = bufs[0].clone()
    for b in bufs[1:]:
        red = torch.maximum(red, b)
    idx, sv = SH.shard_finish(red, nkeys, world, (n0, n1))
    z_all = oracle.gauss_chain(np.transpose(x, (2, 0, 1)), 0.5)
    es, ev = oracle.sum_var(z_all)
    tot, var = (float(v) for v in sv.cpu().numpy())
    assert abs(tot - es) <= 1e-5 * max(1.0, np.abs(z_all.astype(np.float64)).sum())
    assert abs(var - ev) <= 1e-5 * abs(ev)
    assert_exact(idx.as_array().astype(np.int64), oracle.arg_reduce("argmax", z_all, 0), "argmax keys across shards")
    assert torch.all(red[nkeys:] == np.iinfo(np.int64).min), "rows reset for the next exchange"
