"""Host logic of the sharded path, on CPU: the per-shard statistics rows and
the argmax keys exchanged between ranks, run as two gloo ranks.

The device kernels produce the same rows and keys (acd_stats_partial,
acd_argmax_keys); here numpy stands in for them so that the exchange and the
merge are checked without a GPU.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from acediar import sharded as SH


def _stats_row(z):
    """What acd_stats_partial writes for a float32 shard: n, K, s1, s2 (and zero lo parts)."""
    zz = z.astype(np.float64).reshape(-1, order="F")
    k = zz[0]
    d = zz - k
    return [float(zz.size), k, float(d.sum()), float((d * d).sum()), 0.0, 0.0]


def test_key_order_matches_value_then_first_index():
    rng = np.random.default_rng(0)
    v = rng.normal(size=2000).astype(np.float32)
    v[::7] = v[3]  # ties
    v[5] = -0.0
    v[6] = 0.0
    idx = rng.integers(0, 2 ** 32 - 1, size=2000)
    keys = SH.pack_keys_np(v, idx)
    order = np.argsort(keys, kind="stable")
    for a, b in zip(order[:-1], order[1:]):
        assert (v[a] < v[b]) or (v[a] == v[b] and idx[a] >= idx[b])
    np.testing.assert_array_equal(SH.decode_keys_np(keys, one_based=False), idx)


def test_exact_merge_equals_oracle_on_one_array():
    rng = np.random.default_rng(1)
    z = rng.normal(size=(64, 33, 10)).astype(np.float32)
    rows = [_stats_row(z[:, :, :4]), _stats_row(z[:, :, 4:7]), _stats_row(z[:, :, 7:])]
    s, v = SH.merge_stats_exact(rows)
    es, ev = oracle.sum_var(z)
    assert abs(s - es) <= 1e-12 * abs(es) + 1e-9
    assert abs(v - ev) <= 1e-12 * abs(ev)
    ts, tv = SH.merge_stats_torch(torch.tensor(rows, dtype=torch.float64))
    assert abs(float(ts) - es) <= 1e-9 * abs(es) + 1e-9 and abs(float(tv) - ev) <= 1e-9 * abs(ev)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, x, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        n2 = x.shape[2]
        lo, hi = SH.shard_bounds(n2, rank, world)
        shard = x[:, :, lo:hi]
        # z for this shard: permute (3,1,2), fused chain (oracle restatement)
        y = np.transpose(shard, (2, 0, 1))
        z = oracle.gauss_chain(y, 0.5)
        row = torch.tensor(_stats_row(z), dtype=torch.float64)
        rows = [torch.zeros(SH.STATS_WIDTH, dtype=torch.float64) for _ in range(world)]
        dist.all_gather(rows, row)
        # local argmax along the shard axis as keys with the global index base
        zl = z.reshape(z.shape[0], -1, order="F")
        li = np.argmax(zl, axis=0)  # first index on ties
        keys = torch.from_numpy(SH.pack_keys_np(zl[li, np.arange(zl.shape[1])], li + lo).copy())
        dist.all_reduce(keys, op=dist.ReduceOp.MAX)
        if rank == 0:
            q.put((SH.merge_stats_exact([r.tolist() for r in rows]), SH.decode_keys_np(keys.numpy())))
    finally:
        dist.destroy_process_group()


def _rank_main_packed(rank, world, port, x, q):
    """The one-collective exchange: keys and rows in one int64 buffer, one
    MAX all-reduce, then the host reference of acd_shard_finish."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        n2 = x.shape[2]
        lo, hi = SH.shard_bounds(n2, rank, world)
        z = oracle.gauss_chain(np.transpose(x[:, :, lo:hi], (2, 0, 1)), 0.5)
        zl = z.reshape(z.shape[0], -1, order="F")
        li = np.argmax(zl, axis=0)
        keys = SH.pack_keys_np(zl[li, np.arange(zl.shape[1])], li + lo)
        buf = torch.from_numpy(SH.pack_exchange_np(keys, _stats_row(z), rank, world))
        dist.all_reduce(buf, op=dist.ReduceOp.MAX)
        s, v, idx = SH.finish_exchange_np(buf.numpy(), keys.size, world)
        q.put((rank, s, v, idx))
    finally:
        dist.destroy_process_group()


def _run_ranks(target, world, x):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, x, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in range(world)] if target is _rank_main_packed else [q.get(timeout=120)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return out


@pytest.mark.parametrize("world", [2, 3])
def test_one_max_all_reduce_carries_keys_and_rows(world):
    rng = np.random.default_rng(3)
    x = rng.standard_normal((16, 8, 24)).astype(np.float32)
    x[:, :, 5] = x[:, :, 17]  # cross-shard ties
    x[0, 0, :] = -0.0  # a statistics shift of -0.0 must survive the MAX
    z = oracle.gauss_chain(np.transpose(x, (2, 0, 1)), 0.5)
    es, ev = oracle.sum_var(z)
    exp = oracle.arg_reduce("argmax", z, 0).reshape(-1, order="F")
    for rank, s, v, idx in _run_ranks(_rank_main_packed, world, x):
        assert abs(s - es) <= 1e-9 * abs(es) + 1e-9, rank
        assert abs(v - ev) <= 1e-9 * abs(ev), rank
        np.testing.assert_array_equal(idx, exp)


def test_exchange_rows_survive_max_with_negative_and_zero_values():
    rows = [[3.0, -0.0, -5.5, 2.0, -1e-300, 0.0], [2.0, -7.25, 0.5, 1.0, 0.0, -0.0]]
    bufs = [SH.pack_exchange_np(np.zeros(3, dtype=np.int64), r, k, 2) for k, r in enumerate(rows)]
    red = np.maximum(bufs[0], bufs[1])
    got = red[3:].view(np.float64).reshape(2, -1)
    np.testing.assert_array_equal(got.view(np.int64), np.asarray(rows, dtype=np.float64).view(np.int64))


@pytest.mark.parametrize("world", [2])
def test_two_gloo_ranks_reproduce_the_single_rank_result(world):
    rng = np.random.default_rng(2)
    x = rng.standard_normal((16, 8, 24)).astype(np.float32)
    x[:, :, 5] = x[:, :, 17]  # cross-shard ties: the smaller global index must win
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, x, q)) for r in range(world)]
    for p in procs:
        p.start()
    (s, v), idx = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    z = oracle.gauss_chain(np.transpose(x, (2, 0, 1)), 0.5)
    es, ev = oracle.sum_var(z)
    assert abs(s - es) <= 1e-9 * abs(es) + 1e-9
    assert abs(v - ev) <= 1e-9 * abs(ev)
    exp = oracle.arg_reduce("argmax", z, 0).reshape(-1, order="F")
    np.testing.assert_array_equal(idx, exp)
