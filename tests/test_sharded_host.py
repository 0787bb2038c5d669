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
