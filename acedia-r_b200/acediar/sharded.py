"""Sharded execution of the strided-views workload over one process per GPU.

The tensor x (n0 x n1 x n2, column-major) is split along its outermost axis
into contiguous slabs, one per rank; every rank generates or receives only its
slab.  permute_view(x, c(3,1,2)) puts the shard axis first, so contiguous(),
the elementwise chain and the per-element work stay local.  Two steps need the
other ranks:
  * global sum/var: each rank reduces its slab to (n, K, sum(x-K), sum((x-K)^2))
    (K = first element of the slab); the rows are all-gathered and merged in
    rank order, so the result does not depend on the collective's order;
  * argmax along the permuted leading axis (the shard axis): each rank writes
    one order-preserving 64-bit key per output, (ordered value bits << 32) |
    (2^32-1 - global index) with the sign bit flipped, and a MAX all-reduce
    picks the largest value and, among equal values, the smallest index — the
    reference's first-index rule (src/kernels/tensor_kernels.cu:794).
The statistics row and the keys can come from the pass that writes the
elementwise chain (chain_stats_keys), so z is written once and not re-read;
permute_chain_stats_keys does the whole step, the contiguous copy included,
in one kernel that reads x once.

Both exchanges travel in one int64 MAX all-reduce over an exchange buffer
(exchange_buffer, shard_finish): the keys, then one row of six float64 bit
patterns per rank, where every rank leaves the other ranks' rows at
INT64_MIN (the bit pattern of -0.0 and the smallest int64), so MAX copies
each rank's row to all ranks unchanged.
There is no peer-memory access and no multicast: the exchanged bytes are a few
doubles and one key per output (1 MiB at 256 x 512).
"""
import ctypes
from fractions import Fraction

import numpy as np
import torch

from . import _lib as L
from .tensor import _alloc, _stream, context, gpuTensor

STATS_WIDTH = 6  # n, K, s1_hi, s2_hi, s1_lo, s2_lo


# ---------------------------------------------------------------------------
# host references of the exchange formats (also used by the CPU tests)
# ---------------------------------------------------------------------------
def merge_stats_exact(rows):
    """Exact merge of per-shard rows -> (sum, var) as Python floats."""
    n_tot = Fraction(0)
    s1 = Fraction(0)
    s2 = Fraction(0)
    k0 = Fraction(rows[0][1])
    for r in rows:
        n, k = Fraction(r[0]), Fraction(r[1])
        a = Fraction(r[2]) + Fraction(r[4])
        b = Fraction(r[3]) + Fraction(r[5])
        d = k - k0
        s1 += a + n * d
        s2 += b + 2 * d * a + n * d * d
        n_tot += n
    total = n_tot * k0 + s1
    var = (s2 - s1 * s1 / n_tot) / (n_tot - 1) if n_tot > 1 else Fraction(0)
    return float(total), float(var)


def merge_stats_torch(rows):
    """The same merge on the device in float64, rank order (rows: [G, 6])."""
    n = rows[:, 0]
    k = rows[:, 1]
    a = rows[:, 2] + rows[:, 4]
    b = rows[:, 3] + rows[:, 5]
    d = k - k[0]
    s1 = (a + n * d).sum()
    s2 = (b + 2 * d * a + n * d * d).sum()
    nt = n.sum()
    total = nt * k[0] + s1
    var = (s2 - s1 * (s1 / nt)) / (nt - 1)
    return total, var


def pack_keys_np(values, index):
    """Host reference of the key format written by acd_argmax_keys."""
    # -0 and +0 share one key (the reduction treats them as equal)
    v = (np.ascontiguousarray(values, dtype=np.float32) + np.float32(0.0)).view(np.uint32).astype(np.uint64)
    ordered = np.where(v & 0x80000000, (~v) & 0xFFFFFFFF, v | 0x80000000)
    u = (ordered << np.uint64(32)) | (np.uint64(0xFFFFFFFF) - np.asarray(index, dtype=np.uint64))
    return (u ^ np.uint64(0x8000000000000000)).view(np.int64)


INT64_MIN = np.iinfo(np.int64).min


def pack_exchange_np(keys, row, rank, world):
    """Host reference of one rank's exchange buffer: its keys, its statistics
    row as float64 bit patterns in slot `rank`, INT64_MIN in the others."""
    buf = np.full(len(keys) + STATS_WIDTH * world, INT64_MIN, dtype=np.int64)
    buf[:len(keys)] = keys
    buf[len(keys) + STATS_WIDTH * rank:len(keys) + STATS_WIDTH * (rank + 1)] = \
        np.asarray(row, dtype=np.float64).view(np.int64)
    return buf


def finish_exchange_np(buf, nkeys, world, one_based=True):
    """Host reference of acd_shard_finish on an all-reduced buffer: the rows
    (merged in rank order as merge_stats_torch does) and the decoded keys."""
    rows = np.asarray(buf[nkeys:nkeys + STATS_WIDTH * world], dtype=np.int64).view(np.float64).reshape(world, -1)
    tot, var = merge_stats_torch(torch.from_numpy(rows.copy()))
    return float(tot), float(var), decode_keys_np(buf[:nkeys], one_based)


def decode_keys_np(keys, one_based=True):
    u = np.asarray(keys, dtype=np.int64).view(np.uint64) ^ np.uint64(0x8000000000000000)
    idx = (np.uint64(0xFFFFFFFF) - (u & np.uint64(0xFFFFFFFF))).astype(np.int64)
    return idx + (1 if one_based else 0)


# ---------------------------------------------------------------------------
# device path
# ---------------------------------------------------------------------------
def stats_partial(x):
    """This shard's float64[6] statistics row (device tensor)."""
    out = torch.empty(STATS_WIDTH, dtype=torch.float64, device=x.device)
    L.check(L.lib().acd_stats_partial(context(), ctypes.c_void_p(out.data_ptr()), ctypes.byref(x.desc()),
                                      _stream()), "stats_partial")
    return out


def argmax_keys(x, axis0, index_base):
    """Keys of the argmax along 0-based `axis0` with global index offset."""
    kept = [x.shape[d] for d in range(x.ndims) if d != axis0]
    n = int(np.prod(kept)) if kept else 1
    keys = torch.empty(n, dtype=torch.int64, device=x.device)
    L.check(L.lib().acd_argmax_keys(context(), ctypes.c_void_p(keys.data_ptr()), ctypes.byref(x.desc()), axis0,
                                    int(index_base), _stream()), "argmax_keys")
    return keys, kept


def chain_stats_keys(y, p0, index_base):
    """z = y*p0 + exp(-(y^2)) together with this shard's statistics row of z
    and the argmax keys of z along axis 1 (R's 1-based axis; the global index
    offset is `index_base`), from one pass over z: the same three results as
    fused(), stats_partial() and argmax_keys(), without reading z again."""
    z = _alloc(y.shape, y.dtype, y.device)
    stats = torch.empty(STATS_WIDTH, dtype=torch.float64, device=y.device)
    n = int(np.prod(y.shape[1:])) if y.ndims > 1 else 1
    keys = torch.empty(n, dtype=torch.int64, device=y.device)
    L.check(L.lib().acd_fused_stats_keys(context(), ctypes.byref(z.desc()), ctypes.byref(y.desc()), float(p0),
                                         ctypes.c_void_p(stats.data_ptr()), ctypes.c_void_p(keys.data_ptr()),
                                         int(index_base), _stream()), "fused_stats_keys")
    return z, stats, keys


def permute_chain_stats_keys(x, p0, index_base):
    """y = contiguous(x) of the permuted view x, then z = y*p0 + exp(-(y^2)),
    the statistics row of z and its argmax keys along axis 1: the
    strided-views step in one call.  When x is a transpose TMA can read (the
    usual case) this is one kernel that reads x once; otherwise the copy and
    then the one-pass chain."""
    y = _alloc(x.shape, x.dtype, x.device)
    z = _alloc(x.shape, x.dtype, x.device)
    stats = torch.empty(STATS_WIDTH, dtype=torch.float64, device=x.device)
    n = int(np.prod(x.shape[1:])) if x.ndims > 1 else 1
    keys = torch.empty(n, dtype=torch.int64, device=x.device)
    L.check(L.lib().acd_permute_fused_stats_keys(context(), ctypes.byref(y.desc()), ctypes.byref(z.desc()),
                                                 ctypes.byref(x.desc()), float(p0), ctypes.c_void_p(stats.data_ptr()),
                                                 ctypes.c_void_p(keys.data_ptr()), int(index_base), _stream()),
            "permute_fused_stats_keys")
    return y, z, stats, keys


def decode_keys(keys, shape, one_based=True, dtype="int32"):
    out = _alloc(tuple(shape), dtype, keys.device)
    L.check(L.lib().acd_argmax_keys_decode(context(), ctypes.byref(out.desc()), ctypes.c_void_p(keys.data_ptr()),
                                           1 if one_based else 0, _stream()), "argmax_keys_decode")
    return out


def exchange_buffer(nkeys, world, device):
    """The int64 exchange buffer (keys, then one statistics row per rank),
    with every row at INT64_MIN."""
    buf = torch.empty(nkeys + STATS_WIDTH * world, dtype=torch.int64, device=device)
    L.check(L.lib().acd_shard_exchange_init(context(), ctypes.c_void_p(buf.data_ptr()), int(nkeys), int(world),
                                            _stream()), "shard_exchange_init")
    return buf


def row_slot(buf, nkeys, rank):
    """Device address of `rank`'s statistics row inside the exchange buffer."""
    return ctypes.c_void_p(buf.data_ptr() + 8 * (nkeys + STATS_WIDTH * rank))


def shard_finish(buf, nkeys, world, shape, one_based=True, dtype="int32", out=None, sum_var=None):
    """After the MAX all-reduce of `buf`: argmax indices of shape `shape`,
    and a float64[2] device tensor (sum, var); the rows are reset for the
    next exchange."""
    if out is None:
        out = _alloc(tuple(shape), dtype, buf.device)
    if sum_var is None:
        sum_var = torch.empty(2, dtype=torch.float64, device=buf.device)
    L.check(L.lib().acd_shard_finish(context(), ctypes.c_void_p(buf.data_ptr()), int(nkeys), int(world),
                                     ctypes.byref(out.desc()), ctypes.c_void_p(sum_var.data_ptr()),
                                     1 if one_based else 0, _stream()), "shard_finish")
    return out, sum_var


def shard_bounds(n, rank, world):
    """[lo, hi) of the outermost-axis slab owned by `rank`."""
    return n * rank // world, n * (rank + 1) // world
