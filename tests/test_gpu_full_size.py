"""Full-size cases (more than 2^31 elements, the strided-views step's
256x512x32768 float32 = 2^32 elements, 16 GiB), checked through properties
that do not need the oracle to process the whole tensor:

- permute -> contiguous is a bijection: sampled output positions (including
  the ones around 2^31 and the last) equal the input at the permuted index;
- the fused chain x*0.5 + exp(-x^2) at sampled positions matches the oracle
  on those elements (2 ulp of the larger addend plus one rounding);
- argmax along the permuted axis 1 matches numpy on sampled whole fibers;
- which.max / which.min find planted extremes past 2^32 - 2^20, first index
  on ties;
- sum / mean / var of 2^32 ones are exact; an int32 sum that leaves the
  int32 range is R's NA;
- a flattened cumsum of 2^31 + 4103 ones gives float32(k + 1) at position k;
- a whole-tensor softmax of 2^31 + 4103 elements sums to 1 and keeps the
  ratios exp(x_i - x_j) of sampled pairs.
"""
import numpy as np
import pytest
import torch

import oracle
from helpers import assert_exact

pytestmark = pytest.mark.gpu

SHAPE = (256, 512, 32768)
N = 256 * 512 * 32768  # 2^32


def _gather(t, pos):
    """Elements at flat storage positions (int64) of a contiguous tensor."""
    idx = torch.as_tensor(np.asarray(pos, dtype=np.int64), device=t.storage.device)
    v = t.storage[t.offset + idx].cpu().numpy()
    return v.astype(np.bool_) if t.dtype == "bool" else v


def _sample_positions(n, k, seed):
    rng = np.random.default_rng(seed)
    edges = [0, 1, 2 ** 31 - 1, 2 ** 31, 2 ** 31 + 1, n - 2, n - 1]
    return np.concatenate([np.asarray([e for e in edges if e < n], dtype=np.int64),
                           rng.integers(0, n, k, dtype=np.int64)])


def _release():
    """Returns freed device memory to the driver (the caller drops its
    tensors first), so the next 8-16 GiB allocation starts clean."""
    torch.cuda.synchronize()
    torch.cuda.empty_cache()


def test_views_step_at_full_size(acd):
    acd.set_seed(42)
    x = acd.rnorm_tensor(SHAPE, dtype="float")
    p = acd.contiguous(acd.permute_view(x, [3, 1, 2]))  # (32768, 256, 512)
    assert p.shape == (32768, 256, 512)
    pos = _sample_positions(N, 4096, 1)
    i0, i1, i2 = pos % 32768, (pos // 32768) % 256, pos // (32768 * 256)
    xidx = i1 + 256 * i2 + 256 * 512 * i0  # p[i0, i1, i2] = x[i1, i2, i0]
    assert_exact(_gather(p, pos), _gather(x, xidx), "permute -> contiguous at 2^32 elements")
    del x
    _release()

    y = acd.fused("scale_add_exp_neg_square", p, p0=0.5)
    # exp is within 2 ulp of the oracle's and the final add can cancel: the
    # bound is 2 ulp of the larger addend plus one rounding of the result
    xs = _gather(p, pos)
    ref = oracle.gauss_chain(xs, 0.5)
    bound = 2 * np.spacing(np.maximum(np.abs(xs * np.float32(0.5)), np.exp(-(xs * xs)).astype(np.float32))) + \
        np.spacing(np.abs(ref))
    err = np.abs(_gather(y, pos).astype(np.float64) - ref)
    assert np.all(err <= bound), "x*0.5 + exp(-x^2) at 2^32 elements"
    del p
    _release()

    # argmax along axis 1: fibers are contiguous runs of 32768
    a = acd.argmax(y, axis=1)
    assert a.shape == (256, 512)
    am = a.as_array()
    rng = np.random.default_rng(2)
    fibers = [(0, 0), (255, 511), (128, 256)] + [tuple(v) for v in rng.integers(0, [256, 512], (29, 2))]
    for j1, j2 in fibers:
        base = (j1 + 256 * j2) * 32768
        fib = _gather(y, np.arange(base, base + 32768, dtype=np.int64))
        assert am[j1, j2] == int(np.argmax(fib)) + 1, (j1, j2)

    # planted extremes past 2^32 - 2^20, twice each: the first index wins
    hi = [N - 2 ** 20 + 3, N - 5]
    lo = [N - 2 ** 19 + 1, N - 3]
    y.storage[hi] = 100.0
    y.storage[lo] = -100.0
    assert acd.which_max(y) == hi[0] + 1
    assert acd.which_min(y) == lo[0] + 1
    del y, a
    _release()


def test_exact_reductions_of_ones_at_full_size(acd):
    ones = acd.from_torch(torch.ones(N, dtype=torch.float32, device="cuda"), SHAPE, "float")
    assert acd.sum(ones) == float(N)
    assert acd.mean(ones) == 1.0
    assert acd.var(ones) == 0.0
    s3 = acd.tensor_sum(ones, axis=[3]).as_array()
    assert s3.shape == (256, 512) and np.all(s3 == 32768.0)
    del ones
    _release()
    ione = acd.from_torch(torch.ones(N, dtype=torch.int32, device="cuda"), SHAPE, "int32")
    r = acd.tensor_sum(ione).as_array().reshape(-1)[0]
    assert r == np.iinfo(np.int32).min  # 2^32 leaves the int32 range: NA
    s1 = acd.tensor_sum(ione, axis=[1]).as_array()
    assert np.all(s1 == 256)
    del ione
    _release()


def test_flattened_cumsum_past_2_31(acd):
    n = 2 ** 31 + 4103
    ones = acd.from_torch(torch.ones(n, dtype=torch.float32, device="cuda"), (n,), "float")
    c = acd.cumsum(ones)
    pos = _sample_positions(n, 2048, 3)
    assert_exact(_gather(c, pos), (pos + 1).astype(np.float64).astype(np.float32), "cumsum of ones past 2^31")
    acd.check_device_status()
    del ones, c
    _release()


def test_whole_tensor_softmax_past_2_31(acd):
    n = 2 ** 31 + 4103
    acd.set_seed(5)
    x = acd.rnorm_tensor((n,), dtype="float")
    sm = acd.softmax(x)
    total = acd.sum(sm)
    assert abs(total - 1.0) < 1e-5, total
    pos = _sample_positions(n, 1024, 4)
    xs = _gather(x, pos).astype(np.float64)
    ss = _gather(sm, pos).astype(np.float64)
    i, j = np.arange(0, len(pos) - 1), np.arange(1, len(pos))
    ratio = ss[i] / ss[j]
    expect = np.exp(xs[i] - xs[j])
    assert np.max(np.abs(ratio / expect - 1.0)) < 1e-6
    del x, sm
    _release()
