"""Random tensors on the GPU against the oracle's restatement of the same
counter-based generator: uniforms bit-exact, normals within the error of
float32 (float64) Box-Muller arithmetic, shards identical to the whole
tensor, moments of large samples, and the reference's argument errors."""
import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu
NP = {"float": np.float32, "double": np.float64}


@pytest.mark.parametrize("name", ["float", "double"])
def test_uniform_bit_exact(acd, name):
    acd.set_seed(123)
    t = acd.rand_tensor_uniform((1001, 7), dtype=name, min=-3.0, max=5.0)
    exp = oracle.rand(1001 * 7, NP[name], "uniform", -3.0, 5.0, 123, 0).reshape((1001, 7), order="F")
    np.testing.assert_array_equal(t.as_array(), exp)
    t2 = acd.rand_tensor((13,), dtype=name)  # the stream continues at position 7008 (rounded up to 4)
    np.testing.assert_array_equal(t2.as_array(), oracle.rand(13, NP[name], "uniform", 0.0, 1.0, 123, 7008))


@pytest.mark.parametrize("name", ["float", "double"])
def test_normal_matches_oracle(acd, name):
    acd.set_seed(99)
    n = 200003
    t = acd.rnorm_tensor((n,), mean=0.5, sd=2.0, dtype=name).as_array().astype(np.float64)
    exp = oracle.rand(n, NP[name], "normal", 0.5, 2.0, 99, 0).astype(np.float64)
    # absolute error bound, scaled by sd and max(1, |x|): float32 rounds
    # log, sincospi and the products in float32 (a few ulp of the radius,
    # which reaches ~5.5); float64 carries CUDA's log / sincospi errors (ulps)
    tol = 2.0 * (2e-6 if name == "float" else 1.2e-14)
    assert np.all(np.abs(t - exp) <= tol * np.maximum(1.0, np.abs(exp))), np.abs(t - exp).max()


def test_shards_equal_the_whole(acd):
    import ctypes
    import acediar._lib as L
    import acediar.tensor as T
    whole = T._alloc((4096,), "float")
    L.check(L.lib().acd_rand(T.context(), ctypes.byref(whole.desc()), 1, ctypes.c_double(0), ctypes.c_double(1),
                             ctypes.c_uint64(5), ctypes.c_uint64(1000), T._stream()), "rand")
    w = whole.as_array()
    for lo, hi in [(0, 3), (3, 2049), (2049, 4096)]:
        part = T._alloc((hi - lo,), "float")
        L.check(L.lib().acd_rand(T.context(), ctypes.byref(part.desc()), 1, ctypes.c_double(0), ctypes.c_double(1),
                                 ctypes.c_uint64(5), ctypes.c_uint64(1000 + lo), T._stream()), "rand")
        np.testing.assert_array_equal(part.as_array(), w[lo:hi])


def test_large_sample_moments(acd):
    acd.set_seed(2024)
    z = acd.rnorm_tensor((4096, 4096), dtype="float")
    assert abs(acd.tensor_mean(z).as_array()[0]) < 2e-3
    assert abs(acd.tensor_var(z).as_array()[0] - 1.0) < 2e-3
    u = acd.runif(z, -1.0, 1.0)
    assert u.shape == z.shape and u.dtype == "float"
    assert abs(acd.tensor_mean(u).as_array()[0]) < 2e-3
    assert acd.tensor_min(u).as_array()[0] >= -1.0 and acd.tensor_max(u).as_array()[0] < 1.0


def test_argument_errors(acd):
    with pytest.raises(ValueError, match="min must be less than max"):
        acd.rand_tensor_uniform((3,), min=1.0, max=1.0)
    with pytest.raises(ValueError, match="sd must be positive"):
        acd.rand_tensor_normal((3,), sd=0.0)
    with pytest.raises(ValueError, match="Use 'float' or 'double'"):
        acd.rand_tensor((3,), dtype="int32")
    with pytest.raises(ValueError, match="positive"):
        acd.rand_tensor((0, 3))
