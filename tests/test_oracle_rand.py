"""The counter-based generator of the oracle: Philox4x32-10 against the
known-answer vectors published with the algorithm (Random123, Salmon et al.
SC 2011), and the properties the device generator must share."""
import ctypes

import numpy as np

import oracle


def _philox(ctr, key):
    c = (ctypes.c_uint32 * 4)(*ctr)
    k = (ctypes.c_uint32 * 2)(*key)
    o = (ctypes.c_uint32 * 4)()
    oracle.lib().orc_philox(c, k, o)
    return list(o)


def test_philox4x32_10_known_answers():
    assert _philox([0, 0, 0, 0], [0, 0]) == [0x6627e8d5, 0xe169c58d, 0xbc57ac4c, 0x9b00dbd8]
    assert _philox([0xffffffff] * 4, [0xffffffff] * 2) == [0x408f276d, 0x41c83b0e, 0xa20bc7c6, 0x6d5451fd]
    assert _philox([0x243f6a88, 0x85a308d3, 0x13198a2e, 0x03707344], [0xa4093822, 0x299f31d0]) == \
        [0xd16cfe09, 0x94fdcceb, 0x5001e420, 0x24126ea1]


def test_offsets_are_global_positions():
    for dt in (np.float32, np.float64):
        for dist in ("uniform", "normal"):
            whole = oracle.rand(1003, dt, dist, 0.0, 1.0, 7)
            parts = np.concatenate([oracle.rand(5, dt, dist, 0.0, 1.0, 7, 0),
                                    oracle.rand(998, dt, dist, 0.0, 1.0, 7, 5)])
            np.testing.assert_array_equal(whole, parts)


def test_distribution_moments():
    u = oracle.rand(400000, np.float64, "uniform", -2.0, 3.0, 11)
    assert u.min() >= -2.0 and u.max() < 3.0
    assert abs(u.mean() - 0.5) < 0.02 and abs(u.var() - 25 / 12) < 0.03
    z = oracle.rand(400000, np.float32, "normal", 1.5, 2.0, 12).astype(np.float64)
    assert abs(z.mean() - 1.5) < 0.02 and abs(z.std() - 2.0) < 0.02
    # skewness and excess kurtosis of a normal are 0
    s = (z - z.mean()) / z.std()
    assert abs((s ** 3).mean()) < 0.02 and abs((s ** 4).mean() - 3.0) < 0.05
