"""acd_scan_noalloc — the scan entry point for callers that cannot allocate
device memory (it needs no context and uses a static device array).

Called through the C ABI and checked against acd_scan, the allocating entry
point, and against the oracle, on two calls in a row (the second call reuses
the array the first one left behind).  This file is collected last so that a
failure here leaves every other test already run.
"""
import ctypes

import numpy as np
import pytest
import torch

import acediar._lib as L
import acediar.tensor as T
import oracle

pytestmark = pytest.mark.gpu


def _noalloc(lib, op, out, x, axis):
    return lib.acd_scan_noalloc(op, ctypes.byref(out.desc()), ctypes.byref(x.desc()), axis,
                                ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


@pytest.mark.parametrize("name,shape,axis", [("float", (64, 100000), 2), ("double", (1 << 20) + 3, None),
                                             ("float", (333, 77), 1), ("double", (50, 70, 9), 3)])
def test_noalloc_scan_matches_acd_scan_twice(acd, name, shape, axis):
    lib = L.lib()
    lib.acd_scan_noalloc.argtypes = [ctypes.c_int32, ctypes.POINTER(L.Desc), ctypes.POINTER(L.Desc), ctypes.c_int32,
                                     ctypes.c_void_p]
    lib.acd_scan_noalloc.restype = ctypes.c_int32
    tol = 1e-5 if name == "float" else 1e-12
    rng = np.random.default_rng(12)
    shape = shape if isinstance(shape, tuple) else (shape,)
    a = -1 if axis is None else axis - 1
    for call in range(2):
        x = rng.uniform(0, 1, shape).astype(np.float32 if name == "float" else np.float64)
        t = acd.as_tensor(x, dtype=name)
        for op, opname in ((0, "cumsum"), (1, "cumprod")):
            xin = t if op == 0 else acd.as_tensor(1.0 + (x - 0.5) * 1e-3, dtype=name)
            out = T._alloc(t.shape, name)
            L.check(_noalloc(lib, op, out, xin, a), "acd_scan_noalloc")
            ref = getattr(acd, opname)(xin, axis=axis).as_array()
            got = out.as_array()
            err = np.abs(got.astype(np.float64) - ref) - tol * np.abs(ref)
            assert np.all(err <= 0), "call %d %s: max excess %g" % (call, opname, err.max())
            orc = oracle.scan(opname, xin.as_array(), a if axis is not None else None, threads=8)
            err = np.abs(got.astype(np.float64) - orc) - tol * np.abs(orc)
            assert np.all(err <= 0), "call %d %s vs oracle: max excess %g" % (call, opname, err.max())


def test_noalloc_scan_two_lanes_near_its_limit(acd):
    """Two interleaved float32 lanes: every tile costs 516 bytes of the
    static array although only 2 of its 32 lanes are real, so 2 x 4,000,000
    fits (15625 tiles, 8.06 MB) and 2 x 5,000,000 does not."""
    lib = L.lib()
    rng = np.random.default_rng(13)
    x = rng.uniform(0, 1, (2, 4_000_000)).astype(np.float32)
    t = acd.as_tensor(x, dtype="float")
    out = T._alloc(t.shape, "float")
    L.check(_noalloc(lib, 0, out, t, 1), "acd_scan_noalloc")
    orc = oracle.scan("cumsum", x, 1, threads=2)
    err = np.abs(out.as_array().astype(np.float64) - orc) - 1e-5 * np.abs(orc)
    assert np.all(err <= 0), "max excess %g" % err.max()
    big = L.make_desc(1, L.FLOAT32, (2, 5_000_000), (1, 2))
    assert lib.acd_scan_noalloc(0, ctypes.byref(big), ctypes.byref(big), 1, None) == 8


def test_noalloc_scan_rejects_beyond_its_static_scratch(acd):
    lib = L.lib()
    # 64 interleaved float32 lanes x 2^25 steps needs ~134 MB of tile state:
    # rejected on the host before any launch or memory access
    big = L.make_desc(1, L.FLOAT32, (64, 1 << 25), (1, 64))
    st = lib.acd_scan_noalloc(0, ctypes.byref(big), ctypes.byref(big), 1, None)
    assert st == 8
    assert b"static maximum" in lib.acd_last_error()
