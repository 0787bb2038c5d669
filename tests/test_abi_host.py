"""Host-side checks of the C ABI library (no GPU needed): it loads, exports
every function its headers declare, and its host-only helpers (broadcast rule,
fast division, dimension collapsing) agree with independent restatements."""
import ctypes
import os
import random
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared(header):
    text = open(os.path.join(ROOT, "include", header)).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = set(re.findall(r"\b((?:acd|tensor|launch)_\w+)\s*\(", text))
    # expand the declaration macros of acediar_launchers.h
    for m in re.finditer(r"#define (ACEDIAR_\w+)\(NAME\)((?:.*\\\n)*.*)", text):
        macro, body = m.group(1), m.group(2)
        pats = re.findall(r"tensor_##NAME##(\w+)\s*\(", body)
        pre = re.findall(r"tensor_(\w+?)_##NAME##(\w+)\s*\(", body)
        for arg in [a for a in re.findall(r"\b%s\((\w+)\)" % macro, text) if a != "NAME"]:
            for suffix in pats:
                names.add("tensor_%s%s" % (arg, suffix))
            for a, b in pre:
                names.add("tensor_%s_%s%s" % (a, arg, b))
    return {n for n in names if "##" not in n}


@pytest.fixture(scope="module")
def L():
    import acediar._lib as L
    return L


def test_library_loads_and_reports_version(L):
    assert b"sm_100a" in L.lib().acd_version()


@pytest.mark.parametrize("header", ["acd.h", "acediar_launchers.h"])
def test_every_declared_symbol_is_exported(L, header):
    names = _declared(header)
    assert len(names) > 20
    missing = [n for n in sorted(names) if not hasattr(L.lib(), n)]
    assert not missing, missing


def _reference_launchers():
    import json
    with open(os.path.join(ROOT, "tests", "golden", "reference_launchers.json")) as f:
        return json.load(f)["launchers"]


def test_every_reference_launcher_is_declared_and_exported(L):
    """Every function the reference's host code declares extern "C" (parsed
    from acediaR src/*.cpp and src/*.h by tests/golden/make_launcher_names.py)
    is declared in acediar_launchers.h and exported by the library, so the
    Rcpp modules link against it with the reference's own kernels removed."""
    ref = _reference_launchers()
    assert len(ref) == 192
    declared = _declared("acediar_launchers.h")
    not_declared = [e["name"] for e in ref if e["name"] not in declared]
    assert not not_declared, not_declared
    missing = [(e["name"], e["declared"]) for e in ref if not hasattr(L.lib(), e["name"])]
    assert not missing, missing


def _ref_broadcast(a, b):
    import oracle
    return oracle.broadcast_shape(a, b)


REFERENCE_SHAPES = [((2, 3), (3,)), ((3,), (2, 3)), ((2, 3, 4), (2, 3)), ((2, 1, 3), (1, 4, 1)),
                    ((3, 1, 2), (1, 4, 1)), ((1, 3), (2, 3)), ((3, 1), (3, 4)), ((3, 2), (2,)),
                    ((8192, 8192), (1, 8192))]
BAD_SHAPES = [((2, 3), (2, 4)), ((2, 2, 3), (4, 2))]


@pytest.mark.parametrize("a,b", REFERENCE_SHAPES)
def test_broadcast_shape_matches_reference_rule(L, a, b):
    assert L.broadcast_shape(a, b) == _ref_broadcast(a, b)


@pytest.mark.parametrize("a,b", BAD_SHAPES)
def test_broadcast_shape_rejects_like_reference(L, a, b):
    with pytest.raises(L.AcdError) as ei:
        L.broadcast_shape(a, b)
    assert re.search("shape|dimension|broadcast", str(ei.value))
    with pytest.raises(ValueError):
        _ref_broadcast(a, b)


def test_broadcast_random_agrees_with_restatement(L):
    rng = random.Random(7)
    for _ in range(400):
        na, nb = rng.randint(0, 4), rng.randint(0, 4)
        a = tuple(rng.choice([1, 1, 2, 3]) for _ in range(na))
        b = tuple(rng.choice([1, 1, 2, 3]) for _ in range(nb))
        try:
            ref = _ref_broadcast(a, b)
        except ValueError:
            ref = None
        try:
            got = L.broadcast_shape(a, b)
        except L.AcdError:
            got = None
        assert got == ref, (a, b)


def test_broadcast_strides_put_zero_on_expanded_dims(L):
    assert L.broadcast_strides((1, 8192), (1, 1), (8192, 8192)) == (0, 1)
    assert L.broadcast_strides((3,), (1,), (2, 3)) == (0, 1)
    assert L.broadcast_strides((2, 3), (1, 2), (2, 3, 4)) == (1, 2, 0)


def test_fastdiv_selftest(L):
    rng = random.Random(3)
    q = ctypes.c_uint32()
    divisors = [1, 2, 3, 5, 7, 64, 1000, 4096, 65535, 65536, 2 ** 31 - 1, 2 ** 31, 2 ** 32 - 1]
    divisors += [rng.randint(1, 2 ** 32 - 1) for _ in range(200)]
    for d in divisors:
        for n in [0, 1, d - 1, d, d + 1, 2 ** 32 - 1, rng.randint(0, 2 ** 32 - 1), rng.randint(0, 2 ** 32 - 1)]:
            n &= 0xFFFFFFFF
            assert L.lib().acd_selftest_fastdiv(d, n, ctypes.byref(q)) == 0
            assert q.value == n // d, (d, n)


def _collapse(L, shape, s_out, s_in):
    o = L.make_desc(None, L.FLOAT32, shape, s_out)
    i = L.make_desc(None, L.FLOAT32, shape, s_in)
    sh = (ctypes.c_int64 * 8)()
    so = (ctypes.c_int64 * 8)()
    si = (ctypes.c_int64 * 8)()
    nd = L.lib().acd_selftest_collapse(ctypes.byref(o), ctypes.byref(i), sh, so, si)
    return [sh[k] for k in range(nd)], [so[k] for k in range(nd)], [si[k] for k in range(nd)]


def test_collapse_turns_permute_into_2d_transpose(L):
    # permute_view(x, c(3,1,2)) of a 256x512x32768 column-major tensor
    shape = (32768, 256, 512)
    s_in = (256 * 512, 1, 256)
    s_out = (1, 32768, 32768 * 256)
    assert _collapse(L, shape, s_out, s_in) == ([32768, 131072], [1, 32768], [131072, 1])


def test_collapse_contiguous_is_1d(L):
    assert _collapse(L, (4, 5, 6), (1, 4, 20), (1, 4, 20)) == ([120], [1], [1])
    assert _collapse(L, (4, 1, 6), (1, 4, 4), (1, 99, 4)) == ([24], [1], [1])


def test_axis_validation_messages():
    import acediar.tensor as T

    class Fake:
        ndims = 2
    for bad in (5, 0, -1, 1.5):
        with pytest.raises(ValueError, match="axis must be a vector of positive integers"):
            T._axes_mask(Fake(), bad)
    assert T._axes_mask(Fake(), [1, 2])[0] == 3


def test_column_major_strides():
    import acediar.tensor as T
    assert T.col_major_strides((3, 4, 5)) == (1, 3, 12)
    assert T._is_contig((3, 1, 5), (1, 7, 3))
    assert not T._is_contig((3, 4), (4, 1))


def test_device_queries_answer_without_a_device(L):
    """gpu_available / gpu_info / gpu_memory_available never fail: without a
    usable driver they report 0 and a message."""
    import ctypes
    import torch
    lib = L.lib()
    n = lib.acd_gpu_info(None, 0)
    buf = ctypes.create_string_buffer(int(n) + 1)
    assert lib.acd_gpu_info(buf, len(buf)) == n and len(buf.value) == n
    small = ctypes.create_string_buffer(5)
    lib.acd_gpu_info(small, 5)
    assert small.value == buf.value[:4]
    if not torch.cuda.is_available():
        assert lib.acd_gpu_available() == 0 and lib.acd_gpu_memory_available() == 0.0
        assert buf.value.startswith(b"CUDA Error") or buf.value == b"No CUDA-capable devices found"
    else:
        assert lib.acd_gpu_available() == 1 and lib.acd_gpu_memory_available() > 0
        assert buf.value.startswith(b"Found %d CUDA device(s):" % torch.cuda.device_count())
