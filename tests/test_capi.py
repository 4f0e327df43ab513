"""The C-ABI library loads and exports every entry point include/bsa_b200.h declares (no GPU
compute: only symbol lookup, the version and argument validation that fails before any launch)."""

import ctypes
import os
import re

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "bsa_b200.h")


def _declared():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(bsa_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    import sys

    sys.path.insert(0, os.path.join(REPO, "longcat-video-mlx_b200"))
    import build  # longcat-video-mlx_b200/build.py

    path = build.build()
    return ctypes.CDLL(path)


def test_header_declares_entry_points():
    names = _declared()
    for n in ("bsa_mean_pool", "bsa_score_topk", "bsa_attention_indices", "bsa_forward", "bsa_version"):
        assert n in names


def test_library_exports_every_declared_symbol(lib):
    missing = [n for n in _declared() if not hasattr(lib, n)]
    assert not missing, missing


def test_version(lib):
    lib.bsa_version.restype = ctypes.c_int
    assert lib.bsa_version() >= 100


def test_argument_validation_before_launch(lib):
    # a null pointer is rejected on the host (no CUDA call is made)
    f = lib.bsa_score_topk
    f.restype = ctypes.c_int
    rc = f(None, None, 1, 4, 8, 2, None, None, None)
    assert rc == 7  # BSA_ERR_ARG
    buf = ctypes.create_string_buffer(256)
    lib.bsa_last_error(buf, 256)
    assert b"null" in buf.value


def test_forward_scratch_size(lib):
    f = lib.bsa_forward_scratch_bytes
    f.restype = ctypes.c_int64
    f.argtypes = [ctypes.c_int] * 7
    r = lib.bsa_route_scratch_bytes
    r.restype = ctypes.c_int64
    r.argtypes = [ctypes.c_int] * 3
    up = lambda b: (b + 255) // 256 * 256
    rows = 32 * 1350
    # config 2: pooled Q and K (fp32), then the routing scratch: bf16 hi/lo pairs of both (128 columns),
    # their norms, the per-head maximum key norm (+ a counter), the fallback row list and the 16-bit
    # score keys (rows padded to 8)
    route = up(4 * rows * 128 * 2) + up(2 * rows * 4) + up((32 + 4) * 4) + up(rows * 4) + up(rows * 1352 * 2)
    assert r(32, 1350, 128) == route
    assert f(1, 32, 86400, 128, 1, 1, 64) == up(2 * rows * 128 * 4) + route
    # beyond 3,072 blocks per row the score matrix is used instead
    assert r(1, 3073, 128) == 0
    assert f(1, 1, 3073 * 64, 128, 1, 1, 64) == up(2 * 3073 * 128 * 4) + 3073 * 3076 * 4


def _forward_args(lib, name):
    i64p = ctypes.POINTER(ctypes.c_int64)
    vp, i, f = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
    fn = getattr(lib, name)
    head = [vp, vp, vp, i, i, i, i, i, i64p, i64p, i64p, i, i, i, i, i, i, i, f, vp, i, i, i, i, i, i, vp, vp]
    fn.argtypes = head + ([vp] if name == "bsa_forward" else []) + [vp, vp, i64p, vp]
    fn.restype = i
    return fn


@pytest.mark.parametrize("name", ["bsa_forward", "bsa_forward_noalloc"])
@pytest.mark.parametrize("missing", ["block_indices", "out", "out_strides"])
def test_forward_rejects_null_outputs_before_any_launch(lib, name, missing):
    """A null output is refused on the host with BSA_ERR_ARG.  The checks run before the first CUDA call,
    so the pointers below (never dereferenced) and the absent GPU are never touched."""
    fn = _forward_args(lib, name)
    fake = 1 << 20  # 16-byte aligned, never dereferenced
    st = (ctypes.c_int64 * 3)(64 * 128, 64 * 128, 128)
    B, H, S, D = 1, 1, 64, 128
    idx = None if missing == "block_indices" else fake
    out = None if missing == "out" else fake
    ost = None if missing == "out_strides" else st
    args = [fake, fake, fake, 2, B, H, S, D, st, st, st, 1, 1, 64, 1, 1, 64, 1, 0.088, None, 0, 0, 0, 0, 0, 0, None,
            None]
    if name == "bsa_forward":
        args.append(fake)  # scratch
    args += [idx, out, ost, None]
    assert fn(*args) == 7  # BSA_ERR_ARG
    buf = ctypes.create_string_buffer(256)
    lib.bsa_last_error(buf, 256)
    assert b"null" in buf.value


def test_forward_rejects_bad_topk_before_any_launch(lib):
    fn = _forward_args(lib, "bsa_forward")
    fake = 1 << 20
    st = (ctypes.c_int64 * 3)(64 * 128, 64 * 128, 128)
    for topk in (0, 2):  # one 64-token block: topk must be 1
        rc = fn(fake, fake, fake, 2, 1, 1, 64, 128, st, st, st, 1, 1, 64, 1, 1, 64, topk, 0.088, None, 0, 0, 0, 0, 0, 0,
                None, None, fake, fake, fake, st, None)
        assert rc == 1  # BSA_ERR_SHAPE
