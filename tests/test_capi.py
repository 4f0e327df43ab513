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
    # pooled Q and K (2 x B*H x nb x D fp32) + the score matrix (B*H x nb x nb rounded to 4) at config 2
    assert f(1, 32, 86400, 128, 1, 1, 64) == 2 * 32 * 1350 * 128 * 4 + 32 * 1350 * 1352 * 4
