"""bsa_forward_noalloc -- the BSA call for callers that cannot allocate device memory.

Such callers (code running where device memory must be fixed in advance, embedders that own the
whole device budget, host bindings without a device allocator) cannot hand bsa_forward its pooled
Q/K scratch.  bsa_forward_noalloc takes that scratch from an array compiled into the library.  This
file checks, through the C ABI, that it returns what bsa_forward returns with caller-provided
scratch, on two calls in a row (the second reuses the array the first one left behind), and that a
call needing more than the fixed array is refused.  It is collected last on purpose.
"""

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

REL_L2 = 1e-2
MAX_ABS = 2e-2


def _bind(lib):
    i64p = ctypes.POINTER(ctypes.c_int64)
    vp, i, f = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
    fn = lib.bsa_forward_noalloc
    fn.argtypes = [vp, vp, vp, i, i, i, i, i, i64p, i64p, i64p, i, i, i, i, i, i, i, f, vp, i, i, i, i, i, i, vp, vp,
                   vp, vp, i64p, vp]
    fn.restype = i
    return fn


def _strides(t):
    return (ctypes.c_int64 * 3)(*t.stride()[:3])


def _call_noalloc(fn, q, k, v, shape, chunk, topk, scale):
    B, H, S, D = q.shape
    nb = S // (chunk[0] * chunk[1] * chunk[2])
    out = torch.empty_like(q)
    idx = torch.empty((B, H, nb, topk), dtype=torch.int32, device=q.device)
    dtype = 2 if q.dtype == torch.bfloat16 else 1
    rc = fn(q.data_ptr(), k.data_ptr(), v.data_ptr(), dtype, B, H, S, D, _strides(q), _strides(k), _strides(v),
            *shape, *chunk, topk, scale, None, 0, 0, 0, 0, 0, 0, None, None, idx.data_ptr(), out.data_ptr(),
            _strides(out), torch.cuda.current_stream().cuda_stream)
    return rc, out, idx


def test_noalloc_matches_forward_twice(cuda):
    from longcat_video import _native

    lib = _native.lib()
    fn = _bind(lib)
    shape, chunk, topk, scale = (1, 1, 4096), (1, 1, 64), 4, 128 ** -0.5
    for seed, dtype in ((0, torch.bfloat16), (1, torch.float16)):
        g = torch.Generator(device="cpu")
        g.manual_seed(seed)
        q, k, v = (torch.randn((1, 4, 4096, 128), generator=g).to(dtype).to(cuda) for _ in range(3))
        ref_out, ref_idx = _native.forward(q, k, v, shape, chunk, topk, scale)
        rc, out, idx = _call_noalloc(fn, q, k, v, shape, chunk, topk, scale)
        torch.cuda.synchronize()
        assert rc == 0, _native.last_error()
        assert _native.device_error(clear=True) == 0
        assert torch.equal(idx, ref_idx)
        a, b = out.float().cpu().numpy(), ref_out.float().cpu().numpy()
        rel = np.linalg.norm(a - b) / np.linalg.norm(b)
        assert rel <= REL_L2 and np.abs(a - b).max() <= MAX_ABS


def test_noalloc_rejects_oversized_requests(cuda):
    from longcat_video import _native

    lib = _native.lib()
    fn = _bind(lib)
    need = lib.bsa_forward_scratch_bytes(1, 64, 86400, 128, 1, 1, 64)
    assert need > (16 << 20)
    x = torch.zeros((1, 1, 64, 128), dtype=torch.bfloat16, device=cuda)
    st = _strides(x)
    rc = fn(x.data_ptr(), x.data_ptr(), x.data_ptr(), 2, 1, 64, 86400, 128, st, st, st, 1, 1, 86400, 1, 1, 64, 85,
            0.088, None, 0, 0, 0, 0, 0, 0, None, None, None, None, st, torch.cuda.current_stream().cuda_stream)
    assert rc == _native.BSA_ERR_SHAPE
    assert "scratch" in _native.last_error()
