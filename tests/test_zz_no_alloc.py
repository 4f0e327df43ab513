"""bsa_forward_noalloc -- the BSA call for callers that cannot allocate device memory.

Such callers (code running where device memory must be fixed in advance, embedders that own the
whole device budget, host bindings without a device allocator) cannot hand bsa_forward its
scratch.  bsa_forward_noalloc takes that scratch from an array compiled into the library.  This
file checks, through the C ABI, that it returns exactly what bsa_forward returns with
caller-provided scratch: the same kernels run on the same values, so outputs and routing must be
bit-identical.  It does so on calls in a row that reuse the array the previous call left behind,
including a larger call followed by a smaller one and a call with fused 3-D RoPE, and it checks
that a call needing more than the fixed array is refused.  It is collected last on purpose.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


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


def _call_noalloc(fn, q, k, v, shape, chunk, topk, scale, rope=None):
    B, H, S, D = q.shape
    nb = S // (chunk[0] * chunk[1] * chunk[2])
    out = torch.empty_like(q)
    idx = torch.empty((B, H, nb, topk), dtype=torch.int32, device=q.device)
    dtype = 2 if q.dtype == torch.bfloat16 else 1
    rope_ptr, dims, grid, q_rot, k_rot = None, (0, 0, 0), (0, 0, 0), None, None
    if rope is not None:
        tables, dims, grid = rope.native_args()
        rope_ptr = tables.data_ptr()
        q_rot, k_rot = torch.empty_like(q), torch.empty_like(k)
    rc = fn(q.data_ptr(), k.data_ptr(), v.data_ptr(), dtype, B, H, S, D, _strides(q), _strides(k), _strides(v),
            *shape, *chunk, topk, scale, rope_ptr, *dims, *grid, q_rot.data_ptr() if q_rot is not None else None,
            k_rot.data_ptr() if k_rot is not None else None, idx.data_ptr(), out.data_ptr(), _strides(out),
            torch.cuda.current_stream().cuda_stream)
    return rc, out, idx


def _inputs(seed, B, H, S, dtype, cuda):
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    return tuple(torch.randn((B, H, S, 128), generator=g).to(dtype).to(cuda) for _ in range(3))


def test_noalloc_matches_forward_on_calls_in_a_row(cuda):
    from longcat_video import _native
    from longcat_video.models.rope_3d import RopeTables

    fn = _bind(_native.lib())
    scale = 128 ** -0.5
    # (seed, dtype, heads, S, topk, rope grid): the second call is smaller than the first, so it runs
    # over scratch whose tail still holds the first call's values; the third fuses 3-D RoPE
    calls = [(0, torch.bfloat16, 4, 4096, 4, None), (1, torch.float16, 2, 1024, 3, None),
             (2, torch.bfloat16, 2, 2048, 5, (4, 8, 64))]
    for seed, dtype, H, S, topk, grid in calls:
        q, k, v = _inputs(seed, 1, H, S, dtype, cuda)
        shape, chunk = (1, 1, S), (1, 1, 64)
        rope = RopeTables(grid, 128, cuda) if grid is not None else None
        ref_out, ref_idx = _native.forward(q, k, v, shape, chunk, topk, scale,
                                           rope=rope.native_args() if rope is not None else None)
        rc, out, idx = _call_noalloc(fn, q, k, v, shape, chunk, topk, scale, rope=rope)
        torch.cuda.synchronize()
        assert rc == 0, _native.last_error()
        assert _native.device_error(clear=True) == 0
        assert torch.equal(idx, ref_idx), (seed, H, S)
        assert torch.equal(out, ref_out), (seed, H, S)


def test_noalloc_rejects_oversized_requests(cuda):
    from longcat_video import _native

    lib = _native.lib()
    fn = _bind(lib)
    need = lib.bsa_forward_scratch_bytes(1, 64, 86400, 128, 1, 1, 64)
    assert need > (16 << 20)
    x = torch.zeros((1, 1, 64, 128), dtype=torch.bfloat16, device=cuda)
    st = _strides(x)
    idx = torch.zeros((1, 64, 1350, 85), dtype=torch.int32, device=cuda)
    rc = fn(x.data_ptr(), x.data_ptr(), x.data_ptr(), 2, 1, 64, 86400, 128, st, st, st, 1, 1, 86400, 1, 1, 64, 85,
            0.088, None, 0, 0, 0, 0, 0, 0, None, None, idx.data_ptr(), x.data_ptr(), st,
            torch.cuda.current_stream().cuda_stream)
    assert rc == _native.BSA_ERR_SHAPE
    assert "scratch" in _native.last_error()
