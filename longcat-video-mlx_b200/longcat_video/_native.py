"""ctypes binding of the engine's C ABI (include/bsa_b200.h) for torch CUDA tensors.

The shared library is built in-tree by ``longcat-video-mlx_b200/build.py``.  There is no
fallback: if the library is missing or no CUDA device is present, every compute entry point
raises.  Shape / dtype / alignment errors come back as ``ValueError`` with the C layer's
message (the reference raises ``ValueError`` for the same conditions,
``block_sparse_attention.py:86-96`` and ``block_sparse_attention_metal.py:248-262``).
"""

from __future__ import annotations

import ctypes
import os
import threading
from typing import Optional, Sequence, Tuple

import torch

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib", "libbsa_b200.so")

BSA_OK = 0
BSA_ERR_SHAPE = 1
BSA_ERR_DTYPE = 2
BSA_ERR_ALIGN = 3
BSA_ERR_INDEX = 4
BSA_ERR_CUDA = 5
BSA_ERR_TIMEOUT = 6
BSA_ERR_ARG = 7

DTYPE_CODES = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}
_phase = threading.local()  # set_phase_event's event of this host thread

_lib = None
_lock = threading.Lock()

_c_i64p = ctypes.POINTER(ctypes.c_int64)
_vp = ctypes.c_void_p
_i = ctypes.c_int
_f = ctypes.c_float

_SIGNATURES = {
    "bsa_version": ([], _i),
    "bsa_last_error": ([ctypes.c_char_p, _i], _i),
    "bsa_device_error": ([_i], _i),
    "bsa_mean_pool": ([_vp, _i, _i, _i, _i, _i, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, _i, _i, _i, _i, _i, _i,
                       _vp, _i, _i, _i, _i, _i, _i, _vp, _vp, _vp], _i),
    "bsa_score_topk": ([_vp, _vp, _i, _i, _i, _i, _vp, _vp, _vp], _i),
    "bsa_block_scores": ([_vp, _vp, _i, _i, _i, _i, _vp, _vp], _i),
    "bsa_route_scratch_bytes": ([_i, _i, _i], ctypes.c_int64),
    "bsa_route_topk": ([_vp, _vp, _i, _i, _i, _i, _vp, _vp, _vp], _i),
    "bsa_topk_from_scores": ([_vp, _i, _i, _i, _vp, _vp], _i),
    "bsa_attention_indices": ([_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _c_i64p, _c_i64p, _c_i64p, _i, _i, _i, _i, _i,
                               _i, _i, _f, _vp, _c_i64p, _vp], _i),
    "bsa_forward_scratch_bytes": ([_i, _i, _i, _i, _i, _i, _i], ctypes.c_int64),
    "bsa_forward": ([_vp, _vp, _vp, _i, _i, _i, _i, _i, _c_i64p, _c_i64p, _c_i64p, _i, _i, _i, _i, _i, _i, _i, _f,
                     _vp, _i, _i, _i, _i, _i, _i, _vp, _vp, _vp, _vp, _vp, _c_i64p, _vp], _i),
    "bsa_ipc_alloc": ([ctypes.c_int64, ctypes.POINTER(ctypes.c_void_p), ctypes.c_char_p], _i),
    "bsa_ipc_free": ([_vp], _i),
    "bsa_ipc_open": ([ctypes.c_char_p, ctypes.POINTER(ctypes.c_void_p)], _i),
    "bsa_ipc_close": ([_vp], _i),
    "bsa_copy_2d": ([_vp, ctypes.c_int64, _vp, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, _vp], _i),
    "bsa_copy_3d": ([_vp, ctypes.c_int64, ctypes.c_int64, _vp, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                     ctypes.c_int64, ctypes.c_int64, _vp], _i),
    "bsa_copy_3d_list": ([_vp, _i, _vp], _i),
    "bsa_set_phase_event": ([_vp], _i),
    "bsa_attention_indices_ex": ([_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _c_i64p, _c_i64p, _c_i64p, _i, _i, _i, _i,
                                  _i, _i, _i, _f, _vp, _c_i64p, _i, _vp], _i),
    "bsa_forward_ex": ([_vp, _vp, _vp, _i, _i, _i, _i, _i, _c_i64p, _c_i64p, _c_i64p, _i, _i, _i, _i, _i, _i, _i, _f,
                        _vp, _i, _i, _i, _i, _i, _i, _vp, _vp, _vp, _vp, _vp, _c_i64p, _i, _vp], _i),
    "bsa_mean_pool_norm": ([_vp, _i, _i, _i, _i, _i, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, _i, _i, _i, _i,
                            _i, _i, _vp, _i, _i, _i, _i, _i, _i, _vp, _f, _vp, _vp, _vp], _i),
    "bsa_forward_qknorm": ([_vp, _vp, _vp, _i, _i, _i, _i, _i, _c_i64p, _c_i64p, _c_i64p, _i, _i, _i, _i, _i, _i, _i,
                            _f, _vp, _i, _i, _i, _i, _i, _i, _vp, _vp, _f, _vp, _vp, _vp, _vp, _vp, _c_i64p, _i, _vp],
                           _i),
}


class BSAError(RuntimeError):
    """A CUDA-side failure of the BSA engine (launch error, device error flag)."""


class BSAShapeError(ValueError):
    """The latent shape is not a multiple of ``chunk_thw`` or does not match S
    (``block_sparse_attention.py:86-96``).  This is the one ``ValueError`` the DiT hook turns into
    dense attention (``attention.py:174-179``); every other engine error reaches the caller."""


def library_loaded() -> bool:
    return _lib is not None


def lib():
    """Load the engine library once; raise if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise BSAError(
                    f"BSA CUDA library not found at {LIB_PATH}; build it with "
                    "`python longcat-video-mlx_b200/build.py` (there is no CPU fallback)")
            handle = ctypes.CDLL(LIB_PATH)
            for name, (args, res) in _SIGNATURES.items():
                fn = getattr(handle, name)
                fn.argtypes = args
                fn.restype = res
            _lib = handle
    return _lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(512)
    lib().bsa_last_error(buf, 512)
    return buf.value.decode(errors="replace")


def _check(rc: int, what: str) -> None:
    if rc == BSA_OK:
        return
    msg = last_error()
    if rc in (BSA_ERR_SHAPE, BSA_ERR_DTYPE, BSA_ERR_ALIGN, BSA_ERR_ARG):
        raise ValueError(msg or f"{what}: invalid argument (code {rc})")
    raise BSAError(f"{what} failed (code {rc}): {msg}")


def device_error(clear: bool = True) -> int:
    """Sticky device-side error code (0 = none); synchronises the device."""
    return int(lib().bsa_device_error(1 if clear else 0))


def _require_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if not isinstance(t, torch.Tensor):
            raise TypeError("expected torch tensors")
        if not t.is_cuda:
            raise ValueError("BSA engine inputs must be CUDA tensors (there is no CPU path)")


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _strides(t: torch.Tensor):
    if t.stride(-1) != 1:
        raise ValueError("the last (head_dim) axis must be contiguous")
    arr = (ctypes.c_int64 * 3)(t.stride(0), t.stride(1), t.stride(2))
    return arr


def _merge_batch(t: torch.Tensor) -> torch.Tensor:
    """A view the kernels can read in place, else a one-time contiguous copy.

    The kernels read q/k/v through TMA maps: the base address and every stride must be multiples of
    16 bytes, and the last axis of the attention map is b*H + h, so for B > 1 the batch stride must
    equal H times the head stride.  Views that break either rule (the DiT's
    ``reshape(B, N, 3, H, D).permute(2, 0, 3, 1, 4)`` at B > 1, a narrowed or offset view) are copied
    once to a contiguous layout; everything else is used in place."""
    if t.dim() != 4:
        return t
    if _misaligned(t):
        return t.clone(memory_format=torch.contiguous_format)  # a fresh, aligned allocation
    if t.shape[0] > 1 and t.stride(0) != t.shape[1] * t.stride(1):
        return t.contiguous()
    return t


def _misaligned(t: torch.Tensor) -> bool:
    e = t.element_size()
    return bool(t.data_ptr() % 16 or any((t.stride(i) * e) % 16 for i in range(t.dim() - 1) if t.shape[i] > 1))


def _aligned(t: torch.Tensor) -> torch.Tensor:
    """The pooling kernels accept any batch and head strides but need a 16-byte aligned base and
    16-byte multiple strides; other views are copied once to a contiguous layout."""
    return t.clone(memory_format=torch.contiguous_format) if t.dim() == 4 and _misaligned(t) else t


def _dtype_code(t: torch.Tensor) -> int:
    try:
        return DTYPE_CODES[t.dtype]
    except KeyError:
        raise ValueError(f"unsupported dtype {t.dtype}") from None


def _geometry(S: int, shape: Sequence[int], chunk_thw: Sequence[int]):
    T, H_, W = (int(v) for v in shape)
    cT, cH, cW = (int(v) for v in chunk_thw)
    if T % cT or H_ % cH or W % cW:
        raise BSAShapeError(
            f"Latent shape ({T}, {H_}, {W}) must be a multiple of "
            f"chunk_thw {tuple(chunk_thw)}; refinement padding should guarantee this.")
    if S != T * H_ * W:
        raise BSAShapeError(f"S={S} doesn't match T*H*W={T * H_ * W} for shape {tuple(shape)}")
    return T, H_, W, cT, cH, cW


# ------------------------------------------------------------------------------------ ops
def _norm_weight(w: torch.Tensor, like: torch.Tensor) -> torch.Tensor:
    """An RMSNorm weight as the kernels read it: [D], the input's dtype and device, contiguous."""
    w = w.detach().to(device=like.device, dtype=like.dtype).contiguous()
    if w.dim() != 1 or w.numel() != like.shape[-1]:
        raise ValueError(f"norm weight must be [{like.shape[-1]}]")
    return w


def mean_pool(x: torch.Tensor, shape, chunk_thw, rope: Optional[Tuple] = None,
              norm: Optional[Tuple[torch.Tensor, float]] = None) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """fp32 block means [B, H, nb, D]; with ``rope=(tables, dims, grid)`` and / or ``norm=(weight, eps)``
    (the DiT's q/k RMSNorm, fused before the RoPE) also the transformed x."""
    _require_cuda(x)
    if x.dim() != 4:
        raise ValueError("expected x of shape [B, H, S, D]")
    B, H, S, D = x.shape
    T, H_, W, cT, cH, cW = _geometry(S, shape, chunk_thw)
    nb = S // (cT * cH * cW)
    x = _aligned(x)
    pooled = torch.empty((B, H, nb, D), device=x.device, dtype=torch.float32)
    st = _strides(x)
    x_rot = None
    rope_ptr, rdims, rgrid = None, (0, 0, 0), (0, 0, 0)
    if rope is not None:
        tables, rdims, rgrid = rope
        rope_ptr = tables.data_ptr()
    if rope is not None or norm is not None:
        x_rot = torch.empty((B, H, S, D), device=x.device, dtype=x.dtype)
    if norm is not None:
        w = _norm_weight(norm[0], x)
        rc = lib().bsa_mean_pool_norm(x.data_ptr(), _dtype_code(x), B, H, S, D, st[0], st[1], st[2], T, H_, W, cT, cH,
                                      cW, rope_ptr, rdims[0], rdims[1], rdims[2], rgrid[0], rgrid[1], rgrid[2],
                                      w.data_ptr(), float(norm[1]), x_rot.data_ptr(), pooled.data_ptr(), _stream(x))
        _check(rc, "bsa_mean_pool_norm")
        return pooled, x_rot
    rc = lib().bsa_mean_pool(x.data_ptr(), _dtype_code(x), B, H, S, D, st[0], st[1], st[2], T, H_, W, cT, cH, cW,
                             rope_ptr, rdims[0], rdims[1], rdims[2], rgrid[0], rgrid[1], rgrid[2],
                             x_rot.data_ptr() if x_rot is not None else None, pooled.data_ptr(), _stream(x))
    _check(rc, "bsa_mean_pool")
    return pooled, x_rot


def score_topk(qp: torch.Tensor, kp: torch.Tensor, topk: int, return_scores: bool = False):
    """Block scores + per-row top-k.  qp, kp: [B, H, nb, D] fp32 contiguous.  Without ``return_scores``
    the routing runs without materialising the score matrix (bsa_route_topk) where it supports the size;
    both paths return the same indices."""
    _require_cuda(qp, kp)
    if qp.dtype != torch.float32 or kp.dtype != torch.float32:
        raise ValueError("pooled blocks must be fp32")
    qp = qp.contiguous()
    kp = kp.contiguous()
    B, H, nb, D = qp.shape
    if kp.shape != qp.shape:
        raise ValueError("q and k block tensors must have the same shape for top-k routing")
    idx = torch.empty((B, H, nb, topk), device=qp.device, dtype=torch.int32)
    nbytes = int(lib().bsa_route_scratch_bytes(B * H, nb, D)) if not return_scores else 0
    if nbytes > 0:
        scratch = torch.empty((nbytes,), device=qp.device, dtype=torch.uint8)
        rc = lib().bsa_route_topk(qp.data_ptr(), kp.data_ptr(), B * H, nb, D, int(topk), idx.data_ptr(),
                                  scratch.data_ptr(), _stream(qp))
        _check(rc, "bsa_route_topk")
        return idx, None
    scores = torch.empty((B, H, nb, nb), device=qp.device, dtype=torch.float32)  # GEMM output, top-k input
    rc = lib().bsa_score_topk(qp.data_ptr(), kp.data_ptr(), B * H, nb, D, int(topk), idx.data_ptr(),
                              scores.data_ptr(), _stream(qp))
    _check(rc, "bsa_score_topk")
    return idx, (scores if return_scores else None)


def topk_from_scores(score: torch.Tensor, topk: int) -> torch.Tensor:
    """[..., nq, nk] fp32 scores -> [..., nq, topk] int32 ascending block ids."""
    _require_cuda(score)
    s = score.to(torch.float32).contiguous()
    nk = s.shape[-1]
    rows = s.numel() // nk if nk else 0
    idx = torch.empty((*s.shape[:-1], int(topk)), device=s.device, dtype=torch.int32)
    rc = lib().bsa_topk_from_scores(s.data_ptr(), rows, nk, int(topk), idx.data_ptr(), _stream(s))
    _check(rc, "bsa_topk_from_scores")
    return idx


def block_scores(qp: torch.Tensor, kp: torch.Tensor) -> torch.Tensor:
    _require_cuda(qp, kp)
    qp = qp.to(torch.float32).contiguous()
    kp = kp.to(torch.float32).contiguous()
    *lead, nq, D = qp.shape
    nk = kp.shape[-2]
    BH = 1
    for v in lead:
        BH *= int(v)
    out = torch.empty((*lead, nq, nk), device=qp.device, dtype=torch.float32)
    rc = lib().bsa_block_scores(qp.data_ptr(), kp.data_ptr(), BH, nq, nk, D, out.data_ptr(), _stream(qp))
    _check(rc, "bsa_block_scores")
    return out


def attention_indices(q, k, v, block_indices, shape, chunk_thw, sm_scale: float,
                      out: Optional[torch.Tensor] = None) -> torch.Tensor:
    _require_cuda(q, k, v, block_indices)
    if q.shape != k.shape or q.shape != v.shape:
        raise ValueError("q, k, v must have the same shape [B, H, S, D]")
    if q.dtype != k.dtype or q.dtype != v.dtype:
        raise ValueError("q, k, v must share one dtype")
    B, H, S, D = q.shape
    T, H_, W, cT, cH, cW = _geometry(S, shape, chunk_thw)
    bi = block_indices
    if bi.dtype != torch.int32:
        bi = bi.to(torch.int32)
    bi = bi.contiguous()
    nb = S // (cT * cH * cW)
    if bi.dim() != 4 or tuple(bi.shape[:3]) != (B, H, nb):
        raise ValueError(f"block_indices must be [B, H, {nb}, top_k], got {tuple(bi.shape)}")
    if q.dtype == torch.float32:
        # fp32 I/O (the reference kernels accept it): fp16 copies on the device, fp32 result
        o16 = torch.empty((B, H, S, D), device=q.device, dtype=torch.float16)
        _attention_ex(*(t.to(torch.float16) for t in (q, k, v)), bi, shape, chunk_thw, sm_scale, o16, 0)
        if out is None:
            return o16.float()
        out.copy_(o16)
        return out
    if out is None:
        out = torch.empty((B, H, S, D), device=q.device, dtype=q.dtype)
    q, k, v = _merge_batch(q), _merge_batch(k), _merge_batch(v)
    rc = lib().bsa_attention_indices(q.data_ptr(), k.data_ptr(), v.data_ptr(), bi.data_ptr(), _dtype_code(q), B, H, S,
                                     D, _strides(q), _strides(k), _strides(v), T, H_, W, cT, cH, cW, int(bi.shape[-1]),
                                     float(sm_scale), out.data_ptr(), _strides(out), _stream(q))
    _check(rc, "bsa_attention_indices")
    return out


def _forward_f32(q, k, v, shape, chunk_thw, topk, sm_scale, rope, out, block_indices, sm_reserve):
    """fp32 inputs (the reference's config-1 dtype): routing runs on the fp32 values (pooling,
    scores and top-k exactly as for 16-bit inputs); the sparse attention runs on fp16 copies made on
    the device (fp16 keeps 11 significant bits, a relative error of ~5e-4 per input, well inside the
    1e-2 output contract) and the output is returned in fp32."""
    B, H, S, D = q.shape
    qr, kr = q, k
    if rope is not None:
        qp, qr = mean_pool(q, shape, chunk_thw, rope=rope)
        kp, kr = mean_pool(k, shape, chunk_thw, rope=rope)
    else:
        qp, _ = mean_pool(q, shape, chunk_thw)
        kp, _ = mean_pool(k, shape, chunk_thw)
    idx, _ = score_topk(qp, kp, topk)
    if block_indices is not None:
        block_indices.copy_(idx)
        idx = block_indices
    ev = getattr(_phase, "event", None)
    if ev is not None:
        ev.record(torch.cuda.current_stream(q.device))
    o16 = torch.empty((B, H, S, D), device=q.device, dtype=torch.float16)
    qh, kh, vh = (t.to(torch.float16) for t in (qr, kr, v))
    _attention_ex(qh, kh, vh, idx, shape, chunk_thw, sm_scale, o16, sm_reserve)
    if out is None:
        return o16.float(), idx
    out.copy_(o16)
    return out, idx


def _attention_ex(q, k, v, bi, shape, chunk_thw, sm_scale, out, sm_reserve):
    q, k, v = _merge_batch(q), _merge_batch(k), _merge_batch(v)
    B, H, S, D = q.shape
    T, H_, W, cT, cH, cW = _geometry(S, shape, chunk_thw)
    rc = lib().bsa_attention_indices_ex(q.data_ptr(), k.data_ptr(), v.data_ptr(), bi.data_ptr(), _dtype_code(q), B,
                                        H, S, D, _strides(q), _strides(k), _strides(v), T, H_, W, cT, cH, cW,
                                        int(bi.shape[-1]), float(sm_scale), out.data_ptr(), _strides(out),
                                        int(sm_reserve), _stream(q))
    _check(rc, "bsa_attention_indices")


def forward(q, k, v, shape, chunk_thw, topk: int, sm_scale: float, rope: Optional[Tuple] = None,
            out: Optional[torch.Tensor] = None, block_indices: Optional[torch.Tensor] = None,
            scratch: Optional[torch.Tensor] = None, sm_reserve: int = 0,
            qk_norm: Optional[Tuple[torch.Tensor, torch.Tensor, float]] = None):
    """Full BSA call (pool -> score -> top-k -> sparse attention).  Returns (out, block_indices).
    ``sm_reserve`` SMs stay free of the persistent attention kernel (for a concurrent exchange).
    ``qk_norm=(q_weight, k_weight, eps)``: q and k are the raw projections; their RMSNorm runs fused
    with the RoPE and the pooling (bsa_forward_qknorm)."""
    _require_cuda(q, k, v)
    if q.shape != k.shape or q.shape != v.shape:
        raise ValueError("q, k, v must have the same shape [B, H, S, D]")
    if q.dtype != k.dtype or q.dtype != v.dtype:
        raise ValueError("q, k, v must share one dtype")
    B, H, S, D = q.shape
    T, H_, W, cT, cH, cW = _geometry(S, shape, chunk_thw)
    nb = S // (cT * cH * cW)
    if q.dtype == torch.float32:
        if qk_norm is not None:
            raise ValueError("the fused q/k norm runs on bf16 / fp16 inputs")
        return _forward_f32(q, k, v, shape, chunk_thw, topk, sm_scale, rope, out, block_indices, sm_reserve)
    q, k, v = _merge_batch(q), _merge_batch(k), _merge_batch(v)
    if out is None:
        out = torch.empty((B, H, S, D), device=q.device, dtype=q.dtype)
    if block_indices is None:
        block_indices = torch.empty((B, H, nb, int(topk)), device=q.device, dtype=torch.int32)
    nbytes = int(lib().bsa_forward_scratch_bytes(B, H, S, D, cT, cH, cW))
    if scratch is None or scratch.numel() * scratch.element_size() < nbytes:
        scratch = torch.empty((max(nbytes, 16),), device=q.device, dtype=torch.uint8)
    rope_ptr, rdims, rgrid = None, (0, 0, 0), (0, 0, 0)
    q_rot = k_rot = None
    if rope is not None:
        tables, rdims, rgrid = rope
        rope_ptr = tables.data_ptr()
    if rope is not None or qk_norm is not None:
        q_rot = torch.empty((B, H, S, D), device=q.device, dtype=q.dtype)
        k_rot = torch.empty((B, H, S, D), device=q.device, dtype=q.dtype)
    if qk_norm is not None:
        wq, wk = _norm_weight(qk_norm[0], q), _norm_weight(qk_norm[1], k)
        rc = lib().bsa_forward_qknorm(q.data_ptr(), k.data_ptr(), v.data_ptr(), _dtype_code(q), B, H, S, D,
                                      _strides(q), _strides(k), _strides(v), T, H_, W, cT, cH, cW, int(topk),
                                      float(sm_scale), rope_ptr, rdims[0], rdims[1], rdims[2], rgrid[0], rgrid[1],
                                      rgrid[2], wq.data_ptr(), wk.data_ptr(), float(qk_norm[2]), q_rot.data_ptr(),
                                      k_rot.data_ptr(), scratch.data_ptr(), block_indices.data_ptr(), out.data_ptr(),
                                      _strides(out), int(sm_reserve), _stream(q))
        _check(rc, "bsa_forward_qknorm")
        return out, block_indices
    rc = lib().bsa_forward_ex(q.data_ptr(), k.data_ptr(), v.data_ptr(), _dtype_code(q), B, H, S, D, _strides(q),
                           _strides(k), _strides(v), T, H_, W, cT, cH, cW, int(topk), float(sm_scale), rope_ptr,
                           rdims[0], rdims[1], rdims[2], rgrid[0], rgrid[1], rgrid[2],
                           q_rot.data_ptr() if q_rot is not None else None,
                           k_rot.data_ptr() if k_rot is not None else None, scratch.data_ptr(),
                           block_indices.data_ptr(), out.data_ptr(), _strides(out), int(sm_reserve), _stream(q))
    _check(rc, "bsa_forward")
    return out, block_indices


# ------------------------------------------------------------------ peer exchange helpers
IPC_HANDLE_BYTES = 64


def ipc_alloc(nbytes: int) -> Tuple[int, bytes]:
    """cudaMalloc on the current device, exported for other processes: (pointer, handle bytes)."""
    ptr = ctypes.c_void_p()
    h = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
    _check(lib().bsa_ipc_alloc(int(nbytes), ctypes.byref(ptr), h), "bsa_ipc_alloc")
    return int(ptr.value), h.raw


def ipc_free(ptr: int) -> None:
    _check(lib().bsa_ipc_free(ptr), "bsa_ipc_free")


def ipc_open(handle: bytes) -> int:
    """Map a buffer another process of the node exported; returns its address in this process."""
    if len(handle) != IPC_HANDLE_BYTES:
        raise ValueError("IPC handle must be 64 bytes")
    ptr = ctypes.c_void_p()
    _check(lib().bsa_ipc_open(handle, ctypes.byref(ptr)), "bsa_ipc_open")
    return int(ptr.value)


def ipc_close(ptr: int) -> None:
    _check(lib().bsa_ipc_close(ptr), "bsa_ipc_close")


def copy_2d(dst: int, dpitch: int, src: int, spitch: int, width: int, height: int, stream) -> None:
    """`height` rows of `width` bytes between any local / mapped-peer addresses, on `stream`."""
    _check(lib().bsa_copy_2d(dst, dpitch, src, spitch, width, height, stream.cuda_stream), "bsa_copy_2d")


def set_phase_event(event) -> None:
    """Record `event` (a torch.cuda.Event, or None to stop) between the routing and the attention launches
    of this thread's later forward calls (profiling: the two phases of one call)."""
    handle = None
    if event is not None:
        if not event.cuda_event:  # torch creates the CUDA event at its first record
            event.record(torch.cuda.current_stream())
        handle = event.cuda_event
    _check(lib().bsa_set_phase_event(handle), "bsa_set_phase_event")
    _phase.event = event  # the fp32 path (routing and attention as separate calls) records it here


def copy_3d_list(desc, n: int, stream) -> None:
    """n copies of a prebuilt ctypes int64 array of (dst, dpitch, dslice, src, spitch, sslice, width, height,
    depth) rows (bsa_copy_3d), in order on `stream`, in one host call."""
    if n:
        _check(lib().bsa_copy_3d_list(ctypes.cast(desc, ctypes.c_void_p), int(n), stream.cuda_stream),
               "bsa_copy_3d_list")


class _DevBuf:
    """__cuda_array_interface__ view of a raw device allocation (torch.as_tensor wraps it, no copy)."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(int(x) for x in shape), "typestr": typestr,
                                         "data": (int(ptr), False), "version": 3, "strides": None,
                                         "stream": None}


def wrap_device(ptr: int, shape, dtype: torch.dtype, device) -> torch.Tensor:
    """A torch tensor over raw device memory at `ptr` (the caller keeps the memory alive)."""
    if dtype in (torch.bfloat16, torch.float16):
        t = torch.as_tensor(_DevBuf(ptr, shape, "<i2"), device=device)
        return t.view(dtype)
    if dtype == torch.float32:
        return torch.as_tensor(_DevBuf(ptr, shape, "<f4"), device=device)
    if dtype == torch.int32:
        return torch.as_tensor(_DevBuf(ptr, shape, "<i4"), device=device)
    raise ValueError(f"unsupported dtype {dtype}")
