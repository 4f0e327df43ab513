"""CPU oracle for the block-sparse attention (BSA) hot path -- TEST INFRASTRUCTURE ONLY.

This module restates the reference's Tier A algorithm (xocialize/longcat-video-mlx,
``longcat_video/models/block_sparse_attention.py``) in numpy so the CUDA engine can be
checked against it.  Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline
leg of ``bench.py`` may import it; the engine itself never does.

Parity pins (the reference cannot run here: it is MLX-only and MLX is not installable):
  * the reference's own known-answer tests (``tests/smoke/test_bsa_tier_a_smoke.py``)
    are re-run against this module in ``tests/test_oracle_kat.py``;
  * tie-breaking inside ``mx.argpartition`` is unspecified by the reference, so the
    selection rule here is defined explicitly (score descending, then block index
    ascending) and indices are returned sorted ascending.  That part is "parity
    unpinned" with respect to MLX.

Precision: the reference pools and scores in the input dtype (``:104, :112``).  The
oracle (and the engine) upcast to fp32 first, as the engine's contract defines
correctness against an fp32 reference.  Pooling uses a fixed pairwise summation
order and scoring a fixed fma chain (``oracle/bsa_oracle.c``) so that the engine's fp32
pooled scores, and therefore its selected indices, can be compared bit-exactly.
"""

from __future__ import annotations

import ctypes
import math
import os
from typing import Optional, Sequence

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libbsa_oracle.so")
_lib = None


# ----------------------------------------------------------------------------- dtype helpers
def to_f32(x) -> np.ndarray:
    """Exact upcast of an array (numpy or torch CPU tensor, any float dtype) to fp32."""
    if hasattr(x, "detach"):
        import torch

        return x.detach().to("cpu", torch.float32).numpy()
    return np.asarray(x, dtype=np.float32)


def round_to_bf16(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 (round to nearest even) -> fp32, bit-exact with ``cvt.rn.bf16.f32``."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    nan = np.isnan(x)
    out = (rounded.astype(np.uint32) << 16).view(np.float32)
    out = np.where(nan, np.float32(np.nan), out)
    return out.astype(np.float32)


def round_to_f16(x: np.ndarray) -> np.ndarray:
    """fp32 -> fp16 (round to nearest even) -> fp32."""
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "bf16":
        return round_to_bf16(x)
    if dtype == "fp16":
        return round_to_f16(x)
    return np.asarray(x, dtype=np.float32)


# ----------------------------------------------------------------------------- geometry
def _check_shape(shape, chunk_thw, S: Optional[int] = None):
    """Divisibility checks of block_sparse_attention.py:86-96 (same messages)."""
    T, H_, W = shape
    cT, cH, cW = chunk_thw
    if T % cT or H_ % cH or W % cW:
        raise ValueError(
            f"Latent shape ({T}, {H_}, {W}) must be a multiple of "
            f"chunk_thw {tuple(chunk_thw)}; refinement padding should guarantee this."
        )
    if S is not None and S != T * H_ * W:
        raise ValueError(f"S={S} doesn't match T*H*W={T * H_ * W} for shape {tuple(shape)}")


def to_block_major(x: np.ndarray, shape, chunk_thw) -> np.ndarray:
    """[..., S, D] t-major -> [..., nb, n, D] block-major (block_sparse_attention.py:98-104,
    block_sparse_attention_metal.py:185-205): blocks in (bt, bh, bw) order, tokens inside a
    block in (ct, ch, cw) order."""
    T, H_, W = shape
    cT, cH, cW = chunk_thw
    Bt, Bh, Bw = T // cT, H_ // cH, W // cW
    lead = x.shape[:-2]
    D = x.shape[-1]
    y = x.reshape(*lead, Bt, cT, Bh, cH, Bw, cW, D)
    nl = len(lead)
    perm = list(range(nl)) + [nl + 0, nl + 2, nl + 4, nl + 1, nl + 3, nl + 5, nl + 6]
    y = y.transpose(perm)
    return y.reshape(*lead, Bt * Bh * Bw, cT * cH * cW, D)


def from_block_major(y: np.ndarray, shape, chunk_thw) -> np.ndarray:
    """Inverse of ``to_block_major`` (block_sparse_attention_metal.py:208-221)."""
    T, H_, W = shape
    cT, cH, cW = chunk_thw
    Bt, Bh, Bw = T // cT, H_ // cH, W // cW
    lead = y.shape[:-3]
    D = y.shape[-1]
    z = y.reshape(*lead, Bt, Bh, Bw, cT, cH, cW, D)
    nl = len(lead)
    perm = list(range(nl)) + [nl + 0, nl + 3, nl + 1, nl + 4, nl + 2, nl + 5, nl + 6]
    z = z.transpose(perm)
    return z.reshape(*lead, T * H_ * W, D)


def _pairwise_sum(y: np.ndarray, axis: int) -> np.ndarray:
    """Sum along `axis` (power-of-two length) in the fixed order the engine uses: a pairwise
    tree over adjacent elements, (x0 + x1), (x2 + x3), ... then pairs of those, each add an
    fp32 round-to-nearest operation."""
    y = np.moveaxis(np.asarray(y, dtype=np.float32), axis, 0)
    n = y.shape[0]
    if n & (n - 1):
        raise ValueError("the pairwise order needs a power-of-two length")
    while n > 1:
        y = (y[0::2] + y[1::2]).astype(np.float32)
        n //= 2
    return y[0]


# ----------------------------------------------------------------------------- Tier A pieces
def mean_pool_blocks_3d(x, shape, chunk_thw=(4, 4, 4)) -> np.ndarray:
    """block_sparse_attention.py:67-104.  [B,H,S,D] -> fp32 [B,H,nb,D] in (bt,bh,bw) order.
    fp32 mean with the pairwise order; the 1/n scale is exact for n a power of two."""
    x = to_f32(x)
    B, H, S, D = x.shape
    _check_shape(shape, chunk_thw, S)
    y = to_block_major(x, shape, chunk_thw)  # [B,H,nb,n,D]
    n = y.shape[-2]
    if n & (n - 1):
        return y.astype(np.float64).mean(axis=-2).astype(np.float32)
    s = _pairwise_sum(y, axis=3)
    return (s * np.float32(1.0 / n)).astype(np.float32)


def block_routing_scores(q_blocks, k_blocks) -> np.ndarray:
    """block_sparse_attention.py:107-112: q_blocks @ k_blocks^T, fp32, in the engine's exact
    order (one fma chain over d = 0..D-1 per score, ``oracle/bsa_oracle.c``)."""
    qb = np.ascontiguousarray(to_f32(q_blocks))
    kb = np.ascontiguousarray(to_f32(k_blocks))
    lead = qb.shape[:-2]
    nq, D = qb.shape[-2:]
    nk = kb.shape[-2]
    BH = int(np.prod(lead)) if lead else 1
    out = np.empty((BH, nq, nk), dtype=np.float32)
    lib = _load_lib()
    lib.oracle_scores(
        qb.ctypes.data_as(ctypes.c_void_p), kb.ctypes.data_as(ctypes.c_void_p),
        ctypes.c_int(BH), ctypes.c_int(nq), ctypes.c_int(nk), ctypes.c_int(D),
        out.ctypes.data_as(ctypes.c_void_p))
    return out.reshape(*lead, nq, nk)


def num_selected_blocks(num_kv_blocks: int, sparsity: float) -> int:
    """block_sparse_attention.py:127 -- floor rule, clamped to >= 1."""
    return max(1, int((1.0 - sparsity) * num_kv_blocks))


def topk_block_indices(score, sparsity: float = 0.9375, topk: Optional[int] = None):
    """block_sparse_attention.py:115-134 with an explicit selection rule: the k largest
    scores per row, ties broken by smaller block index; returned sorted ascending by block
    index as int32.  ``topk`` overrides the floor rule (the benchmark configs use ceil)."""
    score = np.ascontiguousarray(to_f32(score))
    nk = score.shape[-1]
    k = num_selected_blocks(nk, sparsity) if topk is None else int(topk)
    if not 1 <= k <= nk:
        raise ValueError(f"topk={k} out of range for {nk} KV blocks")
    lead = score.shape[:-1]
    rows = int(np.prod(lead)) if lead else 1
    out = np.empty((rows, k), dtype=np.int32)
    _load_lib().oracle_topk(
        score.ctypes.data_as(ctypes.c_void_p), ctypes.c_int(rows), ctypes.c_int(nk), ctypes.c_int(k),
        out.ctypes.data_as(ctypes.c_void_p))
    return out.reshape(*lead, k), k


def topk_block_indices_numpy(score, k: int) -> np.ndarray:
    """Same rule as ``topk_block_indices`` in plain numpy (stable sort of -score); used to
    cross-check the C restatement."""
    s = to_f32(score)
    s = np.where(s == 0, np.float32(0), s)  # -0.0 and +0.0 are one score
    order = np.argsort(-s, axis=-1, kind="stable")[..., :k]
    return np.sort(order, axis=-1).astype(np.int32)


def build_token_block_indices(shape, chunk_thw=(4, 4, 4)) -> np.ndarray:
    """block_sparse_attention.py:137-159."""
    T, H_, W = shape
    cT, cH, cW = chunk_thw
    Bh, Bw = H_ // cH, W // cW
    s = np.arange(T * H_ * W, dtype=np.int64)
    t = s // (H_ * W)
    hw = s % (H_ * W)
    h = hw // W
    w = hw % W
    return ((t // cT) * (Bh * Bw) + (h // cH) * Bw + (w // cW)).astype(np.int32)


def build_token_pair_mask(block_indices, token_block_index, num_kv_blocks: int) -> np.ndarray:
    """block_sparse_attention.py:162-198: [B,H,nq,k] routing -> [B,H,S,S] bool."""
    bi = np.asarray(block_indices)
    k_range = np.arange(num_kv_blocks, dtype=np.int32)
    one_hot = bi[..., None] == k_range
    block_pair = one_hot.any(axis=-2)  # [B,H,nq,nk]
    tbi = np.asarray(token_block_index)
    # rows/cols past the routed block count (only in hand-built tests with fewer q blocks than
    # tokens) are clipped; with nq == nk every index is in range
    rows = np.take(block_pair, tbi, axis=-2, mode="clip")
    return np.take(rows, tbi, axis=-1, mode="clip")


def _dense_masked_attention(q, k, v, mask, sm_scale) -> np.ndarray:
    """Dense SDPA with the reference's additive 0/-1e9 mask (block_sparse_attention.py:243-250),
    computed in float64."""
    q = q.astype(np.float64)
    k = k.astype(np.float64)
    v = v.astype(np.float64)
    s = np.einsum("bhqd,bhkd->bhqk", q, k) * sm_scale
    if mask is not None:
        s = s + np.where(mask, 0.0, -1e9)
    s = s - s.max(axis=-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(axis=-1, keepdims=True)
    return np.einsum("bhqk,bhkd->bhqd", p, v)


def bsa_attention(q, k, v, shape, sparsity=0.9375, chunk_thw=(4, 4, 4), sm_scale=None,
                  topk: Optional[int] = None):
    """block_sparse_attention.py:201-250 (Tier A): pool -> score -> top-k -> token-pair mask ->
    dense masked SDPA.  Returns (out float64 [B,H,S,D], block_indices int32).  The S^2 mask
    makes this usable only for small S."""
    qf, kf, vf = to_f32(q), to_f32(k), to_f32(v)
    D = qf.shape[-1]
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    qb = mean_pool_blocks_3d(qf, shape, chunk_thw)
    kb = mean_pool_blocks_3d(kf, shape, chunk_thw)
    score = block_routing_scores(qb, kb)
    idx, _ = topk_block_indices(score, sparsity, topk)
    tbi = build_token_block_indices(shape, chunk_thw)
    mask = build_token_pair_mask(idx, tbi, score.shape[-1])
    return _dense_masked_attention(qf, kf, vf, mask, sm_scale), idx


def bsa_sparse_attention(q, k, v, block_indices, shape, chunk_thw=(4, 4, 4), sm_scale=None,
                         heads: Optional[Sequence[int]] = None, qblocks: Optional[Sequence[int]] = None,
                         dtype=np.float64) -> np.ndarray:
    """Kernel-level semantics (block_sparse_attention_metal.py:75-164, :224-295): for every
    q-block, softmax over exactly the tokens of its selected KV blocks, then weighted sum of
    V; ``out = o / l``.  Identical to Tier A's masked SDPA because the -1e9 additive mask
    zeroes every unselected weight.  Gathers per q-block, so it runs at any S for a subset
    of heads / q-blocks.  Returns [B, len(heads), len(qblocks)*n, D] in block-major row
    order when subsets are given, else [B,H,S,D] t-major."""
    qf, kf, vf = to_f32(q), to_f32(k), to_f32(v)
    B, H, S, D = qf.shape
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    idx = np.asarray(block_indices)
    qbm = to_block_major(qf, shape, chunk_thw)
    kbm = to_block_major(kf, shape, chunk_thw)
    vbm = to_block_major(vf, shape, chunk_thw)
    nb, n = qbm.shape[2], qbm.shape[3]
    hs = list(range(H)) if heads is None else list(heads)
    qs = list(range(nb)) if qblocks is None else list(qblocks)
    out = np.zeros((B, len(hs), len(qs), n, D), dtype=dtype)
    for b in range(B):
        for hi, h in enumerate(hs):
            for qi, i in enumerate(qs):
                sel = idx[b, h, i]
                kk = kbm[b, h, sel].reshape(-1, D).astype(dtype)
                vv = vbm[b, h, sel].reshape(-1, D).astype(dtype)
                s = (qbm[b, h, i].astype(dtype) @ kk.T) * dtype(sm_scale)
                s = s - s.max(axis=-1, keepdims=True)
                p = np.exp(s)
                l = p.sum(axis=-1, keepdims=True)
                out[b, hi, qi] = (p @ vv) / l
    if heads is None and qblocks is None:
        return from_block_major(out, shape, chunk_thw)
    return out.reshape(B, len(hs), len(qs) * n, D)


# ----------------------------------------------------------------------------- 3D RoPE
def rope_axis_dims(head_dim: int):
    """rope_3d.py:60-62: (dim_t, dim_h, dim_w)."""
    d6 = head_dim // 6
    return head_dim - 4 * d6, 2 * d6, 2 * d6


def rope_axis_tables(grid, head_dim: int, base: float = 10000.0):
    """Per-axis angle tables of rope_3d.py:53-105, fp32.  Returns
    [(cos_t, sin_t), (cos_h, sin_h), (cos_w, sin_w)] with shapes [T, dim_t/2], [H, dim_h/2],
    [W, dim_w/2]: one entry per rotated pair (the reference repeats each frequency twice,
    :91-93, so both elements of a pair share one angle)."""
    tabs = []
    for n, dim in zip(grid, rope_axis_dims(head_dim)):
        idx = np.arange(0, dim, 2, dtype=np.float32)[: dim // 2]
        freqs = (np.float32(1.0) / (np.float32(base) ** (idx / np.float32(dim)))).astype(np.float32)
        pos = np.arange(0, n, dtype=np.float32)
        ang = (pos[:, None] * freqs[None, :]).astype(np.float32)
        tabs.append((np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)))
    return tabs


def rope_full_tables(grid, head_dim: int, base: float = 10000.0):
    """[S, D] cos and sin tables in the reference's layout (rope_3d.py:91-105)."""
    T, H_, W = grid
    (ct, st), (ch, sh), (cw, sw) = rope_axis_tables(grid, head_dim, base)
    rep = lambda a: np.repeat(a, 2, axis=-1)
    dt, dh, dw = rope_axis_dims(head_dim)
    cos = np.concatenate([
        np.broadcast_to(rep(ct)[:, None, None, :], (T, H_, W, dt)),
        np.broadcast_to(rep(ch)[None, :, None, :], (T, H_, W, dh)),
        np.broadcast_to(rep(cw)[None, None, :, :], (T, H_, W, dw))], axis=-1).reshape(T * H_ * W, head_dim)
    sin = np.concatenate([
        np.broadcast_to(rep(st)[:, None, None, :], (T, H_, W, dt)),
        np.broadcast_to(rep(sh)[None, :, None, :], (T, H_, W, dh)),
        np.broadcast_to(rep(sw)[None, None, :, :], (T, H_, W, dw))], axis=-1).reshape(T * H_ * W, head_dim)
    return cos.astype(np.float32), sin.astype(np.float32)


def rotate_half(x: np.ndarray) -> np.ndarray:
    """rope_3d.py:23-34: pairs (x0, x1) -> (-x1, x0)."""
    y = x.reshape(*x.shape[:-1], x.shape[-1] // 2, 2)
    return np.stack([-y[..., 1], y[..., 0]], axis=-1).reshape(x.shape)


def rms_norm_fp32(x, weight, eps: float, out_dtype: str) -> np.ndarray:
    """RMSNorm_FP32 (longcat_video/models/blocks.py:55-73): ``(x * rsqrt(mean(x^2) + eps)).astype(dtype)
    * weight`` with the weight in the input dtype; the norm here in fp64 (the engine's fp32 rsqrt is
    within a few fp32 ulps of it), each product rounded to fp32 and then to the input dtype."""
    xf = to_f32(x).astype(np.float64)
    r = 1.0 / np.sqrt(np.mean(xf * xf, axis=-1, keepdims=True) + eps)
    n = round_to((xf * r).astype(np.float32), out_dtype)
    w = round_to(to_f32(weight), out_dtype)
    return round_to((n * w).astype(np.float32), out_dtype)


def apply_rope(x, cos: np.ndarray, sin: np.ndarray, out_dtype: str) -> np.ndarray:
    """rope_3d.py:120-128: fp32 ``x*cos + rotate_half(x)*sin`` (each product and the sum
    rounded to fp32, no fused multiply-add), cast back to the input dtype."""
    xf = to_f32(x)
    a = (xf * cos).astype(np.float32)
    b = (rotate_half(xf) * sin).astype(np.float32)
    return round_to((a + b).astype(np.float32), out_dtype)


# ----------------------------------------------------------------------------- C restatement
def _load_lib():
    global _lib
    if _lib is None:
        src = os.path.join(_HERE, "bsa_oracle.c")
        if not os.path.exists(_LIB_PATH) or (os.path.exists(src) and
                                             os.path.getmtime(src) > os.path.getmtime(_LIB_PATH)):
            build_oracle_lib()
        lib = ctypes.CDLL(_LIB_PATH)
        lib.oracle_scores.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                      ctypes.c_int, ctypes.c_void_p]
        lib.oracle_topk.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
        lib.oracle_pool.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                    ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                    ctypes.c_void_p]
        _lib = lib
    return _lib


def build_oracle_lib() -> str:
    """Compile oracle/bsa_oracle.c into oracle/_build/libbsa_oracle.so (gcc, no FMA contraction)."""
    import subprocess

    os.makedirs(os.path.dirname(_LIB_PATH), exist_ok=True)
    src = os.path.join(_HERE, "bsa_oracle.c")
    subprocess.check_call(["gcc", "-O2", "-shared", "-fPIC", "-ffp-contract=off", "-fno-fast-math", "-o",
                           _LIB_PATH, src, "-lm"])
    return _LIB_PATH


def oracle_pool_c(x: np.ndarray, shape, chunk_thw) -> np.ndarray:
    """C restatement of the pooling order (cross-check for ``mean_pool_blocks_3d``)."""
    x = np.ascontiguousarray(to_f32(x))
    B, H, S, D = x.shape
    T, H_, W = shape
    cT, cH, cW = chunk_thw
    nb = S // (cT * cH * cW)
    out = np.empty((B, H, nb, D), dtype=np.float32)
    _load_lib().oracle_pool(x.ctypes.data_as(ctypes.c_void_p), B * H, S, D, T, H_, W, cT, cH, cW,
                            out.ctypes.data_as(ctypes.c_void_p))
    return out
