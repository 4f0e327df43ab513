"""Block Sparse Attention (BSA) on B200 -- the reference's Tier A API over the CUDA engine.

Same public surface as xocialize/longcat-video-mlx ``longcat_video/models/block_sparse_attention.py``
(``__all__`` at :57-64): a caller that imported the MLX module can import this one instead.
Every function runs on the GPU through the engine's C ABI; there is no CPU path.

Differences from the MLX Tier A, all deliberate:
  * routing is computed in fp32 (pooled means and block scores), whatever the input dtype;
    MLX computes it in the input dtype (:104, :112), which ties massively in bf16/fp16;
  * top-k ties are broken by the smaller block id and every index row is sorted ascending
    (``mx.argpartition`` leaves both unspecified, :130-134);
  * ``bsa_attention`` never materialises the S x S mask (:236-247): the sparse kernel walks the
    selected KV blocks directly, which is the same function (the -1e9 additive mask zeroes
    exactly the unselected weights);
  * keyword-only extras: ``topk`` overrides the floor rule of :127 (the benchmark configs use
    ceil), ``rope`` fuses the 3-D RoPE of rope_3d.py into the routing kernel, and
    ``return_indices`` also returns the routing.
"""

from __future__ import annotations

import math
from typing import Optional, Tuple

import torch

from .. import _native

__all__ = [
    "mean_pool_blocks_3d",
    "block_routing_scores",
    "topk_block_indices",
    "build_token_block_indices",
    "build_token_pair_mask",
    "bsa_attention",
    "num_selected_blocks",
]


def num_selected_blocks(num_kv_blocks: int, sparsity: float) -> int:
    """block_sparse_attention.py:127 -- ``max(1, int((1 - sparsity) * num_kv_blocks))``."""
    return max(1, int((1.0 - sparsity) * num_kv_blocks))


def mean_pool_blocks_3d(x: torch.Tensor, shape: Tuple[int, int, int],
                        chunk_thw: Tuple[int, int, int] = (4, 4, 4)) -> torch.Tensor:
    """block_sparse_attention.py:67-104.  [B, H, S, D] -> fp32 [B, H, num_blocks, D], blocks in
    (bt, bh, bw) order.  Raises ``ValueError`` for shapes that are not multiples of chunk_thw."""
    pooled, _ = _native.mean_pool(x, shape, chunk_thw)
    return pooled


def block_routing_scores(q_blocks: torch.Tensor, k_blocks: torch.Tensor) -> torch.Tensor:
    """block_sparse_attention.py:107-112: ``q_blocks @ k_blocks^T`` in fp32,
    [B, H, nq, nk]."""
    return _native.block_scores(q_blocks, k_blocks)


def topk_block_indices(score: torch.Tensor, sparsity: float,
                       topk: Optional[int] = None) -> Tuple[torch.Tensor, int]:
    """block_sparse_attention.py:115-134.  Returns ([B, H, nq, k] int32 ascending block ids, k)."""
    nk = int(score.shape[-1])
    k = num_selected_blocks(nk, sparsity) if topk is None else int(topk)
    return _native.topk_from_scores(score, k), k


def build_token_block_indices(shape: Tuple[int, int, int], chunk_thw: Tuple[int, int, int] = (4, 4, 4),
                              device=None) -> torch.Tensor:
    """block_sparse_attention.py:137-159: token (t-major) -> block id ``bt*Bh*Bw + bh*Bw + bw``."""
    T, H_, W = shape
    cT, cH, cW = chunk_thw
    Bh, Bw = H_ // cH, W // cW
    s = torch.arange(T * H_ * W, dtype=torch.int64, device=device)
    t = s // (H_ * W)
    hw = s % (H_ * W)
    h = hw // W
    w = hw % W
    return ((t // cT) * (Bh * Bw) + (h // cH) * Bw + (w // cW)).to(torch.int32)


def build_token_pair_mask(block_indices: torch.Tensor, token_block_index: torch.Tensor,
                          num_kv_blocks: int) -> torch.Tensor:
    """block_sparse_attention.py:162-198: [B, H, S, S] bool.  Provided for API completeness
    (the engine never builds it: S^2 elements are infeasible at 720p)."""
    bi = block_indices.long()
    B, H, nq, _ = bi.shape
    block_pair = torch.zeros((B, H, nq, num_kv_blocks), dtype=torch.bool, device=bi.device)
    block_pair.scatter_(-1, bi, True)
    tbi = token_block_index.long().to(bi.device)
    # hand-built routings may have fewer q blocks than token blocks: clamp those rows, as
    # they are never consulted (with nq == nk every index is in range)
    rows = block_pair[..., tbi.clamp(max=nq - 1), :]
    return rows[..., tbi.clamp(max=num_kv_blocks - 1)]


def bsa_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, shape: Tuple[int, int, int],
                  sparsity: float = 0.9375, chunk_thw: Tuple[int, int, int] = (4, 4, 4),
                  sm_scale: Optional[float] = None, *, topk: Optional[int] = None, rope=None,
                  return_indices: bool = False):
    """block_sparse_attention.py:201-250 (Tier A entry) on the CUDA engine.

    q, k, v: [B, H, S, D] (bf16 or fp16 CUDA tensors, d contiguous), S = T*H*W, 64-token blocks.
    rope: optional ``RotaryPositionalEmbedding`` tables from ``rope_3d.rope_tables(...)``; when
    given, q and k are pre-RoPE and the rotation is fused into the routing kernel.
    Returns [B, H, S, D] (and the [B, H, nb, k] routing when ``return_indices``).
    """
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(int(q.shape[-1]))
    S = int(q.shape[-2])
    _native._geometry(S, shape, chunk_thw)
    nb = S // (chunk_thw[0] * chunk_thw[1] * chunk_thw[2])
    k_sel = num_selected_blocks(nb, sparsity) if topk is None else int(topk)
    rope_arg = rope.native_args() if rope is not None else None
    out, idx = _native.forward(q, k, v, shape, chunk_thw, k_sel, sm_scale, rope=rope_arg)
    return (out, idx) if return_indices else out
