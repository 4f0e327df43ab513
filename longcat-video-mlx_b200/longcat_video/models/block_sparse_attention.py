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
    ceil), ``rope`` fuses the 3-D RoPE of rope_3d.py into the routing kernel,
    ``return_indices`` also returns the routing, and ``sm_reserve`` leaves SMs free for a
    concurrent exchange;
  * host (CPU) tensors are streamed through the current CUDA device in head groups.
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
                  return_indices: bool = False, sm_reserve: int = 0, out: Optional[torch.Tensor] = None,
                  qk_norm=None):
    """block_sparse_attention.py:201-250 (Tier A entry) on the CUDA engine.

    q, k, v: [B, H, S, D] (bf16 or fp16, d contiguous), S = T*H*W, 64-token blocks.  CUDA tensors
    run in place on their device.  Host (CPU) tensors are streamed through the current CUDA device
    in head groups -- the copy in of group i+1 and the copy out of group i-1 overlap the compute of
    group i -- and the result comes back as a host tensor (pinned), complete on return.
    rope: optional ``RotaryPositionalEmbedding`` tables from ``rope_3d.rope_tables(...)``; when
    given, q and k are pre-RoPE and the rotation is fused into the routing kernel.
    sm_reserve: SMs kept free of the persistent attention kernel, for kernels of a concurrent
    exchange on other streams (device tensors only).
    out: optional preallocated [B, H, S, D] output on q's device (device tensors only).
    qk_norm: optional ``(q_weight, k_weight, eps)`` (device tensors only): q and k are the raw projections
    and their RMSNorm_FP32 (blocks.py:55-73) runs fused with the RoPE and the pooling.
    Returns [B, H, S, D] (and the [B, H, nb, k] routing when ``return_indices``).
    """
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(int(q.shape[-1]))
    S = int(q.shape[-2])
    _native._geometry(S, shape, chunk_thw)
    nb = S // (chunk_thw[0] * chunk_thw[1] * chunk_thw[2])
    k_sel = num_selected_blocks(nb, sparsity) if topk is None else int(topk)
    rope_arg = rope.native_args() if rope is not None else None
    if not q.is_cuda and not k.is_cuda and not v.is_cuda:
        if out is not None or qk_norm is not None:
            raise ValueError("out= and qk_norm= are for device tensors")
        out, idx = _forward_host_streamed(q, k, v, shape, chunk_thw, k_sel, sm_scale, rope_arg, return_indices)
    else:
        out, idx = _native.forward(q, k, v, shape, chunk_thw, k_sel, sm_scale, rope=rope_arg, sm_reserve=sm_reserve,
                                   out=out, qk_norm=qk_norm)
    return (out, idx) if return_indices else out


def _forward_host_streamed(q, k, v, shape, chunk_thw, k_sel, sm_scale, rope_arg, want_indices,
                           heads_per_group: Optional[int] = None):
    """BSA call on host tensors: three-stream pipeline over head groups on the current CUDA device.

    Heads are independent (routing and attention are per (b, h)), so the call splits into head
    groups.  Group i is copied in on a copy-in stream, computed on the current stream, and copied
    out on a copy-out stream; two device slots alternate, so the host-to-device copy of group i+1
    and the device-to-host copy of group i-1 run while group i computes.
    """
    if q.shape != k.shape or q.shape != v.shape:
        raise ValueError("q, k, v must have the same shape [B, H, S, D]")
    if q.dtype != k.dtype or q.dtype != v.dtype:
        raise ValueError("q, k, v must share one dtype")
    if not torch.cuda.is_available():
        raise _native.BSAError("bsa_attention on host tensors needs a CUDA device (there is no CPU path)")
    dev = torch.device("cuda", torch.cuda.current_device())
    B, H, S, D = (int(x) for x in q.shape)
    nb = S // (chunk_thw[0] * chunk_thw[1] * chunk_thw[2])
    # one head per group: the copies dominate (PCIe), so the smallest first copy-in and last
    # copy-out leave the least exposed; a head is still ~1,350 attention units of work at 720p
    G = max(1, min(H, int(heads_per_group or 1)))
    groups = [(h0, min(h0 + G, H)) for h0 in range(0, H, G)]
    out = torch.empty((B, H, S, D), dtype=q.dtype, pin_memory=True)
    idx_host = torch.empty((B, H, nb, k_sel), dtype=torch.int32, pin_memory=True) if want_indices else None
    compute = torch.cuda.current_stream(dev)
    s_in = torch.cuda.Stream(dev)
    s_out = torch.cuda.Stream(dev)
    nslot = min(2, len(groups))
    # flat slot buffers; a group of n heads uses a contiguous [B, n, ...] view of the front
    qd, kd, vd, od = ([torch.empty((B * G * S * D,), device=dev, dtype=q.dtype) for _ in range(nslot)]
                      for _ in range(4))
    idd = [torch.empty((B * G * nb * k_sel,), device=dev, dtype=torch.int32) for _ in range(nslot)]

    def view(buf, n, *rest):
        m = B * n
        for r in rest:
            m *= r
        return buf[:m].view(B, n, *rest)

    nbytes = int(_native.lib().bsa_forward_scratch_bytes(B, G, S, D, *chunk_thw))
    scratch = torch.empty((max(nbytes, 16),), device=dev, dtype=torch.uint8)
    ev_in = [torch.cuda.Event() for _ in groups]
    ev_done = [torch.cuda.Event() for _ in groups]
    ev_out = [torch.cuda.Event() for _ in groups]
    s_in.wait_stream(compute)  # device buffers were allocated on the compute stream
    for i, (h0, h1) in enumerate(groups):
        n, sl = h1 - h0, i % nslot
        with torch.cuda.stream(s_in):
            if i >= nslot:
                s_in.wait_event(ev_done[i - nslot])  # slot inputs free once group i-2 has computed
            for dst, src in ((qd[sl], q), (kd[sl], k), (vd[sl], v)):
                view(dst, n, S, D).copy_(src[:, h0:h1], non_blocking=True)
            ev_in[i].record(s_in)
        compute.wait_event(ev_in[i])
        if i >= nslot:
            compute.wait_event(ev_out[i - nslot])  # slot output free once group i-2 is copied out
        _native.forward(view(qd[sl], n, S, D), view(kd[sl], n, S, D), view(vd[sl], n, S, D), shape, chunk_thw,
                        k_sel, sm_scale, rope=rope_arg, out=view(od[sl], n, S, D),
                        block_indices=view(idd[sl], n, nb, k_sel), scratch=scratch)
        ev_done[i].record(compute)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_done[i])
            out[:, h0:h1].copy_(view(od[sl], n, S, D), non_blocking=True)
            if idx_host is not None:
                idx_host[:, h0:h1].copy_(view(idd[sl], n, nb, k_sel), non_blocking=True)
            ev_out[i].record(s_out)
    compute.wait_stream(s_out)
    compute.wait_stream(s_in)
    ev_out[-1].synchronize()
    return out, idx_host
