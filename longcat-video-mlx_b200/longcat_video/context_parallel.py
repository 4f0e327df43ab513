"""Ulysses-style sequence <-> head re-sharding around the BSA call (one process per GPU).

The DiT runs sequence-sharded ([B, H, S/P, D] per rank); BSA needs whole sequences because a
query block may select any KV block.  Heads are independent, so one all-to-all turns the
sequence shard of all heads into all tokens of H/P heads, BSA runs locally on those heads, and a
second all-to-all returns the output to sequence shards.  The upstream PyTorch model did this
with ``ulysses_wrapper`` / ``context_parallel_util``, which the MLX port dropped
(rope_3d.py:14; stubbed in tests/parity/test_dit_block_parity.py:88-112).

Plumbing is ``torch.distributed.all_to_all_single`` (NCCL over NVLink on GPUs, gloo on CPU for
tests).  Q, K and V travel in one collective.  Pre-RoPE Q/K travel and RoPE is applied after the
exchange, because the rotation needs each token's global position.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.distributed as dist

from .models.block_sparse_attention import bsa_attention

__all__ = ["seq_to_heads", "heads_to_seq", "ulysses_bsa_attention"]


def _world(group) -> int:
    return dist.get_world_size(group) if dist.is_initialized() else 1


def seq_to_heads(x: torch.Tensor, group=None) -> torch.Tensor:
    """[..., B, H, S/P, D] sequence shard (rank r holds tokens r*S/P .. (r+1)*S/P - 1 of every
    head) -> [..., B, H/P, S, D] head shard (rank r holds heads r*H/P .. (r+1)*H/P - 1)."""
    P = _world(group)
    if P == 1:
        return x
    *lead, B, H, Sl, D = x.shape
    if H % P:
        raise ValueError(f"{H} heads do not split over {P} ranks")
    L = len(lead)
    y = x.reshape(*lead, B, P, H // P, Sl, D)
    # bring the destination-rank axis to the front: [P, lead..., B, H/P, Sl, D]
    y = y.movedim(L + 1, 0).contiguous()
    recv = torch.empty_like(y)
    dist.all_to_all_single(recv, y, group=group)
    # recv[p] = rank p's sequence shard of my heads -> concatenate along the sequence axis
    recv = recv.movedim(0, L + 2)  # [lead..., B, H/P, P, Sl, D]
    return recv.reshape(*lead, B, H // P, P * Sl, D)


def heads_to_seq(o: torch.Tensor, group=None) -> torch.Tensor:
    """Inverse of ``seq_to_heads``: [..., B, H/P, S, D] -> [..., B, H, S/P, D]."""
    P = _world(group)
    if P == 1:
        return o
    *lead, B, Hl, S, D = o.shape
    if S % P:
        raise ValueError(f"S={S} does not split over {P} ranks")
    L = len(lead)
    y = o.reshape(*lead, B, Hl, P, S // P, D)
    y = y.movedim(L + 2, 0).contiguous()  # [P, lead..., B, Hl, Sl, D]
    recv = torch.empty_like(y)
    dist.all_to_all_single(recv, y, group=group)
    recv = recv.movedim(0, L + 1)  # [lead..., B, P, Hl, Sl, D]
    return recv.reshape(*lead, B, P * Hl, S // P, D)


def _seq_to_heads_async(x: torch.Tensor, P: int, group):
    """Start seq_to_heads of [3, B, Hg, S/P, D]; returns (work, finish) where finish() -> [3, B, Hg/P, S, D]."""
    L, (B, H, Sl, D) = 1, x.shape[1:]
    y = x.reshape(3, B, P, H // P, Sl, D).movedim(L + 1, 0).contiguous()
    recv = torch.empty_like(y)
    work = dist.all_to_all_single(recv, y, group=group, async_op=True)

    def finish():
        return recv.movedim(0, L + 2).reshape(3, B, H // P, P * Sl, D)

    return work, finish


def _heads_to_seq_async(o: torch.Tensor, P: int, group):
    """Start heads_to_seq of [B, Hg/P, S, D]; returns (work, finish) where finish() -> [B, Hg, S/P, D]."""
    B, Hl, S, D = o.shape
    y = o.reshape(B, Hl, P, S // P, D).movedim(2, 0).contiguous()
    recv = torch.empty_like(y)
    work = dist.all_to_all_single(recv, y, group=group, async_op=True)

    def finish():
        return recv.movedim(0, 1).reshape(B, P * Hl, S // P, D)

    return work, finish


def _head_groups(H: int, P: int, groups: Optional[int]) -> int:
    if groups is None:
        groups = min(4, H // P) if H >= P else 1
    groups = max(1, int(groups))
    while groups > 1 and (H % groups or (H // groups) % P):
        groups -= 1
    return groups


def ulysses_bsa_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, shape: Tuple[int, int, int],
                          sparsity: float = 0.9375, chunk_thw: Tuple[int, int, int] = (4, 4, 4),
                          sm_scale: Optional[float] = None, *, topk: Optional[int] = None, rope=None,
                          group=None, head_groups: Optional[int] = None) -> torch.Tensor:
    """Sequence-sharded BSA: q, k, v are this rank's [B, H, S/P, D] shards; returns the output
    shard [B, H, S/P, D].  ``shape`` is the full latent (T, H, W) of the whole sequence.

    The heads are processed in ``head_groups`` groups (default: up to 4, each a multiple of P
    heads) so the exchanges overlap the compute: the all-to-all that brings in group g+1 and the
    one that returns group g-1 run on the communicator's stream while group g computes.  Every
    rank issues the same collectives in the same order.
    """
    P = _world(group)
    if P == 1:
        return bsa_attention(q, k, v, shape, sparsity, chunk_thw, sm_scale, topk=topk, rope=rope)
    B, H, Sl, D = q.shape
    if H % P:
        raise ValueError(f"{H} heads do not split over {P} ranks")
    G = _head_groups(H, P, head_groups)
    Hg = H // G
    sl = [slice(g * Hg, (g + 1) * Hg) for g in range(G)]
    out = torch.empty_like(q)
    pending_in = _seq_to_heads_async(torch.stack((q[:, sl[0]], k[:, sl[0]], v[:, sl[0]])), P, group)
    pending_out = []
    for g in range(G):
        work, finish = pending_in
        # enqueue the next group's exchange before this group's compute so it does not wait on it
        if g + 1 < G:
            pending_in = _seq_to_heads_async(torch.stack((q[:, sl[g + 1]], k[:, sl[g + 1]], v[:, sl[g + 1]])), P,
                                             group)
        work.wait()
        qkv_h = finish()
        o = bsa_attention(qkv_h[0], qkv_h[1], qkv_h[2], shape, sparsity, chunk_thw, sm_scale, topk=topk, rope=rope)
        pending_out.append((g, _heads_to_seq_async(o, P, group)))
    for g, (work, finish) in pending_out:
        work.wait()
        out[:, sl[g]] = finish()
    return out
