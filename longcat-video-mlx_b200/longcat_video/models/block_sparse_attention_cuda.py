"""Kernel-level BSA entry on B200: attention over pre-computed block indices.

Drop-in for the reference's Tier B wrappers (xocialize/longcat-video-mlx
``longcat_video/models/block_sparse_attention_metal.py``): ``bsa_attention_metal``
(:224-295), ``_v2`` (:484-548), ``_v3`` (:729-810), ``_v4`` (:985-1046) and
``prewarm_metal_kernel`` (:298-333) all keep their signatures and route to the single sm_100a
kernel (``bsa_attention_cuda``).  There is no block-major permute: the kernel's 5-D TMA boxes
read 4x4x4 voxels (or contiguous 64-token blocks) in place.

Contract, as in the reference: ``shape`` is required (``ValueError`` otherwise, :248-252); the
block size ``prod(chunk_thw)`` must be 64 and divide S (:257-262); ``block_indices`` is
[B, H, num_q_blocks, top_k] int32; the softmax scale defaults to ``1/sqrt(D)`` (:114).
Supported: fp16 / bf16, D a multiple of 8 up to 128.
"""

from __future__ import annotations

import math
from typing import Optional, Tuple

import torch

from .. import _native

__all__ = [
    "bsa_attention_cuda",
    "bsa_attention_metal",
    "bsa_attention_metal_v2",
    "bsa_attention_metal_v3",
    "bsa_attention_metal_v4",
    "prewarm_cuda_kernel",
    "prewarm_metal_kernel",
]


def bsa_attention_cuda(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, block_indices: torch.Tensor,
                       chunk_thw: Tuple[int, int, int] = (4, 4, 4), shape: Optional[Tuple[int, int, int]] = None,
                       sm_scale: Optional[float] = None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Sparse attention of every query block over its selected KV blocks (fp32 online softmax,
    ``out = o / l``), [B, H, S, D] in the input dtype and token order."""
    if shape is None:
        raise ValueError(
            "shape=(T_lat, H_lat, W_lat) is required for Tier B BSA "
            "(needed to locate the tokens of each block)")
    B, H, S, D = q.shape
    BS = chunk_thw[0] * chunk_thw[1] * chunk_thw[2]
    if S % BS != 0:
        raise ValueError(f"S={S} must be a multiple of block_size={BS}.")
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    return _native.attention_indices(q, k, v, block_indices, shape, chunk_thw, sm_scale, out=out)


def bsa_attention_metal(q, k, v, block_indices, chunk_thw=(4, 4, 4), shape=None):
    """Name of block_sparse_attention_metal.py:224 (Phase 1), served by the sm_100a kernel."""
    return bsa_attention_cuda(q, k, v, block_indices, chunk_thw=chunk_thw, shape=shape)


def bsa_attention_metal_v2(q, k, v, block_indices, chunk_thw=(4, 4, 4), shape=None):
    """Name of block_sparse_attention_metal.py:484 (Phase 2), served by the sm_100a kernel."""
    return bsa_attention_cuda(q, k, v, block_indices, chunk_thw=chunk_thw, shape=shape)


def bsa_attention_metal_v3(q, k, v, block_indices, chunk_thw=(4, 4, 4), shape=None):
    """Name of block_sparse_attention_metal.py:729 (Phase 3), served by the sm_100a kernel."""
    return bsa_attention_cuda(q, k, v, block_indices, chunk_thw=chunk_thw, shape=shape)


def bsa_attention_metal_v4(q, k, v, block_indices, chunk_thw=(4, 4, 4), shape=None):
    """Name of block_sparse_attention_metal.py:985 (Phase 4), served by the sm_100a kernel."""
    return bsa_attention_cuda(q, k, v, block_indices, chunk_thw=chunk_thw, shape=shape)


def prewarm_cuda_kernel(head_dim: int = 128, block_size: int = 64, dtype: torch.dtype = torch.bfloat16,
                        device: str = "cuda") -> None:
    """Load the engine and run one tiny full BSA call (pooling, routing, attention) so the first real
    call pays no one-time cost (library load, shared-memory opt-ins of every kernel, the tensor-map
    entry point lookup).  block_sparse_attention_metal.py:298-333 does the same for the Metal JIT."""
    if block_size != 64:
        raise ValueError("the sm_100a kernel uses 64-token blocks")
    from .block_sparse_attention import bsa_attention

    g = torch.Generator(device="cpu").manual_seed(0)
    q = torch.randn((1, 1, 128, head_dim), generator=g).to(dtype).to(device)
    bsa_attention(q, q, q, (1, 1, 128), chunk_thw=(1, 1, 64), topk=1)
    torch.cuda.synchronize()


def prewarm_metal_kernel(head_dim: int = 128, block_size: int = 64, top_k_values=(6, 64, 128),
                         dtype: torch.dtype = torch.float16) -> None:
    """Signature of block_sparse_attention_metal.py:298; prewarms the sm_100a kernel."""
    del top_k_values
    prewarm_cuda_kernel(head_dim=head_dim, block_size=block_size, dtype=dtype)
