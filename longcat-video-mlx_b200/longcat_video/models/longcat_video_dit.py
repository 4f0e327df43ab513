"""BSA switch of the LongCat-Video DiT (xocialize/longcat-video-mlx
``longcat_video/models/longcat_video_dit.py:193-262``).

Only the part of the DiT that the BSA path touches is built here: the per-block attention
modules and the ``from_config`` / ``enable_bsa`` / ``disable_bsa`` plumbing that flips them.
The rest of the 48-block transformer (AdaLN, FFN, embedders, final layer) is outside this
engine's scope; ``LongCatSingleStreamBlock`` therefore carries only ``attn``.
"""

from __future__ import annotations

from typing import List, Optional, Tuple

import torch

from .attention import BSA_BACKENDS, Attention


class LongCatSingleStreamBlock(torch.nn.Module):
    """Holds the block's self-attention (longcat_video_dit.py:38-139 keeps it at ``.attn``)."""

    def __init__(self, hidden_size: int, num_heads: int):
        super().__init__()
        self.attn = Attention(hidden_size, num_heads)


class LongCatVideoTransformer3DModel(torch.nn.Module):
    def __init__(self, hidden_size: int = 4096, depth: int = 48, num_heads: int = 32, **_unused):
        super().__init__()
        self.depth = depth
        self.blocks = torch.nn.ModuleList(
            [LongCatSingleStreamBlock(hidden_size=hidden_size, num_heads=num_heads) for _ in range(depth)])
        self._bsa_sparsity: float = 0.9375
        self._bsa_chunk_thw: Tuple[int, int, int] = (4, 4, 4)
        self._bsa_topk: Optional[int] = None

    @classmethod
    def from_config(cls, config: dict) -> "LongCatVideoTransformer3DModel":
        """longcat_video_dit.py:193-218: ``bsa_params.sparsity`` / ``chunk_3d_shape_q`` are kept
        on the instance; ``enable_bsa: true`` turns BSA on at construction."""
        model = cls(hidden_size=config.get("hidden_size", 4096), depth=config.get("depth", 48),
                    num_heads=config.get("num_heads", 32))
        bsa_params = config.get("bsa_params") or {}
        model._bsa_sparsity = float(bsa_params.get("sparsity", 0.9375))
        model._bsa_chunk_thw = tuple(bsa_params.get("chunk_3d_shape_q", [4, 4, 4]))
        topk = bsa_params.get("topk")
        model._bsa_topk = int(topk) if topk is not None else None
        if config.get("enable_bsa", False):
            model.enable_bsa()
        return model

    def enable_bsa(self, backend: str = "tier_a") -> None:
        """longcat_video_dit.py:220-257.  Every backend name of the reference (``tier_a``,
        ``metal``, ``metal_v2..4``) plus ``cuda`` is accepted; all run the sm_100a engine."""
        assert backend in BSA_BACKENDS, f"unknown BSA backend: {backend!r}. Choose from {BSA_BACKENDS}"
        for block in self.blocks:
            block.attn.enable_bsa = True
            block.attn.bsa_sparsity = self._bsa_sparsity
            block.attn.bsa_chunk_thw = self._bsa_chunk_thw
            block.attn.bsa_backend = backend
            block.attn.bsa_topk = self._bsa_topk
        self._prewarm()

    def _prewarm(self) -> None:
        """Pay the engine's one-time costs at enable time, not in the first denoising step (the Metal
        tier's prewarm, block_sparse_attention_metal.py:298-333).  Only where the model lives on a CUDA
        device: a model on the host has no engine to warm."""
        p = next(self.parameters(), None)
        if p is None or not p.is_cuda:
            return
        from .block_sparse_attention_cuda import prewarm_cuda_kernel

        dtype = p.dtype if p.dtype in (torch.bfloat16, torch.float16) else torch.bfloat16
        with torch.cuda.device(p.device):
            prewarm_cuda_kernel(head_dim=self.blocks[0].attn.head_dim, dtype=dtype, device=str(p.device))

    def disable_bsa(self) -> None:
        """longcat_video_dit.py:259-262."""
        for block in self.blocks:
            block.attn.enable_bsa = False

    def attention_modules(self) -> List[Attention]:
        return [b.attn for b in self.blocks]
