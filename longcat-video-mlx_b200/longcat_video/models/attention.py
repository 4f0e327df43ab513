"""DiT visual self-attention with the BSA hook (xocialize/longcat-video-mlx
``longcat_video/models/attention.py:35-275``), in torch, with the hook routed to the B200 engine.

Only what the BSA path needs is here: QKV projection, fp32 RMSNorm on q/k (blocks.py:55-73),
3-D RoPE, ``_process_attn`` (the hook, :71-179) and the output projection.  On the BSA path the q/k
RMSNorm and the RoPE run fused in the engine's routing kernel, and the engine writes its output in the
[B, N, H, D] order the projection reads.  Every BSA backend
name the reference accepts routes to the one CUDA engine; the hook's own fallback -- a
shape that is not a multiple of chunk_thw falls back to dense attention (:174-179) -- is kept as
the reference has it, and only for that error.  With BSA on, RoPE is fused into the routing
kernel instead of being applied as a separate pass.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.nn.functional as F

from .._native import BSAShapeError
from .block_sparse_attention import bsa_attention
from .rope_3d import RotaryPositionalEmbedding

BSA_BACKENDS = ("tier_a", "metal", "metal_v2", "metal_v3", "metal_v4", "cuda")


class RMSNorm_FP32(torch.nn.Module):
    """blocks.py:55-73: fp32 RMS normalisation, weight applied in the input dtype."""

    def __init__(self, dim: int, eps: float):
        super().__init__()
        self.eps = eps
        self.weight = torch.nn.Parameter(torch.ones(dim))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        xf = x.float()
        norm = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps)
        return norm.to(x.dtype) * self.weight.to(x.dtype)


class Attention(torch.nn.Module):
    def __init__(self, dim: int, num_heads: int):
        super().__init__()
        assert dim % num_heads == 0, "dim must be divisible by num_heads"
        self.dim = dim
        self.num_heads = num_heads
        self.head_dim = dim // num_heads
        self.scale = self.head_dim ** -0.5
        self.qkv = torch.nn.Linear(dim, dim * 3, bias=True)
        self.q_norm = RMSNorm_FP32(self.head_dim, eps=1e-6)
        self.k_norm = RMSNorm_FP32(self.head_dim, eps=1e-6)
        self.proj = torch.nn.Linear(dim, dim)
        self.rope_3d = RotaryPositionalEmbedding(self.head_dim)
        # attention.py:62-69 defaults
        self.enable_bsa: bool = False
        self.bsa_sparsity: float = 0.9375
        self.bsa_chunk_thw: Tuple[int, int, int] = (4, 4, 4)
        self.bsa_backend: str = "tier_a"
        self.bsa_topk: Optional[int] = None  # explicit k overrides the floor rule

    def _bsa_ok(self, q: torch.Tensor, k: torch.Tensor, shape) -> bool:
        return self.enable_bsa and shape is not None and q.shape[-2] == k.shape[-2]

    def _process_attn(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                      shape: Optional[Tuple[int, int, int]] = None, rope_grid=None,
                      out: Optional[torch.Tensor] = None, raw_qk: bool = False) -> torch.Tensor:
        """attention.py:71-179.  q, k, v: [B, H, S, D].  With ``rope_grid`` set, q and k are
        pre-RoPE: the BSA path fuses the rotation, the dense path applies it first.  With ``raw_qk``
        they are also pre-RMSNorm (attention.py:195-196): the BSA path fuses q_norm / k_norm in front of
        the rotation, the dense path applies them first.  ``out`` (device tensors only): a
        [B, H, S, D] view the BSA path writes in place -- any strides, e.g. a permuted [B, S, H, D]
        buffer; the dense path ignores it."""
        if self._bsa_ok(q, k, shape):
            try:
                rope = self.rope_3d.tables(rope_grid, q.device) if rope_grid is not None else None
                qk_norm = (self.q_norm.weight, self.k_norm.weight, self.q_norm.eps) if raw_qk else None
                return bsa_attention(q, k, v, shape=shape, sparsity=self.bsa_sparsity,
                                     chunk_thw=self.bsa_chunk_thw, sm_scale=self.scale, topk=self.bsa_topk,
                                     rope=rope, out=out, qk_norm=qk_norm)
            except BSAShapeError:
                # shape not a multiple of chunk_thw: the reference falls back to dense attention
                # here (attention.py:174-179).  Every other engine error (unsupported head_dim or
                # dtype) propagates: a silent dense fallback would cost 1/(1 - sparsity) times the
                # FLOPs with no message.  Views the kernels cannot read in place are copied once by
                # the engine's host layer, not refused.
                pass
        if raw_qk:
            q, k = self.q_norm(q), self.k_norm(k)
        if rope_grid is not None:
            q, k = self.rope_3d(q, k, rope_grid)
        return F.scaled_dot_product_attention(q, k, v, scale=self.scale)

    def forward(self, x: torch.Tensor, shape: Tuple[int, int, int],
                num_cond_latents: Optional[int] = None, return_kv: bool = False):
        """attention.py:181-233.  x: [B, N, C] -> [B, N, C].  With ``return_kv`` also returns the
        (k, v) of this call for a later :meth:`forward_with_kv_cache`: k after RMSNorm, before RoPE."""
        B, N, C = x.shape
        qkv = self.qkv(x).reshape(B, N, 3, self.num_heads, self.head_dim).permute(2, 0, 3, 1, 4)
        q, k, v = qkv[0], qkv[1], qkv[2]
        # the q/k RMSNorm runs fused in the engine's routing kernel (one read of the raw q/k, one write of
        # the normalised, rotated q/k) when the call takes the BSA path on the GPU in bf16/fp16
        fuse_norm = (not return_kv and not (num_cond_latents is not None and num_cond_latents > 0)
                     and self._bsa_ok(q, k, shape) and q.is_cuda and q.dtype in (torch.bfloat16, torch.float16)
                     and self.q_norm.eps == self.k_norm.eps)
        if not fuse_norm:
            q = self.q_norm(q)
            k = self.k_norm(k)
        kv = (k, v) if return_kv else None
        if num_cond_latents is not None and num_cond_latents > 0:
            q, k = self.rope_3d(q, k, shape)
            ncl = num_cond_latents * (N // shape[0])
            cond_shape = (num_cond_latents, shape[1], shape[2])
            x_cond = self._process_attn(q[:, :, :ncl], k[:, :, :ncl], v[:, :, :ncl], shape=cond_shape)
            x_noise = self._process_attn(q[:, :, ncl:], k, v, shape=None)
            out = torch.cat([x_cond, x_noise], dim=2)
        else:
            # the engine writes straight into a [B, N, H, D] buffer (attention.py:228-229 transposes to
            # it), so proj reads the result without a transpose copy
            o_nhd = None
            if self.enable_bsa and q.is_cuda:
                o_nhd = torch.empty((B, N, self.num_heads, self.head_dim), device=q.device, dtype=q.dtype)
            out = self._process_attn(q, k, v, shape=shape, rope_grid=shape,
                                     out=o_nhd.permute(0, 2, 1, 3) if o_nhd is not None else None,
                                     raw_qk=fuse_norm)
            if o_nhd is not None and out.data_ptr() == o_nhd.data_ptr():
                out = self.proj(o_nhd.view(B, N, C))
                return (out, kv) if return_kv else out
        out = self.proj(out.transpose(1, 2).reshape(B, N, C))
        return (out, kv) if return_kv else out

    def forward_with_kv_cache(self, x: torch.Tensor, shape: Tuple[int, int, int], num_cond_latents: Optional[int],
                              kv_cache: Tuple[torch.Tensor, torch.Tensor]) -> torch.Tensor:
        """attention.py:235-275: chunked continuation.  The fresh K/V are appended to the cached ones
        (a cache stored at batch 1 is broadcast to B).  With conditioning latents, q is padded with zeros
        over the cache positions so that RoPE over the extended grid (T + num_cond_latents, H, W) gives
        q and k their global positions.  Q and KV lengths differ, so the hook takes its dense path."""
        B, N, C = x.shape
        qkv = self.qkv(x).reshape(B, N, 3, self.num_heads, self.head_dim).permute(2, 0, 3, 1, 4)
        q, k, v = qkv[0], qkv[1], qkv[2]
        q = self.q_norm(q)
        k = self.k_norm(k)
        T, Hl, Wl = shape
        k_cache, v_cache = kv_cache
        if k_cache.shape[0] == 1 and B > 1:
            k_cache = k_cache.expand(B, *k_cache.shape[1:])
            v_cache = v_cache.expand(B, *v_cache.shape[1:])
        k_full = torch.cat([k_cache, k], dim=2)
        v_full = torch.cat([v_cache, v], dim=2)
        if num_cond_latents is not None and num_cond_latents > 0:
            q_pad = torch.cat([torch.zeros_like(k_cache), q], dim=2)
            q_pad, k_full = self.rope_3d(q_pad, k_full, (T + num_cond_latents, Hl, Wl))
            q = q_pad[:, :, -N:]
        out = self._process_attn(q, k_full, v_full, shape=None)
        return self.proj(out.transpose(1, 2).reshape(B, N, C))
