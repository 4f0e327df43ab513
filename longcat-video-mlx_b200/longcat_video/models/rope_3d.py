"""3-D rotary position embedding (xocialize/longcat-video-mlx ``longcat_video/models/rope_3d.py``).

The head dimension is split into (dim_t, dim_h, dim_w) = (D - 4*(D//6), 2*(D//6), 2*(D//6))
(:60-62), each axis uses inverse frequencies ``base^-(2i/dim)`` (:65-70) over integer grid
positions (:79-82), every frequency drives one adjacent pair (:91-93), and
``x*cos + rotate_half(x)*sin`` is evaluated in fp32 and cast back (:120-128).

On B200 the rotation is fused into the BSA routing kernel: ``RopeTables`` builds the per-axis
fp32 angle tables once per grid and hands them to the engine (``bsa_attention(..., rope=...)``),
which rotates Q and K on their single pass through HBM.  ``RotaryPositionalEmbedding.__call__``
keeps the unfused torch form for the dense (non-BSA) attention path.
"""

from __future__ import annotations

from typing import Dict, Tuple

import numpy as np
import torch

__all__ = ["rotate_half", "rope_axis_dims", "rope_axis_tables", "RopeTables", "RotaryPositionalEmbedding"]


def rope_axis_dims(head_dim: int) -> Tuple[int, int, int]:
    d6 = head_dim // 6
    return head_dim - 4 * d6, 2 * d6, 2 * d6


def rope_axis_tables(grid: Tuple[int, int, int], head_dim: int, base: float = 10000.0):
    """Per-axis fp32 (cos, sin) tables, one column per rotated pair:
    [(T, dt/2), (H, dh/2), (W, dw/2)].  All arithmetic in fp32 as in rope_3d.py:65-93."""
    out = []
    for n, dim in zip(grid, rope_axis_dims(head_dim)):
        idx = np.arange(0, dim, 2, dtype=np.float32)[: dim // 2]
        freqs = (np.float32(1.0) / (np.float32(base) ** (idx / np.float32(dim)))).astype(np.float32)
        pos = np.arange(0, n, dtype=np.float32)
        ang = (pos[:, None] * freqs[None, :]).astype(np.float32)
        out.append((np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)))
    return out


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    """rope_3d.py:23-34: adjacent pairs (x0, x1) -> (-x1, x0)."""
    y = x.unflatten(-1, (-1, 2))
    return torch.stack((-y[..., 1], y[..., 0]), dim=-1).flatten(-2)


class RopeTables:
    """Device-resident per-axis tables for one grid, in the layout the engine's C ABI expects
    (cos_t | sin_t | cos_h | sin_h | cos_w | sin_w, fp32)."""

    def __init__(self, grid: Tuple[int, int, int], head_dim: int, device, base: float = 10000.0):
        self.grid = tuple(int(g) for g in grid)
        self.head_dim = int(head_dim)
        self.dims = rope_axis_dims(self.head_dim)
        tabs = rope_axis_tables(self.grid, self.head_dim, base)
        flat = np.concatenate([np.concatenate([c.ravel(), s.ravel()]) for c, s in tabs]).astype(np.float32)
        self.host = flat
        self.tables = torch.from_numpy(flat).to(device)

    def native_args(self):
        return self.tables, self.dims, self.grid

    def full(self) -> Tuple[torch.Tensor, torch.Tensor]:
        """[S, D] cos and sin in the reference's layout (rope_3d.py:91-105), on the device."""
        T, H_, W = self.grid
        tabs = rope_axis_tables(self.grid, self.head_dim)
        reps = []
        for (c, s), bshape in zip(tabs, ((T, 1, 1), (1, H_, 1), (1, 1, W))):
            c2 = np.repeat(c, 2, axis=-1)
            s2 = np.repeat(s, 2, axis=-1)
            reps.append((np.broadcast_to(c2.reshape(*bshape, -1), (T, H_, W, c2.shape[-1])),
                         np.broadcast_to(s2.reshape(*bshape, -1), (T, H_, W, s2.shape[-1]))))
        cos = np.concatenate([r[0] for r in reps], axis=-1).reshape(T * H_ * W, self.head_dim)
        sin = np.concatenate([r[1] for r in reps], axis=-1).reshape(T * H_ * W, self.head_dim)
        dev = self.tables.device
        return torch.from_numpy(np.ascontiguousarray(cos)).to(dev), torch.from_numpy(np.ascontiguousarray(sin)).to(dev)


class RotaryPositionalEmbedding(torch.nn.Module):
    """rope_3d.py:37-128; tables are memoised per (grid, device)."""

    def __init__(self, head_dim: int):
        super().__init__()
        assert head_dim % 8 == 0, "head_dim must be a multiple of 8 for 3D RoPE"
        self.head_dim = head_dim
        self.base = 10000
        self._cache: Dict[tuple, RopeTables] = {}

    def tables(self, grid_size: Tuple[int, int, int], device) -> RopeTables:
        key = (tuple(grid_size), str(device))
        if key not in self._cache:
            self._cache[key] = RopeTables(grid_size, self.head_dim, device, self.base)
        return self._cache[key]

    def forward(self, q: torch.Tensor, k: torch.Tensor, grid_size: Tuple[int, int, int]):
        """q, k: [B, H, S, D] -> rotated (q, k), fp32 math, cast back (rope_3d.py:107-128)."""
        cos, sin = self.tables(grid_size, q.device).full()
        out_dtype = q.dtype
        qf, kf = q.float(), k.float()
        q_r = qf * cos + rotate_half(qf) * sin
        k_r = kf * cos + rotate_half(kf) * sin
        return q_r.to(out_dtype), k_r.to(out_dtype)
