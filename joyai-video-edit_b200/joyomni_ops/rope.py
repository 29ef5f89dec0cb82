"""Host-side RoPE table construction for the fused q/k kernels.

The tables are built once per forward and shared by every block, exactly as
the reference does (deploy/xvideo/models/dit/dit.py:896-934 and :1159-1163):

* ``rope_1d``: interleaved (repeat-interleaved) cos/sin of one axis,
  ``freqs = 1 / theta ** (arange(0, dim, 2)[:dim//2] / dim)``
  (deploy/xvideo/models/dit/rope.py:31-52);
* ``rope_3d``: the (t, h, w) tables concatenated along the head dimension;
* ``paired_tables``: the half-width bf16 ``[L, D/2]`` tables the paired kernels
  read, taken as every other column of the full-width tables
  (deploy/xvideo/models/dit/sgl_fused_ops.py:94-119).

These are small torch tensor computations, not kernels; the hot path only
consumes their output.
"""
from __future__ import annotations

from typing import Sequence, Tuple

import torch


def rope_1d(dim: int, pos: torch.Tensor, theta: float = 10000.0) -> Tuple[torch.Tensor, torch.Tensor]:
    """Full-width interleaved cos/sin [len(pos), dim] (fp32) for one axis."""
    if dim % 2:
        raise ValueError(f"RoPE dimension must be even, got {dim}")
    pos = pos.to(torch.float32)
    freqs = 1.0 / (theta ** (torch.arange(0, dim, 2, device=pos.device)[: dim // 2].float() / dim))
    ang = torch.outer(pos, freqs)
    return ang.cos().repeat_interleave(2, dim=1), ang.sin().repeat_interleave(2, dim=1)


def grid_positions(frames: int, height: int, width: int, t0: int = 0, device=None):
    """(t, h, w) integer positions of a frames x height x width token grid, frame-major."""
    t = torch.arange(frames, device=device, dtype=torch.float32) + float(t0)
    h = torch.arange(height, device=device, dtype=torch.float32)
    w = torch.arange(width, device=device, dtype=torch.float32)
    tt = t.repeat_interleave(height * width)
    hh = h.repeat_interleave(width).repeat(frames)
    ww = w.repeat(frames * height)
    return tt, hh, ww


def rope_3d(positions: Sequence[torch.Tensor], dims: Sequence[int], theta: float = 10000.0):
    """Concatenate per-axis tables: returns full-width fp32 cos/sin [L, sum(dims)]."""
    cos, sin = [], []
    for d, p in zip(dims, positions):
        c, s = rope_1d(d, p, theta)
        cos.append(c)
        sin.append(s)
    return torch.cat(cos, dim=1), torch.cat(sin, dim=1)


def paired_tables(cos: torch.Tensor, sin: torch.Tensor, device=None):
    """Half-width bf16 [L, D/2] tables (one entry per rotated pair)."""
    return (cos[..., ::2].to(device=device, dtype=torch.bfloat16).contiguous(),
            sin[..., ::2].to(device=device, dtype=torch.bfloat16).contiguous())


def video_chunk_tables(frames: int = 3, height: int = 45, width: int = 80, t0: int = 0,
                       dims: Sequence[int] = (44, 42, 42), theta: float = 10000.0, device=None):
    """bf16 [F*H*W, D/2] cos/sin for one streaming chunk's token grid."""
    pos = grid_positions(frames, height, width, t0)
    cos, sin = rope_3d(pos, dims, theta)
    return paired_tables(cos, sin, device=device)
