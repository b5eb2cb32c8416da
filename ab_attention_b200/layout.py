"""Video token layouts: the optional 4x4x4 cube permutation.

`cube_layout(t, h, w)` returns the token order the reference installs at the
transformer entry (ab_attention/video.py:97-105): the row-major (t, h, w) grid
is padded to multiples of 4 with -1, split into 4x4x4 cubes in (cube_t,
cube_h, cube_w) order, flattened, and the padding dropped, so boundary cubes
hold their valid tokens only. `inverse` restores raster order.
"""
from __future__ import annotations

import torch


def cube_layout(t: int, h: int, w: int, device=None):
    grid = torch.arange(t * h * w, device=device).reshape(t, h, w)
    grid = torch.nn.functional.pad(grid, (0, -w % 4, 0, -h % 4, 0, -t % 4), value=-1)
    nt, nh, nw = (size // 4 for size in grid.shape)
    order = grid.reshape(nt, 4, nh, 4, nw, 4).permute(0, 2, 4, 1, 3, 5).reshape(-1)
    order = order[order >= 0]
    return order, order.argsort()


def to_cubes(x: torch.Tensor, order: torch.Tensor, dim: int = 2) -> torch.Tensor:
    """Permute the token axis of x into cube order."""
    return x.index_select(dim, order)


def from_cubes(x: torch.Tensor, inverse: torch.Tensor, dim: int = 2) -> torch.Tensor:
    """Restore raster order."""
    return x.index_select(dim, inverse)
