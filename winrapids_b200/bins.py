"""Statistics of sorted contiguous bins, with the names and return layout of the reference's
Python wrappers (archive/fintek-contributions/src/fused_bin_stats.py:90-160) over the kernel
specification src/winrapids/kernels/bin_stats.cu:25-151.

``fused_bin_stats(data, boundaries)`` returns device tensors count, sum, sum_sq, mean,
variance, std, min, max, first, last for the bins [boundaries[i], boundaries[i + 1]); all of
them come from one library call (tbgb_fused_bin_stats), the derived ones included.
"""
from __future__ import annotations

from . import _torch


def _ctx(device: int):
    from .frame import _ctx as frame_ctx

    return frame_ctx(device)


def _as_device(x, dtype, device: int):
    torch = _torch()
    if isinstance(x, torch.Tensor):
        return x.to(device=f"cuda:{device}", dtype=dtype).contiguous()
    return torch.as_tensor(x, dtype=dtype).to(f"cuda:{device}").contiguous()


def fused_bin_stats(data, boundaries, device: int = 0) -> dict:
    """fused_bin_stats (fused_bin_stats.py:90-144): all basic statistics of every bin."""
    torch = _torch()
    d = _as_device(data, torch.float64, device)
    b = _as_device(boundaries, torch.int64, device)
    if d.dim() != 1:
        raise ValueError("fused_bin_stats takes one column; use fused_multi_column_bin_stats")
    return _ctx(device).fused_bin_stats(d, b)


def fused_multi_column_bin_stats(columns: dict, boundaries, device: int = 0) -> dict:
    """fused_multi_column_bin_stats (fused_bin_stats.py:147-160): {name: stats} for columns
    sharing the boundaries, computed in one launch over the stacked columns (the
    fused_bin_stats_multi layout, bin_stats.cu:85-151)."""
    torch = _torch()
    names = list(columns)
    if not names:
        return {}
    stacked = torch.stack([_as_device(columns[k], torch.float64, device) for k in names])
    b = _as_device(boundaries, torch.int64, device)
    out = _ctx(device).fused_bin_stats(stacked, b)
    return {k: {f: (t if f == "count" else t[j]) for f, t in out.items()} for j, k in enumerate(names)}
