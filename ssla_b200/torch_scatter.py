"""``torch_scatter``-compatible ``scatter_sum`` / ``scatter_mean`` / ``scatter_max`` for dim 0.

Drop-in for the imports of layers/sparse_pooling.py:5.  The index may be ``[R]`` or the
``[R, C]`` expansion of one row index that sparse pooling passes (layers/sparse_pooling.py:33);
only ``dim=0`` on 2-D ``src`` is supported, which is the only form the reference uses.  The
reductions run on the GPU: max and mean through the one-pass ``ssla_scatter_pool`` kernel,
sum through a deterministic CSR (see ``ssla_b200.ops.segment``).
"""
from __future__ import annotations

from typing import Optional

import torch

from .ops import segment as _seg


def _prep(src, index, dim, dim_size):
    if dim not in (0, -2) or src.dim() != 2:
        raise NotImplementedError("ssla_b200.torch_scatter supports dim=0 on 2-D src only")
    if index.dim() == 2:
        index = index[:, 0]
    if index.numel() != src.shape[0]:
        raise ValueError("index must have one entry per row of src")
    if dim_size is None:
        dim_size = int(index.max()) + 1 if index.numel() else 0
    return index, int(dim_size)


def scatter_sum(src, index, dim=-1, out=None, dim_size: Optional[int] = None):
    index, S = _prep(src, index, dim, dim_size)
    off, rows = _seg.segment_csr(index, S)
    return _seg.segment_reduce_ad(src, index, off, rows, _seg.SUM)


scatter_add = scatter_sum


def scatter_mean(src, index, dim=-1, out=None, dim_size: Optional[int] = None):
    index, S = _prep(src, index, dim, dim_size)
    return _seg.scatter_mean_ad(src, index, S)


def scatter_max(src, index, dim=-1, out=None, dim_size: Optional[int] = None):
    index, S = _prep(src, index, dim, dim_size)
    return _seg.scatter_max_ad(src, index, S)


def scatter(src, index, dim=-1, out=None, dim_size=None, reduce: str = "sum"):
    if reduce in ("sum", "add"):
        return scatter_sum(src, index, dim, out, dim_size)
    if reduce == "mean":
        return scatter_mean(src, index, dim, out, dim_size)
    if reduce == "max":
        return scatter_max(src, index, dim, out, dim_size)[0]
    raise NotImplementedError(f"reduce={reduce!r}")
