"""CPU restatement of the segment reductions used by sparse pooling (test infrastructure only).

The reference calls ``torch_scatter.scatter_max`` / ``scatter_mean`` on rows grouped by
``unique_consecutive`` inverse ids (layers/sparse_pooling.py:26-33).  torch_scatter is a
third-party package (installed from the torch-2.6.0+cu124 wheel index per README.md:18,
version unpinned, not vendored, not installed here), so this restates its documented
semantics for ``dim=0`` with ``dim_size``:
  * scatter_sum: out[s] = sum of src rows with index s, accumulated in ascending row order
    (its CPU kernel's order) in the output dtype's fp32 promotion; empty segments 0;
  * scatter_mean: scatter_sum / count, count clamped to >= 1;
  * scatter_max: out initialised to the dtype's lowest value, updated when a row is strictly
    greater (so the first maximum wins), argmax initialised to the number of rows; entries
    left at the lowest value are set to 0.
``index_add`` restates ``zeros(E,C).index_add_(0, idx, src)`` of utils/async_utils.py:262-263
on the CPU (sequential in ascending source row).
Parity status: unpinned against torch_scatter (absent); pinned for index_add by comparing
with CPU ``torch.index_add_`` in the tests.
"""
from __future__ import annotations

import torch


def scatter_sum(src, index, dim_size):
    out = torch.zeros(dim_size, src.shape[1], dtype=torch.float32)
    for r in range(src.shape[0]):
        out[int(index[r])] += src[r].float()
    return out.to(src.dtype)


def scatter_sum_fast(src, index, dim_size):
    """Same accumulation order as ``scatter_sum`` (CPU index_add_ is sequential)."""
    out = torch.zeros(dim_size, src.shape[1], dtype=torch.float32)
    out.index_add_(0, index.to(torch.int64), src.float())
    return out.to(src.dtype)


def scatter_mean(src, index, dim_size):
    s = torch.zeros(dim_size, src.shape[1], dtype=torch.float32)
    s.index_add_(0, index.to(torch.int64), src.float())
    cnt = torch.bincount(index.to(torch.int64), minlength=dim_size).clamp(min=1).to(torch.float32)
    return (s / cnt[:, None]).to(src.dtype)


def scatter_max(src, index, dim_size):
    """(out, argmax) with first-maximum tie breaking; argmax = R for empty segments."""
    R, C = src.shape
    idx = index.to(torch.int64)
    srcf = src.float()
    lowest = float(torch.finfo(src.dtype).min)
    out = torch.full((dim_size, C), lowest, dtype=torch.float32)
    out.scatter_reduce_(0, idx[:, None].expand(R, C), srcf, reduce="amax", include_self=True)
    # first row achieving the max: candidates where src == out[idx] and src > lowest
    hit = (srcf == out[idx]) & (srcf > lowest)
    rows = torch.arange(R)[:, None].expand(R, C)
    cand = torch.where(hit, rows, torch.full_like(rows, R))
    arg = torch.full((dim_size, C), R, dtype=torch.int64)
    arg.scatter_reduce_(0, idx[:, None].expand(R, C), cand, reduce="amin", include_self=True)
    out = torch.where(out == lowest, torch.zeros_like(out), out)
    return out.to(src.dtype), arg


def index_add_rows(src, index, num_rows):
    out = torch.zeros(num_rows, src.shape[1], dtype=torch.float32)
    out.index_add_(0, index.to(torch.int64), src.float())
    return out.to(src.dtype)
