"""Deterministic segment reductions, row gathers and index_add on the ssla_b200 C ABI.

Replaces the ``torch_scatter.scatter_max`` / ``scatter_mean`` calls of sparse pooling
(layers/sparse_pooling.py:5,33) and the ``index_add_`` gather-back of the MoS routing
(utils/async_utils.py:243-264).  Sums accumulate in fp32 in ascending row order, so fp32
results equal the CPU PyTorch / torch_scatter results bit for bit; max returns the first
maximal row as argmax (the number of rows for empty segments) and 0 for empty segments.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from .. import _lib

SUM, MEAN, MAX = 0, 1, 2


def _i64(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.int64).contiguous()


def segment_offsets_sorted(index: torch.Tensor, num_segments: int) -> torch.Tensor:
    """``[S+1]`` offsets of a non-decreasing row->segment index."""
    _lib.require_cuda(index, what="segment_offsets_sorted")
    index = _i64(index)
    off = torch.empty(num_segments + 1, device=index.device, dtype=torch.int64)
    _lib.check(
        _lib.load().ssla_segment_offsets_sorted(index.data_ptr(), index.numel(), num_segments,
                                                off.data_ptr(), _lib.stream_of(index)),
        "segment_offsets_sorted",
    )
    return off


def segment_csr(index: torch.Tensor, num_segments: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """(offsets [S+1], rows [R]) for an arbitrary index; rows ascending within each segment."""
    _lib.require_cuda(index, what="segment_csr")
    index = _i64(index)
    R = index.numel()
    L = _lib.load()
    off = torch.empty(num_segments + 1, device=index.device, dtype=torch.int64)
    rows = torch.empty(max(R, 1), device=index.device, dtype=torch.int64)
    nb = L.ssla_segment_csr_workspace_bytes(R, num_segments)
    ws = torch.empty(max(nb, 1), device=index.device, dtype=torch.uint8)
    _lib.check(L.ssla_segment_csr(index.data_ptr(), R, num_segments, off.data_ptr(), rows.data_ptr(),
                                  ws.data_ptr(), nb, _lib.stream_of(index)), "segment_csr")
    return off, rows


def segment_reduce(src: torch.Tensor, offsets: torch.Tensor, rows: Optional[torch.Tensor], op: int,
                   want_arg: bool = False):
    """Reduce rows of ``src [R, C]`` per segment described by ``offsets`` (and ``rows``)."""
    _lib.require_cuda(src, offsets, what="segment_reduce")
    src = src.contiguous()
    if src.dim() != 2:
        raise ValueError(f"segment_reduce expects src [R, C], got {tuple(src.shape)}")
    R, C = src.shape
    S = offsets.numel() - 1
    out = torch.empty((S, C), device=src.device, dtype=src.dtype)
    arg = torch.empty((S, C), device=src.device, dtype=torch.int64) if (op == MAX and want_arg) else None
    _lib.check(
        _lib.load().ssla_segment_reduce(src.data_ptr(), _lib.dtype_code(src), offsets.data_ptr(),
                                        _lib.ptr(rows), R, S, C, op, out.data_ptr(), _lib.ptr(arg),
                                        _lib.stream_of(src)),
        "segment_reduce",
    )
    return out, arg


def gather_rows(src: torch.Tensor, index: torch.Tensor) -> torch.Tensor:
    """``src[index]`` for 2-D src (row gather)."""
    _lib.require_cuda(src, index, what="gather_rows")
    src = src.contiguous()
    index = _i64(index)
    out = torch.empty((index.numel(), src.shape[1]), device=src.device, dtype=src.dtype)
    _lib.check(_lib.load().ssla_gather_rows(src.data_ptr(), _lib.dtype_code(src), index.data_ptr(),
                                            index.numel(), src.shape[1], out.data_ptr(),
                                            _lib.stream_of(src)), "gather_rows")
    return out


def scatter_pool(src: torch.Tensor, index: torch.Tensor, num_segments: int, want_max: bool = True,
                 want_mean: bool = True, want_back: bool = False, want_arg: bool = False,
                 want_offsets: bool = False) -> dict:
    """Scatter max and mean of the rows of ``src [R, C]`` into ``num_segments`` segments of an
    arbitrary ``index [R]``, plus the gather of the max back to every row (``back = max[index]``),
    in one pass (``ssla_scatter_pool``).  Returns a dict with the requested of ``max``, ``arg``,
    ``mean``, ``back`` and ``offsets``; results equal :func:`segment_reduce` / :func:`gather_rows`
    bit for bit."""
    _lib.require_cuda(src, index, what="scatter_pool")
    src = src.contiguous()
    index = _i64(index)
    R, C = src.shape
    S = int(num_segments)
    L = _lib.load()
    dev = src.device
    res = {}
    if want_max or want_back or want_arg:
        res["max"] = torch.empty((S, C), device=dev, dtype=src.dtype)
    if want_arg:
        res["arg"] = torch.empty((S, C), device=dev, dtype=torch.int64)
    if want_mean:
        res["mean"] = torch.empty((S, C), device=dev, dtype=src.dtype)
    if want_back:
        res["back"] = torch.empty((R, C), device=dev, dtype=src.dtype)
    if want_offsets:
        res["offsets"] = torch.empty(S + 1, device=dev, dtype=torch.int64)
    nb = L.ssla_scatter_pool_workspace_bytes(R, S)
    ws = torch.empty(max(nb, 1), device=dev, dtype=torch.uint8)
    _lib.check(L.ssla_scatter_pool(src.data_ptr(), _lib.dtype_code(src), index.data_ptr(), R, S, C,
                                   _lib.ptr(res.get("max")), _lib.ptr(res.get("arg")), _lib.ptr(res.get("mean")),
                                   _lib.ptr(res.get("back")), _lib.ptr(res.get("offsets")), ws.data_ptr(), nb,
                                   _lib.stream_of(src)), "scatter_pool")
    return res


def index_add_rows(src: torch.Tensor, index: torch.Tensor, num_rows: int) -> torch.Tensor:
    """``zeros(num_rows, C).index_add_(0, index, src)`` with a fixed (ascending-row) sum order."""
    _lib.require_cuda(src, index, what="index_add_rows")
    src = src.contiguous()
    index = _i64(index)
    P, C = src.shape
    L = _lib.load()
    out = torch.empty((num_rows, C), device=src.device, dtype=src.dtype)
    nb = L.ssla_index_add_rows_workspace_bytes(P, num_rows)
    ws = torch.empty(max(nb, 1), device=src.device, dtype=torch.uint8)
    _lib.check(L.ssla_index_add_rows(src.data_ptr(), _lib.dtype_code(src), index.data_ptr(), P, num_rows,
                                     C, out.data_ptr(), ws.data_ptr(), nb, _lib.stream_of(src)),
               "index_add_rows")
    return out


# --------------------------------------------------------------------------- autograd wrappers
class _GatherRows(torch.autograd.Function):
    @staticmethod
    def forward(ctx, src, index):
        ctx.save_for_backward(index)
        ctx.n = src.shape[0]
        return gather_rows(src, index)

    @staticmethod
    def backward(ctx, grad):
        (index,) = ctx.saved_tensors
        return index_add_rows(grad.contiguous(), index, ctx.n), None


class _IndexAddRows(torch.autograd.Function):
    @staticmethod
    def forward(ctx, src, index, num_rows):
        ctx.save_for_backward(index)
        return index_add_rows(src, index, num_rows)

    @staticmethod
    def backward(ctx, grad):
        (index,) = ctx.saved_tensors
        return gather_rows(grad.contiguous(), index), None, None


class _SegmentReduce(torch.autograd.Function):
    """Reduction with gradients: sum / mean broadcast the output gradient to the rows of each
    segment (divided by the count for mean); max routes it to the arg-max row."""

    @staticmethod
    def forward(ctx, src, seg_of_row, offsets, rows, op):
        out, arg = segment_reduce(src, offsets, rows, op, want_arg=(op == MAX))
        ctx.op = op
        ctx.shape = src.shape
        ctx.save_for_backward(seg_of_row, offsets, arg if arg is not None else offsets)
        return out

    @staticmethod
    def backward(ctx, grad):
        seg, offsets, arg = ctx.saved_tensors
        R, C = ctx.shape
        grad = grad.contiguous()
        if ctx.op == MAX:
            gin = torch.zeros((R + 1, C), device=grad.device, dtype=grad.dtype)  # row R: empty segments
            gin.scatter_(0, arg, grad)
            return gin[:R], None, None, None, None
        g = gather_rows(grad, seg)
        if ctx.op == MEAN:
            cnt = (offsets[1:] - offsets[:-1]).clamp(min=1).to(grad.dtype)
            g = g / gather_rows(cnt.view(-1, 1).contiguous(), seg)
        return g, None, None, None, None


def gather_rows_ad(src: torch.Tensor, index: torch.Tensor) -> torch.Tensor:
    """Differentiable ``src[index]``."""
    return _GatherRows.apply(src.contiguous(), _i64(index))


def index_add_rows_ad(src: torch.Tensor, index: torch.Tensor, num_rows: int) -> torch.Tensor:
    """Differentiable deterministic ``zeros(num_rows, C).index_add_(0, index, src)``."""
    return _IndexAddRows.apply(src.contiguous(), _i64(index), int(num_rows))


def segment_reduce_ad(src: torch.Tensor, seg_of_row: torch.Tensor, offsets: torch.Tensor, rows, op: int):
    """Differentiable segment reduction; ``seg_of_row`` is the segment id of every row."""
    return _SegmentReduce.apply(src.contiguous(), _i64(seg_of_row), offsets, rows, op)


class _ScatterPool(torch.autograd.Function):
    """One-pass scatter max (with argmax) or mean of an arbitrary index, with gradients:
    max routes the output gradient to the arg-max row, mean spreads it over the segment."""

    @staticmethod
    def forward(ctx, src, index, num_segments, op):
        is_max = op == MAX
        res = scatter_pool(src, index, num_segments, want_max=is_max, want_mean=not is_max, want_arg=is_max,
                           want_offsets=not is_max)
        ctx.op = op
        ctx.shape = src.shape
        if is_max:
            ctx.save_for_backward(res["arg"])
            ctx.mark_non_differentiable(res["arg"])
            return res["max"], res["arg"]
        ctx.save_for_backward(index, res["offsets"])
        return res["mean"], res["offsets"]

    @staticmethod
    def backward(ctx, grad, _unused):
        R, C = ctx.shape
        grad = grad.contiguous()
        if ctx.op == MAX:
            (arg,) = ctx.saved_tensors
            gin = torch.zeros((R + 1, C), device=grad.device, dtype=grad.dtype)  # row R: empty segments
            gin.scatter_(0, arg, grad)
            return gin[:R], None, None, None
        index, offsets = ctx.saved_tensors
        cnt = (offsets[1:] - offsets[:-1]).clamp(min=1).to(grad.dtype)
        return gather_rows(grad, index) / gather_rows(cnt.view(-1, 1).contiguous(), index), None, None, None


def scatter_max_ad(src: torch.Tensor, index: torch.Tensor, num_segments: int):
    """Differentiable one-pass ``(max, argmax)`` of an arbitrary index (torch_scatter.scatter_max)."""
    return _ScatterPool.apply(src.contiguous(), _i64(index), int(num_segments), MAX)


def scatter_mean_ad(src: torch.Tensor, index: torch.Tensor, num_segments: int) -> torch.Tensor:
    """Differentiable one-pass mean of an arbitrary index (torch_scatter.scatter_mean)."""
    return _ScatterPool.apply(src.contiguous(), _i64(index), int(num_segments), MEAN)[0]
