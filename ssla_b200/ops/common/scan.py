"""Element-wise gated scan ``h_t = g_t * h_{t-1} + u_t`` (ops/common/scan.py:140-163).

Same signature, layout and autograd behaviour as the reference ``scan``; the forward and
backward kernels are ``ssla_scan_fwd`` / ``ssla_scan_bwd`` of the C ABI.
"""
from __future__ import annotations

from typing import Tuple

import torch
from torch.autograd import Function

from ... import _lib
from ..utils.guard import prepare_cu_seqlens


def scan_fwd(u: torch.Tensor, g: torch.Tensor, cu_seqlens: torch.Tensor) -> torch.Tensor:
    """h [T, C] in u's dtype (ops/common/scan.py:92-114)."""
    _lib.require_cuda(u, g, what="scan")
    if u.dim() != 2 or g.shape != u.shape:
        raise ValueError(f"scan expects u, g of one shape [T, C], got {tuple(u.shape)} and {tuple(g.shape)}")
    u = u.contiguous()
    g = g.contiguous()
    cu = prepare_cu_seqlens(cu_seqlens, u.device)
    T, C = u.shape
    h = torch.empty_like(u)
    with torch.cuda.device(u.device):
        _lib.check(
            _lib.load().ssla_scan_fwd(
                u.data_ptr(), _lib.dtype_code(u), g.data_ptr(), _lib.dtype_code(g), h.data_ptr(),
                _lib.dtype_code(h), cu.data_ptr(), cu.numel() - 1, T, C, _lib.stream_of(u),
            ),
            "scan",
        )
    return h


def scan_bwd(do: torch.Tensor, g: torch.Tensor, h: torch.Tensor, cu_seqlens: torch.Tensor):
    """(du, dg) (ops/common/scan.py:116-137)."""
    do = do.to(h.dtype).contiguous()
    cu = prepare_cu_seqlens(cu_seqlens, h.device)
    T, C = h.shape
    du = torch.empty_like(h)
    dg = torch.empty_like(g)
    with torch.cuda.device(h.device):
        _lib.check(
            _lib.load().ssla_scan_bwd(
                do.data_ptr(), _lib.dtype_code(do), g.data_ptr(), _lib.dtype_code(g), h.data_ptr(),
                _lib.dtype_code(h), du.data_ptr(), _lib.dtype_code(du), dg.data_ptr(),
                _lib.dtype_code(dg), cu.data_ptr(), cu.numel() - 1, T, C, _lib.stream_of(h),
            ),
            "scan backward",
        )
    return du, dg


class SequentialScan(Function):
    @staticmethod
    def forward(ctx, u: torch.Tensor, g: torch.Tensor, cu_seqlens: torch.Tensor) -> torch.Tensor:
        g = g.contiguous()
        h = scan_fwd(u, g, cu_seqlens)
        ctx.save_for_backward(g, h)
        ctx.cu_seqlens = cu_seqlens
        return h

    @staticmethod
    def backward(ctx, do: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor, None]:
        g, h = ctx.saved_tensors
        du, dg = scan_bwd(do, g, h, ctx.cu_seqlens)
        return du, dg, None


@torch.compiler.disable
def scan(u: torch.Tensor, g: torch.Tensor, cu_seqlens: torch.Tensor) -> torch.Tensor:
    r"""Causal scan with forget gates: ``h_t = g_t * h_{t-1} + u_t`` per channel.

    Args:
        u: inputs ``[T, C]``.
        g: forget gates ``[T, C]``.
        cu_seqlens: cumulative sequence lengths ``[N+1]`` (packed variable-length layout).
    Returns:
        h: ``[T, C]`` in u's dtype.
    """
    return SequentialScan.apply(u, g, cu_seqlens)
