"""Scalar-state GLA (ops/gla/chunk_scalar.py:1044-1092): one scalar state per (sequence,
channel), q, k, v, g ``[T, H]``, state ``[N, H]``, default scale 1.0.

The recurrence ``S_t = exp(g_t) S_{t-1} + k_t v_t``, ``o_t = scale q_t S_t``
(ops/gla/naive_scalar.py:7-66) is element-wise, so it runs token by token per channel in
``ssla_gla_scalar_fwd`` / ``ssla_gla_scalar_bwd`` (HBM-bound, no chunking needed).
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from ... import _lib
from ..utils.guard import input_guard, prepare_cu_seqlens


def _norm(q, k, v, g):
    if q.dim() != 2 or k.shape != q.shape or v.shape != q.shape or g.shape != q.shape:
        raise ValueError(f"chunk_gla_scalar expects q, k, v, g of one shape [T, H]; got {tuple(q.shape)}")
    _lib.require_cuda(q, k, v, g, what="chunk_gla_scalar")
    dt = q.dtype
    _lib.dtype_code(q)
    if g.dtype not in (dt, torch.float32):
        g = g.float()
    return q.contiguous(), k.to(dt).contiguous(), v.to(dt).contiguous(), g.contiguous()


class ChunkGLAScalarFunction(torch.autograd.Function):
    @staticmethod
    @input_guard
    def forward(ctx, q, k, v, g, scale, initial_state, output_final_state, cu_seqlens):
        q, k, v, g = _norm(q, k, v, g)
        cu = prepare_cu_seqlens(cu_seqlens, q.device)
        T, H = q.shape
        N = cu.numel() - 1
        o = torch.empty_like(q)
        ht = torch.empty((N, H), device=q.device, dtype=torch.float32) if output_final_state else None
        h0 = initial_state.float().contiguous() if initial_state is not None else None
        _lib.check(
            _lib.load().ssla_gla_scalar_fwd(
                q.data_ptr(), k.data_ptr(), v.data_ptr(), g.data_ptr(), _lib.dtype_code(q),
                _lib.dtype_code(g), cu.data_ptr(), N, T, H, float(scale), _lib.ptr(h0), o.data_ptr(),
                _lib.ptr(ht), _lib.stream_of(q),
            ),
            "chunk_gla_scalar forward",
        )
        ctx.save_for_backward(q, k, v, g, h0, cu)
        ctx.scale = scale
        return o, ht

    @staticmethod
    @input_guard
    def backward(ctx, do, dht):
        q, k, v, g, h0, cu = ctx.saved_tensors
        T, H = q.shape
        N = cu.numel() - 1
        do = do.to(q.dtype).contiguous()
        dht = dht.float().contiguous() if dht is not None else None
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        dg = torch.empty((T, H), device=q.device, dtype=torch.float32)
        dh0 = torch.empty((N, H), device=q.device, dtype=torch.float32) if h0 is not None else None
        _lib.check(
            _lib.load().ssla_gla_scalar_bwd(
                q.data_ptr(), k.data_ptr(), v.data_ptr(), g.data_ptr(), _lib.dtype_code(q),
                _lib.dtype_code(g), cu.data_ptr(), N, T, H, float(ctx.scale), _lib.ptr(h0),
                do.data_ptr(), _lib.ptr(dht), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(),
                dg.data_ptr(), _lib.ptr(dh0), _lib.stream_of(q),
            ),
            "chunk_gla_scalar backward",
        )
        return dq, dk, dv, dg, None, dh0, None, None


@torch.compiler.disable
def chunk_gla_scalar(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    g: torch.Tensor,
    cu_seqlens: torch.LongTensor,
    scale: Optional[float] = None,
    initial_state: Optional[torch.Tensor] = None,
    output_final_state: bool = False,
) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    r"""Scalar-state GLA over ``[T, H]``; returns ``(o [T, H], final_state [N, H] or None)``."""
    if initial_state is not None and initial_state.shape[0] != len(cu_seqlens) - 1:
        raise ValueError(
            f"The number of initial states is expected to be equal to the number of input sequences, "
            f"i.e., {len(cu_seqlens) - 1} rather than {initial_state.shape[0]}."
        )
    if scale is None:
        scale = 1.0
    return ChunkGLAScalarFunction.apply(q, k, v, g, scale, initial_state, output_final_state, cu_seqlens)
