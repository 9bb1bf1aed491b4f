"""Recurrent (token-by-token) GLA for low-latency streaming inference.

``fused_recurrent_gla`` has ``chunk_gla``'s signature (ops/gla/chunk.py:1120-1129) and the
semantics of ``naive_gla_recurrent`` (ops/gla/naive.py:50-111): per token the state is first
decayed and updated, ``S_t = diag(exp(g_t)) S_{t-1} + k_t v_t^T``, then read out,
``o_t = (scale q_t)^T S_t`` (o in q's dtype, state fp32).  The reference has no fused
recurrent kernel; the forward here is ``ssla_recurrent_gla_fwd``.  Gradients are exact
gradients of the same function and are computed with the chunked backward kernels.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from ... import _lib
from ..utils.guard import input_guard, prepare_cu_seqlens
from .chunk import chunk_gla_bwd, chunk_gla_fwd, norm_inputs


def fused_recurrent_gla_fwd(q, k, v, g, scale, initial_state, output_final_state, cu_seqlens):
    T, H, K = q.shape
    V = v.shape[-1]
    N = cu_seqlens.numel() - 1
    o = torch.empty((T, H, V), device=q.device, dtype=q.dtype)
    ht = torch.empty((N, H, K, V), device=q.device, dtype=torch.float32) if output_final_state else None
    h0 = initial_state.float().contiguous() if initial_state is not None else None
    _lib.check(
        _lib.load().ssla_recurrent_gla_fwd(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), g.data_ptr(), _lib.dtype_code(q),
            _lib.dtype_code(g), cu_seqlens.data_ptr(), N, T, H, K, V, float(scale), _lib.ptr(h0),
            o.data_ptr(), _lib.ptr(ht), _lib.stream_of(q),
        ),
        "fused_recurrent_gla",
    )
    return o, ht


class FusedRecurrentGLAFunction(torch.autograd.Function):
    @staticmethod
    @input_guard
    def forward(ctx, q, k, v, g, scale, initial_state, output_final_state, cu_seqlens):
        q, k, v, g = norm_inputs(q, k, v, g)
        cu = prepare_cu_seqlens(cu_seqlens, q.device)
        o, ht = fused_recurrent_gla_fwd(q, k, v, g, scale, initial_state, output_final_state, cu)
        h0 = initial_state.float().contiguous() if initial_state is not None else None
        ctx.save_for_backward(q, k, v, g, h0, cu)
        ctx.scale = scale
        return o, ht

    @staticmethod
    @input_guard
    def backward(ctx, do, dht):
        q, k, v, g, h0, cu = ctx.saved_tensors
        # chunk-start states of the same recurrence, then the chunked adjoint pass
        _, _, states = chunk_gla_fwd(q, k, v, g, ctx.scale, h0, False, cu)
        dq, dk, dv, dg, dh0 = chunk_gla_bwd(q, k, v, g, ctx.scale, h0 is not None, states, do, dht, cu)
        return dq, dk, dv, dg, None, dh0, None, None


@torch.compiler.disable
def fused_recurrent_gla(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    g: torch.Tensor,
    cu_seqlens: torch.LongTensor,
    scale: Optional[float] = None,
    initial_state: Optional[torch.Tensor] = None,
    output_final_state: bool = False,
) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    r"""Recurrent GLA; arguments and returns as ``chunk_gla``.  Carry ``final_state`` into the
    next call as ``initial_state`` to stream one step at a time."""
    if initial_state is not None and initial_state.shape[0] != len(cu_seqlens) - 1:
        raise ValueError(
            f"The number of initial states is expected to be equal to the number of input sequences, "
            f"i.e., {len(cu_seqlens) - 1} rather than {initial_state.shape[0]}."
        )
    if scale is None:
        scale = q.shape[-1] ** -0.5
    return FusedRecurrentGLAFunction.apply(q, k, v, g, scale, initial_state, output_final_state, cu_seqlens)
