"""Chunked gated linear attention (ops/gla/chunk.py:1119-1167) on the ssla_b200 C ABI.

``chunk_gla(q, k, v, g, cu_seqlens, scale=None, initial_state=None, output_final_state=False)``
keeps the reference signature, packed layout (q, k, g ``[T, H, K]``, v ``[T, H, V]``,
``cu_seqlens [N+1]``), dtypes (o in v's dtype, final state fp32, dg fp32 before autograd's
cast) and error behaviour (``ValueError`` when ``initial_state`` does not have one entry per
sequence, ops/gla/chunk.py:1159-1163).
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from ... import _lib
from ..utils.guard import input_guard, prepare_cu_seqlens


def norm_inputs(q, k, v, g):
    if q.dim() != 3 or k.shape != q.shape or g.shape != q.shape or v.dim() != 3 or v.shape[:2] != q.shape[:2]:
        raise ValueError(
            f"expected q, k, g [T, H, K] and v [T, H, V]; got q {tuple(q.shape)}, k {tuple(k.shape)}, "
            f"v {tuple(v.shape)}, g {tuple(g.shape)}"
        )
    _lib.require_cuda(q, k, v, g, what="chunk_gla")
    dt = q.dtype
    _lib.dtype_code(q)
    k = k.to(dt).contiguous()
    v = v.to(dt).contiguous()
    if g.dtype not in (dt, torch.float32):
        g = g.float()
    return q.contiguous(), k, v, g.contiguous()


def chunk_gla_fwd(q, k, v, g, scale, initial_state, output_final_state, cu_seqlens):
    """Returns (o, ht or None, states).  ``states`` is the opaque device buffer the forward
    leaves for the backward (the chunk table, which chunks the exact kernels handle, and the
    state at every chunk start)."""
    T, H, K = q.shape
    V = v.shape[-1]
    N = cu_seqlens.numel() - 1
    L = _lib.load()
    dev = q.device
    dt, dtg = _lib.dtype_code(q), _lib.dtype_code(g)
    o = torch.empty_like(v)
    st_bytes = L.ssla_chunk_gla_states_bytes(N, T, H, K, V, dt, dtg)
    states = torch.empty(max(st_bytes, 1), device=dev, dtype=torch.uint8)
    ht = torch.empty((N, H, K, V), device=dev, dtype=torch.float32) if output_final_state else None
    h0 = initial_state.float().contiguous() if initial_state is not None else None
    ws_bytes = L.ssla_chunk_gla_workspace_bytes(N, T, H, K, V, dt, dtg)
    ws = torch.empty(max(ws_bytes, 1), device=dev, dtype=torch.uint8)
    _lib.check(
        L.ssla_chunk_gla_fwd(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), g.data_ptr(), dt, dtg, cu_seqlens.data_ptr(), N, T, H, K, V,
            float(scale), _lib.ptr(h0), o.data_ptr(), _lib.ptr(ht), states.data_ptr(), st_bytes, ws.data_ptr(),
            ws_bytes, _lib.stream_of(q),
        ),
        "chunk_gla forward",
    )
    return o, ht, states


def chunk_gla_bwd(q, k, v, g, scale, has_h0, states, do, dht, cu_seqlens):
    T, H, K = q.shape
    V = v.shape[-1]
    N = cu_seqlens.numel() - 1
    L = _lib.load()
    dev = q.device
    dt, dtg = _lib.dtype_code(q), _lib.dtype_code(g)
    do = do.to(q.dtype).contiguous()
    dht = dht.float().contiguous() if dht is not None else None
    dq = torch.empty_like(q)
    dk = torch.empty_like(k)
    dv = torch.empty_like(v)
    dg = torch.empty(g.shape, device=dev, dtype=torch.float32)
    dh0 = torch.empty((N, H, K, V), device=dev, dtype=torch.float32) if has_h0 else None
    ws_bytes = L.ssla_chunk_gla_workspace_bytes(N, T, H, K, V, dt, dtg)
    ws = torch.empty(max(ws_bytes, 1), device=dev, dtype=torch.uint8)
    _lib.check(
        L.ssla_chunk_gla_bwd(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), g.data_ptr(), dt, dtg, cu_seqlens.data_ptr(), N, T, H, K, V,
            float(scale), states.data_ptr(), states.numel(), do.data_ptr(), _lib.ptr(dht), dq.data_ptr(),
            dk.data_ptr(), dv.data_ptr(), dg.data_ptr(), _lib.ptr(dh0), ws.data_ptr(), ws_bytes, _lib.stream_of(q),
        ),
        "chunk_gla backward",
    )
    return dq, dk, dv, dg, dh0


class ChunkGLAFunction(torch.autograd.Function):
    @staticmethod
    @input_guard
    def forward(ctx, q, k, v, g, scale, initial_state, output_final_state, cu_seqlens):
        q, k, v, g = norm_inputs(q, k, v, g)
        cu = prepare_cu_seqlens(cu_seqlens, q.device)
        o, ht, states = chunk_gla_fwd(q, k, v, g, scale, initial_state, output_final_state, cu)
        ctx.save_for_backward(q, k, v, g, states, cu)
        ctx.scale = scale
        ctx.has_h0 = initial_state is not None
        return o, ht

    @staticmethod
    @input_guard
    def backward(ctx, do, dht):
        q, k, v, g, states, cu = ctx.saved_tensors
        dq, dk, dv, dg, dh0 = chunk_gla_bwd(q, k, v, g, ctx.scale, ctx.has_h0, states, do, dht, cu)
        return dq, dk, dv, dg, None, dh0, None, None


@torch.compiler.disable
def chunk_gla(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    g: torch.Tensor,
    cu_seqlens: torch.LongTensor,
    scale: Optional[float] = None,
    initial_state: Optional[torch.Tensor] = None,
    output_final_state: bool = False,
) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    r"""Chunked GLA over packed variable-length sequences.

    Args:
        q, k: ``[T, H, K]``; v: ``[T, H, V]``; g: log forget gates ``[T, H, K]``.
        cu_seqlens: cumulative sequence lengths ``[N+1]``.
        scale: score scale, default ``K ** -0.5``.
        initial_state: ``[N, H, K, V]`` or None.
        output_final_state: also return the final state ``[N, H, K, V]`` (fp32).
    Returns:
        ``(o [T, H, V], final_state or None)``.
    """
    if initial_state is not None and initial_state.shape[0] != len(cu_seqlens) - 1:
        raise ValueError(
            f"The number of initial states is expected to be equal to the number of input sequences, "
            f"i.e., {len(cu_seqlens) - 1} rather than {initial_state.shape[0]}."
        )
    if scale is None:
        scale = q.shape[-1] ** -0.5
    return ChunkGLAFunction.apply(q, k, v, g, scale, initial_state, output_final_state, cu_seqlens)
