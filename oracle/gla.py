"""CPU restatements of the reference GLA algorithms (test infrastructure only).

* ``naive_gla_recurrent``  — ops/gla/naive.py:50-111 (token recurrence, fp32 state);
  ``naive_gla_recurrent_step`` the same for one token of many sequences at once.
* ``naive_gla_parallel``   — ops/gla/naive.py:6-47 (O(T^2) parallel form).
* ``naive_gla_recurrent_scalar`` — ops/gla/naive_scalar.py:7-66.
* ``chunk_gla_ref``        — the chunked algorithm of ops/gla/chunk.py:906-960 evaluated in
  float64 (chunk states as in ops/common/chunk_h_naive.py:16-91); differentiable, used as the
  reference for large shapes where the token loop is too slow.
* ``scan_ref`` / ``scan_ref_bwd`` — ops/common/scan.py:35-43 and :71-86.
"""
from __future__ import annotations

import torch


def naive_gla_recurrent(q, k, v, g, cu_seqlens, scale=None, initial_state=None, output_final_state=False):
    """Token recurrence of ops/gla/naive.py:50-111: per step S = exp(g) * S + k v^T (:95), then
    o = (q * scale)^T S (:97-98); state and final state fp32, o in q's dtype."""
    T, H, K = q.shape
    V = v.shape[-1]
    dtype = q.dtype
    if scale is None:
        scale = K ** -0.5
    outs, finals = [], []
    cu = [int(x) for x in cu_seqlens.tolist()]
    for n in range(len(cu) - 1):
        b, e = cu[n], cu[n + 1]
        qn, kn, vn, gn = (x[b:e].to(torch.float32) for x in (q, k, v, g))
        S = torch.zeros(H, K, V, dtype=torch.float32, device=q.device)
        if initial_state is not None:
            S = S + initial_state[n].to(torch.float32)
        on = []
        for t in range(e - b):
            S = torch.exp(gn[t])[:, :, None] * S + kn[t][:, :, None] * vn[t][:, None, :]
            on.append(torch.einsum("hk,hkv->hv", qn[t] * scale, S).to(dtype))
        outs.append(torch.stack(on, 0) if on else q.new_zeros((0, H, V), dtype=dtype))
        finals.append(S)
    o = torch.cat(outs, 0) if outs else q.new_zeros((0, H, V))
    return o, (torch.stack(finals, 0) if output_final_state else None)


def naive_gla_recurrent_step(q, k, v, g, state, scale=None):
    """One token of every sequence through the recurrence of ops/gla/naive.py:50-111 (state
    update :95, read-out :97-98), vectorised over the sequences: q, k, g [N, H, K], v [N, H, V],
    state [N, H, K, V] fp32 -> (o [N, H, V] in q's dtype, new state fp32).  Equal to
    ``naive_gla_recurrent`` on N sequences of one token each (tests/test_oracle.py)."""
    K = q.shape[-1]
    if scale is None:
        scale = K ** -0.5
    qf, kf, vf, gf = (x.to(torch.float32) for x in (q, k, v, g))
    S = torch.exp(gf)[..., None] * state.to(torch.float32) + kf[..., None] * vf[..., None, :]
    o = torch.einsum("nhk,nhkv->nhv", qf * scale, S).to(q.dtype)
    return o, S


def naive_gla_parallel(q, k, v, g, cu_seqlens, scale=None):
    """Parallel form of ops/gla/naive.py:6-47 (A = (q k^T) with exp(cumsum) decay, causal)."""
    T, H, K = q.shape
    dtype = q.dtype
    if scale is None:
        scale = K ** -0.5
    outs = []
    cu = [int(x) for x in cu_seqlens.tolist()]
    for n in range(len(cu) - 1):
        b, e = cu[n], cu[n + 1]
        qn, kn, gn, vn = (x[b:e].to(torch.float32).transpose(0, 1) for x in (q, k, g, v))
        Tn = qn.shape[1]
        gc = torch.cumsum(gn, dim=1)
        A = (qn[:, :, None, :] * kn[:, None, :, :] * torch.exp(gc[:, :, None, :] - gc[:, None, :, :])).sum(-1)
        A = A * scale
        A = A.masked_fill(~torch.tril(torch.ones(Tn, Tn, dtype=torch.bool)), 0)
        outs.append(torch.matmul(A, vn).transpose(0, 1).to(dtype))
    return torch.cat(outs, 0)


def naive_gla_recurrent_scalar(q, k, v, g, cu_seqlens, scale=None, initial_state=None, output_final_state=False):
    """ops/gla/naive_scalar.py:7-66: S = exp(g) S + k v; o = (q * scale) S; scale default 1.0."""
    T, H = q.shape
    dtype = q.dtype
    if scale is None:
        scale = 1.0
    outs, finals = [], []
    cu = [int(x) for x in cu_seqlens.tolist()]
    for n in range(len(cu) - 1):
        b, e = cu[n], cu[n + 1]
        qn, kn, vn, gn = (x[b:e].to(torch.float32) for x in (q, k, v, g))
        S = torch.zeros(H, dtype=torch.float32)
        if initial_state is not None:
            S = S + initial_state[n].to(torch.float32)
        on = []
        for t in range(e - b):
            S = torch.exp(gn[t]) * S + kn[t] * vn[t]
            on.append((qn[t] * scale * S).to(dtype))
        outs.append(torch.stack(on, 0) if on else q.new_zeros((0, H)))
        finals.append(S)
    o = torch.cat(outs, 0)
    return o, (torch.stack(finals, 0) if output_final_state else None)


def chunk_gla_ref(q, k, v, g, cu_seqlens, scale=None, initial_state=None, output_final_state=False,
                  chunk_size=64, dtype=torch.float64):
    """Chunked GLA in float64 on the CPU (differentiable through autograd).

    Per 64-token chunk with in-chunk cumulative log decay gc and chunk-start state h
    (ops/gla/chunk.py:906-960, ops/common/chunk_h.py:13-128):
        o   = scale (q exp(gc)) h + tril(scale (q exp(gc)) (k exp(-gc))^T) v
        h'  = exp(gc_last) h + (k exp(gc_last - gc))^T v
    The factorisation exp(gc_i - gc_j) = exp(gc_i) exp(-gc_j) is exact in float64 as long as
    |gc| stays far from the float64 exponent range, which the test inputs guarantee (asserted).
    Returns (o in q's dtype, final state fp32 or None)."""
    T, H, K = q.shape
    V = v.shape[-1]
    if scale is None:
        scale = K ** -0.5
    out_dtype = q.dtype
    qd, kd, vd, gd = (x.to(dtype) for x in (q, k, v, g))
    cu = [int(x) for x in cu_seqlens.tolist()]
    outs, finals = [], []
    for n in range(len(cu) - 1):
        b, e = cu[n], cu[n + 1]
        h = torch.zeros(H, K, V, dtype=dtype)
        if initial_state is not None:
            h = h + initial_state[n].to(dtype)
        for c0 in range(b, e, chunk_size):
            c1 = min(c0 + chunk_size, e)
            qc, kc, vc, gcum = qd[c0:c1], kd[c0:c1], vd[c0:c1], torch.cumsum(gd[c0:c1], 0)
            assert float(gcum.detach().abs().max()) < 600.0, "decay range too large for the float64 factorisation"
            L = c1 - c0
            qe = qc * torch.exp(gcum) * scale          # [L,H,K]
            ke = kc * torch.exp(-gcum)
            A = torch.einsum("ihk,jhk->hij", qe, ke)
            A = A * torch.tril(torch.ones(L, L, dtype=dtype))
            o = torch.einsum("ihk,hkv->ihv", qe, h) + torch.einsum("hij,jhv->ihv", A, vc)
            outs.append(o)
            gl = gcum[-1]                               # [H,K]
            kl = kc * torch.exp(gl[None] - gcum)
            h = torch.exp(gl)[:, :, None] * h + torch.einsum("jhk,jhv->hkv", kl, vc)
        finals.append(h)
    o = torch.cat(outs, 0).to(out_dtype) if outs else q.new_zeros((0, H, V))
    ht = torch.stack(finals, 0).to(torch.float32) if output_final_state else None
    return o, ht


def scan_ref(u, g, cu_seqlens):
    """ops/common/scan.py:35-43: h = h * g + u in fp32 per step (two roundings), h in u's dtype."""
    uf, gf = u.to(torch.float32), g.to(torch.float32)
    h = torch.zeros_like(uf)
    cu = [int(x) for x in cu_seqlens.tolist()]
    for n in range(len(cu) - 1):
        b, e = cu[n], cu[n + 1]
        acc = torch.zeros(u.shape[1], dtype=torch.float32)
        for t in range(b, e):
            acc = acc * gf[t] + uf[t]
            h[t] = acc
    return h.to(u.dtype)


def scan_ref_vectorized(u, g, cu_seqlens):
    """Same operation order as ``scan_ref`` (so bit-identical in fp32), vectorised over
    sequences by stepping all sequences' t-th tokens together; fast for many short sequences."""
    uf, gf = u.to(torch.float32), g.to(torch.float32)
    cu = cu_seqlens.to(torch.int64)
    lens = cu[1:] - cu[:-1]
    h = torch.zeros_like(uf)
    if uf.shape[0] == 0 or lens.numel() == 0:
        return h.to(u.dtype)
    acc = torch.zeros(lens.numel(), u.shape[1], dtype=torch.float32)
    for t in range(int(lens.max())):
        act = lens > t
        rows = cu[:-1][act] + t
        acc[act] = acc[act] * gf[rows] + uf[rows]
        h[rows] = acc[act]
    return h.to(u.dtype)


def scan_ref_bwd(do, g, h, cu_seqlens):
    """ops/common/scan.py:71-86: dh += do; dg = dh * h_{t-1} (0 at t=0); du = dh; dh *= g."""
    dof, gf, hf = do.to(torch.float32), g.to(torch.float32), h.to(torch.float32)
    du = torch.zeros_like(dof)
    dg = torch.zeros_like(gf)
    cu = [int(x) for x in cu_seqlens.tolist()]
    for n in range(len(cu) - 1):
        b, e = cu[n], cu[n + 1]
        dh = torch.zeros(do.shape[1], dtype=torch.float32)
        for t in range(e - 1, b - 1, -1):
            dh = dh + dof[t]
            hm1 = hf[t - 1] if t > b else torch.zeros_like(dh)
            dg[t] = dh * hm1
            du[t] = dh
            dh = dh * gf[t]
    return du.to(h.dtype), dg.to(g.dtype)


def scan_ref_bwd_vectorized(do, g, h, cu_seqlens):
    """Vectorised over sequences with ``scan_ref_bwd``'s operation order."""
    dof, gf, hf = do.to(torch.float32), g.to(torch.float32), h.to(torch.float32)
    cu = cu_seqlens.to(torch.int64)
    lens = cu[1:] - cu[:-1]
    du = torch.zeros_like(dof)
    dg = torch.zeros_like(gf)
    if dof.shape[0] == 0 or lens.numel() == 0:
        return du.to(h.dtype), dg.to(g.dtype)
    dh = torch.zeros(lens.numel(), do.shape[1], dtype=torch.float32)
    for t in range(int(lens.max()) - 1, -1, -1):
        act = lens > t
        rows = cu[:-1][act] + t
        d = dh[act] + dof[rows]
        prev = hf[rows - 1] if t > 0 else torch.zeros_like(d)
        dg[rows] = d * prev
        du[rows] = d
        dh[act] = d * gf[rows]
    return du.to(h.dtype), dg.to(g.dtype)
