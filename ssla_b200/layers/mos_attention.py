"""MoS attention (layers/mos_attention.py:12-199): pixel events are replicated into the kxk
patches around them, projected per patch position, run through the gated scan along each
patch's time-ordered event sequence, projected back per position and summed onto their pixel
events, then residual + LayerNorm.  Parameter and buffer names match the reference so its
state_dicts load unchanged.

Per-position projections without masks: a pixel event sits at a given position of exactly one
patch, so
  * scatter projection: Y_j = x W_j^T for all positions j is one batched GEMM over the pixel
    events, and the patch rows are the gather Y[pos, src] (the routing gather itself);
  * gather projection + gather-back: out[e] = sum_j W_j o[row(e, j)] is one GEMM of the
    [E, positions * C] buffer of patch outputs (deterministic scatter, zeros where a position
    has no patch) with the concatenated weights.
The reference does 9 boolean-masked F.linear calls per projection and an atomics-based
index_add_ (layers/mos_attention.py:148-167, utils/async_utils.py:262-263).  GPU work:
routing (ssla_b200.utils.routing), GEMMs (cuBLAS; in the inference path the split-TF32
tensor-core GEMM of ``csrc/gemm_tf32.cu``), the scan (``ssla_scan_fwd/bwd``) and row
gathers (``ssla_gather_rows``)."""
from __future__ import annotations

import math
from typing import Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..ops import mos as _mos
from ..ops.common.scan import scan
from ..ops.segment import gather_rows_ad, index_add_rows_ad
from ..utils.async_utils import get_patch2pixel_lut
from ..utils.routing import replicate_to_fields


def _per_position_linear(x: torch.Tensor, pos_id: torch.Tensor, weights: torch.Tensor, out_features: int):
    """y[r] = weights[pos_id[r]] @ x[r] (weights [P, out, in]); rows are grouped by position so
    each position is one GEMM."""
    P = weights.shape[0]
    out = torch.empty((x.shape[0], out_features), device=x.device, dtype=torch.float32)
    if P == 1:
        return F.linear(x, weights[0])
    order = torch.sort(pos_id, stable=True)[1]
    counts = torch.bincount(pos_id, minlength=P).tolist()
    start = 0
    for i, n in enumerate(counts):
        if n:
            rows = order[start:start + n]
            out[rows] = F.linear(x[rows], weights[i])
        start += n
    return out


class MosAttention(nn.Module):
    def __init__(self, input_size: int, hidden_size: int, frame_size: Tuple[int, int], kernel_size: Tuple[int, int],
                 stride: Tuple[int, int] = (1, 1), scatter_proj: bool = True, gather_proj: bool = True):
        super().__init__()
        self.input_size = input_size
        self.hidden_size = hidden_size
        self.frame_size = frame_size
        self.frame_output_size = frame_size
        self.kernel_size = kernel_size
        self.stride = stride
        self.scatter_proj = scatter_proj
        self.gather_proj = gather_proj
        n_pos = kernel_size[0] * kernel_size[1]
        self.register_parameter("scatter_conv_weights", nn.Parameter(
            torch.zeros([n_pos if scatter_proj else 1, input_size * hidden_size], dtype=torch.float32)))
        self.register_parameter("gather_conv_weights", nn.Parameter(
            torch.zeros([n_pos if gather_proj else 1, hidden_size * hidden_size], dtype=torch.float32)))
        self._initialize_weights()
        self.q_proj = nn.Linear(hidden_size, hidden_size, bias=False)
        self.v_proj = nn.Linear(hidden_size, hidden_size, bias=False)
        self.g_proj = nn.Linear(hidden_size, hidden_size, bias=False)
        self.o_proj = nn.Linear(hidden_size, hidden_size, bias=False)
        self.norm = nn.LayerNorm(hidden_size)
        lut = get_patch2pixel_lut(frame_size, kernel_size, stride)
        self.register_buffer("patch2pixel_lut", lut)
        self.register_buffer("patch_outcoord", torch.zeros([lut.shape[0], 2], dtype=torch.int))
        self.input_proj = nn.Linear(input_size, hidden_size, bias=False) if input_size != hidden_size else None

    @torch.no_grad()
    def _initialize_weights(self):
        std = math.sqrt(2.0 / (self.input_size + self.hidden_size))  # Xavier
        self.scatter_conv_weights.normal_(0, std)
        self.gather_conv_weights.normal_(0, std)

    def forward(self, inputs):
        residual = inputs["events"]
        if residual.shape[0] != inputs["time"].shape[0]:
            raise ValueError("events and time must have one row per event")
        r = replicate_to_fields(inputs["batch_id"], inputs["h"], inputs["w"], inputs["lengths"], inputs["time"],
                                self.frame_size, tuple(self.kernel_size), tuple(self.stride),
                                batch_size=inputs.get("batch_size"))
        src, pos_id = r["src"], r["pos_id"]
        E = residual.shape[0]
        C = self.hidden_size
        if not torch.is_grad_enabled() and residual.dtype == torch.float32 and C % 4 == 0:
            return self._forward_fused(inputs, residual, r)
        # scatter projection: all positions at once on the pixel events, then the routing gather
        ws = self.scatter_conv_weights.reshape(-1, C, self.input_size)
        P = ws.shape[0]
        y = torch.matmul(residual.unsqueeze(0), ws.transpose(1, 2))  # [P, E, C]
        key = src if P == 1 else pos_id * E + src
        x = gather_rows_ad(y.reshape(P * E, C), key)
        q = self.q_proj(x)
        v = self.v_proj(x)
        g = torch.sigmoid(self.g_proj(x))
        lengths = r["lengths"]
        cu = torch.zeros(lengths.numel() + 1, dtype=torch.int64, device=lengths.device)
        cu[1:] = lengths.cumsum(0)
        h = scan(u=v, g=g, cu_seqlens=cu)
        o = self.o_proj(q * h)
        # gather projection + gather-back: [E, P, C] buffer of patch outputs, one GEMM
        wg = self.gather_conv_weights.reshape(-1, C, C)
        Pg = wg.shape[0]
        if Pg == 1:
            out = index_add_rows_ad(o, src, E) @ wg[0].t()
        else:
            z = torch.zeros((E * Pg, C), device=o.device, dtype=o.dtype)
            z = z.index_put((src * Pg + pos_id,), o)  # unique (event, position) pairs
            out = z.view(E, Pg * C) @ wg.permute(0, 2, 1).reshape(Pg * C, C)
        if self.input_proj is not None:
            residual = self.input_proj(residual)
        out = self.norm(out + residual)
        return {"events": out, "time": inputs["time"], "w": inputs["w"], "h": inputs["h"],
                "batch_id": inputs["batch_id"], "lengths": inputs["lengths"], "batch_size": inputs["batch_size"]}

    def _forward_fused(self, inputs, residual, r):
        """Inference path.  The q/v/g projections are folded into the per-position scatter
        weights ([Wq; Wv; Wg] Ws_p) and o_proj into the gather weights (Wg_p Wo), so the only
        per-patch-event work is one fused kernel: gather of the event's projected row (one GEMM
        over the pixel events computes all positions; when that buffer would be very large the
        projection runs inside the kernel from shared-memory weights instead), sigmoid gate,
        scan and q*h written into the [E, P*C] buffer; one GEMM over that buffer closes the
        layer."""
        src, pos_id = r["src"], r["pos_id"]
        E, C = residual.shape[0], self.hidden_size
        w_all, g_rows, g_back, g_in = self._folded_weights()
        P, Pg = w_all.shape[0], g_back.K // C
        lengths = r["lengths"]
        cu = torch.zeros(lengths.numel() + 1, dtype=torch.int64, device=lengths.device)
        cu[1:] = lengths.cumsum(0)
        rows = src.numel()
        if Pg == 1:
            qh = torch.empty((rows, C), device=residual.device, dtype=torch.float32)
        else:
            qh = torch.zeros((E * Pg, C), device=residual.device, dtype=torch.float32)
        if _mos.use_patch_scan_proj(E, P, C, self.input_size):
            # projection inside the scan kernel (weights in shared memory): no [E, P*3C] buffer
            dst = torch.arange(rows, device=residual.device) if Pg == 1 else src * Pg + pos_id
            _mos.patch_scan_proj(residual, w_all, src, pos_id if P > 1 else torch.zeros_like(src), dst, cu, qh)
        else:
            y = g_rows(residual)  # rows (e, p) of 3C
            # key = src * P + pos and dst = src * Pg + pos (unique (event, position) pairs), or the
            # patch event's own row when Pg == 1, are formed inside the kernel
            _mos.patch_scan_routed(y.view(-1, 3 * C), src, pos_id if (P > 1 or Pg > 1) else None, P,
                                   0 if Pg == 1 else Pg, cu, C, qh)
        if Pg == 1:
            out = g_back(index_add_rows_ad(qh, src, E))
        else:
            out = g_back(qh.view(E, Pg * C))
        if self.input_proj is not None:
            residual = g_in(residual)
        out = _mos.layernorm_residual(out, residual, self.norm.weight, self.norm.bias, self.norm.eps)
        return {"events": out, "time": inputs["time"], "w": inputs["w"], "h": inputs["h"],
                "batch_id": inputs["batch_id"], "lengths": inputs["lengths"], "batch_size": inputs["batch_size"]}

    def _folded_weights(self):
        """Folded inference weights: w_all [P, 3C, I] = [Wq; Wv; Wg] Ws_p, and as GEMM operands
        (``RowsGemm``) its [I, P*3C] form, the gather-back operand [Pg*C, C] (row block p =
        (Wg_p Wo)^T) and the input projection (None without one).  Recomputed only when a
        parameter changed (tensor version counters) or moved."""
        params = (self.scatter_conv_weights, self.gather_conv_weights, self.q_proj.weight, self.v_proj.weight,
                  self.g_proj.weight, self.o_proj.weight) + (
                      (self.input_proj.weight,) if self.input_proj is not None else ())
        key = tuple((p.data_ptr(), p._version) for p in params)
        cached = getattr(self, "_folded", None)
        if cached is not None and cached[0] == key:
            return cached[1:]
        C = self.hidden_size
        ws = self.scatter_conv_weights.reshape(-1, C, self.input_size)
        wqvg = torch.cat([self.q_proj.weight, self.v_proj.weight, self.g_proj.weight], 0)  # [3C, C]
        w_all = torch.matmul(wqvg, ws).contiguous()
        wgo = torch.matmul(self.gather_conv_weights.reshape(-1, C, C), self.o_proj.weight)  # [Pg, C, C]
        g_rows = _mos.RowsGemm(w_all.reshape(-1, self.input_size).t())
        g_back = _mos.RowsGemm(wgo.permute(0, 2, 1).reshape(-1, C))
        g_in = _mos.RowsGemm(self.input_proj.weight.t()) if self.input_proj is not None else None
        self._folded = (key, w_all, g_rows, g_back, g_in)
        return w_all, g_rows, g_back, g_in

    def _apply_scatter_proj(self, x, pos_id):
        w = self.scatter_conv_weights.reshape(-1, self.hidden_size, self.input_size)
        return _per_position_linear(x, pos_id, w, self.hidden_size)

    def _apply_gather_proj(self, x, pos_id):
        w = self.gather_conv_weights.reshape(-1, self.hidden_size, self.hidden_size)
        return _per_position_linear(x, pos_id, w, self.hidden_size)

    def compute_flops(self, inputs):
        E = inputs["events"].shape[0]
        P = E * self.kernel_size[0] * self.kernel_size[1]
        C, I = self.hidden_size, self.input_size
        flops = P * C * (2 * I - 1) + 3 * P * C * (2 * C - 1) + P * C * 4 + P * C * 2 + P * C
        flops += P * C * (2 * C - 1) * 2 + P * C
        flops += E * C * (2 * I - 1) if self.input_proj is not None else 0
        flops += E * C + E * (8 * C + 1)
        return flops
