"""Linear attention over whole per-sample event streams (layers/linear_attention.py:11-102):
events of each sample are ordered by time (stable), run through the gated scan as one sequence
per non-empty sample, and scattered back to their group order."""
from __future__ import annotations

from typing import Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..ops.common.scan import scan


class LinearAttention(nn.Module):
    def __init__(self, input_size: int, hidden_size: int, frame_size: Tuple[int, int]):
        super().__init__()
        self.input_size = input_size
        self.hidden_size = hidden_size
        self.frame_size = frame_size
        self.frame_output_size = frame_size
        self.q_proj = nn.Linear(hidden_size, hidden_size, bias=False)
        self.v_proj = nn.Linear(hidden_size, hidden_size, bias=False)
        self.g_proj = nn.Linear(hidden_size, hidden_size, bias=False)
        self.o_proj = nn.Linear(hidden_size, hidden_size, bias=False)
        self.norm = nn.LayerNorm(hidden_size)
        if input_size != hidden_size:
            self.input_proj = nn.Linear(input_size, hidden_size, bias=False)
            self.residual_proj = nn.Linear(input_size, hidden_size, bias=False)
        else:
            self.input_proj = None
            self.residual_proj = None

    def forward(self, inputs):
        x_in = inputs["events"]
        t = inputs["time"]
        B = inputs["batch_size"]
        x = self.input_proj(x_in) if self.input_proj is not None else x_in
        ev_batch = inputs["batch_id"].repeat_interleave(inputs["lengths"])
        lengths = torch.bincount(ev_batch, minlength=B)
        by_time = torch.argsort(t, stable=True)
        order = by_time[torch.argsort(ev_batch[by_time], stable=True)]
        inv = torch.empty_like(order)
        inv[order] = torch.arange(order.numel(), device=order.device)
        xs = x[order]
        nz = lengths[lengths > 0]
        cu = torch.zeros(nz.numel() + 1, dtype=torch.int64, device=nz.device)
        cu[1:] = nz.cumsum(0)
        q = self.q_proj(xs)
        v = self.v_proj(xs)
        g = torch.sigmoid(self.g_proj(xs))
        h = scan(u=v, g=g, cu_seqlens=cu)
        o = self.o_proj(q * h)[inv]
        res = self.residual_proj(x_in) if self.residual_proj is not None else x_in
        out = self.norm(o + res)
        return {"events": out, "time": t, "w": inputs["w"], "h": inputs["h"], "batch_id": inputs["batch_id"],
                "lengths": inputs["lengths"], "batch_size": B}
