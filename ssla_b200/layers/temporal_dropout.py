"""Temporal dropout (layers/temporal_dropout.py:6-59): of each sequence of length L keep
ceil(L / w) events, every w-th counted back from the last (the last event is always kept)."""
from __future__ import annotations

import torch

from ..ops.segment import gather_rows_ad
from .async_sparse_module import AsyncSparseModule

_ROW_DTYPES = (torch.float32, torch.bfloat16, torch.float16)


class TemporalDropout(AsyncSparseModule):
    def __init__(self, window_size, *args, **kwargs):
        super().__init__(*args, **kwargs)
        if window_size <= 0:
            raise ValueError("window_size must be greater than 0.")
        self.window_size = window_size

    def forward(self, inputs, grouped_events=True):
        inputs = self.prepare_inputs(inputs, grouped_events)
        lengths = inputs["lengths"]
        w = self.window_size
        dev = lengths.device
        with torch.no_grad():
            start = torch.cumsum(lengths, 0) - lengths
            keep_n = torch.div(lengths + (w - 1), w, rounding_mode="floor")
            kend = torch.cumsum(keep_n, 0)
            total = int(kend[-1]) if kend.numel() else 0  # the one host read: output size
            seq = torch.repeat_interleave(torch.arange(lengths.numel(), device=dev), keep_n, output_size=total)
            kstart = kend - keep_n
            j = torch.arange(total, device=dev) - kstart[seq]
            first = torch.remainder(lengths - 1, w)  # offset of the first kept event
            idx = start[seq] + first[seq] + j * w
        ev = inputs["events"]
        kept = gather_rows_ad(ev, idx) if (ev.dim() == 2 and ev.is_cuda and ev.dtype in _ROW_DTYPES) else ev[idx]
        return {"events": kept, "time": inputs["time"][idx], "lengths": keep_n,
                "batch_id": inputs["batch_id"], "h": inputs["h"], "w": inputs["w"],
                "batch_size": inputs["batch_size"]}
