"""Sparse pooling (layers/sparse_pooling.py:8-103): events of a receptive field that share a
timestamp are merged by max or mean.

The merge is a segment reduction over rows that are already grouped: after the receptive-field
gather, rows are ordered by (field, time), so a segment opens at every field start and every
change of time, the running count of openings is a non-decreasing segment id, and the reduction
runs on ``ssla_segment_reduce`` with offsets from
``ssla_segment_offsets_sorted`` — no sort, no atomics, bit-exact against the CPU reduction
(the reference calls torch_scatter.scatter_max / scatter_mean, layers/sparse_pooling.py:33).
"""
from __future__ import annotations

import math

import torch

from ..ops import segment as _seg
from .async_sparse_module import AsyncSparseModule


class SparsePool(AsyncSparseModule):
    def __init__(self, op, *args, kernel_size=(1, 1), stride=None, **kwargs):
        stride = stride if stride else kernel_size
        super().__init__(*args, kernel_size=kernel_size, stride=stride, **kwargs)
        self.op = op

    def forward(self, inputs, grouped_events=True):
        inputs = self.prepare_inputs(inputs, grouped_events)
        lengths = inputs["lengths"]
        time = inputs["time"]
        events = inputs["events"]
        dev = time.device
        N = time.numel()
        # A row opens a segment where its time differs from the previous row's or where a
        # receptive field starts; segment ids are the running count of openings.
        ends = torch.cumsum(lengths.to(torch.int64), 0)
        starts = ends - lengths
        opens = torch.zeros(N + 1, dtype=torch.bool, device=dev)
        opens.index_fill_(0, starts, True)  # empty fields mark the next start (or the sentinel)
        opens = opens[:N]
        if N:
            opens[1:] |= time[1:] != time[:-1]
        cnt = torch.zeros(N + 1, dtype=torch.int64, device=dev)
        torch.cumsum(opens, 0, out=cnt[1:])
        seg = cnt[1:] - 1
        S = int(cnt[-1])  # the one host read of the layer: output size
        off = _seg.segment_offsets_sorted(seg, S)
        new_events = _seg.segment_reduce_ad(events, seg, off, None, self.op)
        new_time = time[off[:-1]]
        new_lengths = (cnt[ends] - cnt[starts]).to(lengths.dtype)
        return {"events": new_events, "time": new_time, "lengths": new_lengths, "batch_id": inputs["batch_id"],
                "h": inputs["h"], "w": inputs["w"], "batch_size": inputs["batch_size"]}

    def compute_flops(self, inputs, grouped_events=True, elementwise_agg_flops=0):
        x = self.prepare_inputs(inputs, grouped_events)
        lengths, time, events = x["lengths"], x["time"], x["events"]
        rf = torch.repeat_interleave(torch.arange(lengths.shape[0], device=time.device), lengths)
        key = time + rf * (time.max() + 1)
        agg_n = key.shape[0] - torch.unique_consecutive(key).shape[0]
        return agg_n * events.shape[-1] * elementwise_agg_flops


class SparseMaxPool(SparsePool):
    def __init__(self, *args, **kwargs):
        super().__init__(_seg.MAX, *args, **kwargs)

    def compute_flops(self, inputs, grouped_events=True):
        return super().compute_flops(inputs, grouped_events, elementwise_agg_flops=1)


class SparseAvgPool(SparsePool):
    def __init__(self, *args, **kwargs):
        super().__init__(_seg.MEAN, *args, **kwargs)

    def compute_flops(self, inputs, grouped_events=True):
        return super().compute_flops(inputs, grouped_events, elementwise_agg_flops=2)


class SparseAdaptiveMaxPool(SparseMaxPool):
    def __init__(self, frame_size, output_size):
        if output_size[0] > frame_size[0] or output_size[1] > frame_size[1]:
            raise ValueError("SparseAdaptiveMaxPool cannot be used to unpool the input frame.")
        kernel_size = [math.ceil(frame_size[0] / output_size[0]), math.ceil(frame_size[1] / output_size[1])]
        super().__init__(frame_size, kernel_size=kernel_size)


class SparseAdaptiveAvgPool(SparseAvgPool):
    def __init__(self, frame_size, output_size):
        if output_size[0] > frame_size[0] or output_size[1] > frame_size[1]:
            raise ValueError("SparseAdaptiveMaxPool cannot be used to unpool the input frame.")
        kernel_size = [math.ceil(frame_size[0] / output_size[0]), math.ceil(frame_size[1] / output_size[1])]
        super().__init__(frame_size, kernel_size=kernel_size)
