"""Base module of the receptive-field layers (layers/async_sparse_module.py:8-45): holds the
frame geometry and look-up tables as buffers of the same names."""
from __future__ import annotations

import torch
import torch.nn as nn

from ..utils.farsecnn_utils import compute_rf2pixels, gather_receptive_fields, group_events


class AsyncSparseModule(nn.Module):
    def __init__(self, frame_size, kernel_size=(1, 1), stride=(1, 1), max_events_per_rf=512):
        super().__init__()
        self.frame_size = frame_size
        self.kernel_size = kernel_size
        self.stride = stride
        self.register_buffer("max_events_per_rf", torch.tensor(max_events_per_rf))
        rf2pixel_lut, rf_outcoord = compute_rf2pixels(self.frame_size, self.kernel_size, self.stride)
        self.register_buffer("rf2pixel_lut", rf2pixel_lut)
        self.register_buffer("rf_outcoord", rf_outcoord)
        out_max = rf_outcoord.max(dim=0)[0].tolist()  # <x, y>
        self.frame_output_size = (out_max[1] + 1, out_max[0] + 1)

    def prepare_inputs(self, inputs, grouped_events):
        if not grouped_events:
            inputs = self.group_events(inputs)
        if not (self.kernel_size[0] == 1 and self.kernel_size[1] == 1 and self.stride[0] == 1 and self.stride[1] == 1):
            inputs = self.gather_receptive_fields(inputs)
        return inputs

    def group_events(self, inputs):
        with torch.no_grad():
            return group_events(inputs, self.frame_size)

    def gather_receptive_fields(self, inputs):
        return gather_receptive_fields(inputs, self.frame_size, self.rf2pixel_lut, self.rf_outcoord,
                                       kernel_size=self.kernel_size, stride=self.stride)

    def compute_flops(self, inputs, grouped_events=True):
        return 0
