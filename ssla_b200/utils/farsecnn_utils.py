"""Receptive-field routing with the interface of the reference's utils/farsecnn_utils.py."""
from __future__ import annotations

import math

import torch

from ..ops import segment as _seg
from .routing import _geometry, compute_padding_1d, group_events, receptive_field_lut, replicate_to_fields, truncate_packed_sequence

__all__ = ["compute_padding_1d", "compute_output_size_1d", "compute_rf2pixels", "group_events",
           "gather_receptive_fields", "truncate_packed_sequence"]


def compute_output_size_1d(padded_in_size, kernel_size, stride):
    return math.floor((padded_in_size - kernel_size) / stride + 1)


def compute_rf2pixels(frame_size, kernel_size, stride):
    """(rf2pixel LUT [n_rf, kh*kw] with -1 padding, output coords [n_rf, 2] <x, y>)
    (utils/farsecnn_utils.py:95-128)."""
    return receptive_field_lut(frame_size, kernel_size, stride)


def gather_receptive_fields(inputs, frame_size, rf2pixel_lut, rf_outcoord, kernel_size=None, stride=None):
    """Pixel groups -> non-empty receptive fields with their time-ordered events
    (utils/farsecnn_utils.py:177-265).  Kernel and stride default to the values implied by the
    look-up tables (square kernels with stride = kernel, the pooling configuration)."""
    n_rf = rf_outcoord.shape[0]
    if kernel_size is None:
        k = int(round(rf2pixel_lut.shape[1] ** 0.5))
        kernel_size = (k, k)
    if stride is None:
        stride = kernel_size
    ow = _geometry(frame_size, kernel_size, stride)[-1]
    r = replicate_to_fields(inputs["batch_id"], inputs["h"], inputs["w"], inputs["lengths"], inputs["time"],
                            frame_size, kernel_size, stride, batch_size=inputs.get("batch_size"))
    fid = r["field_id"]
    f = fid % n_rf
    return {
        "events": _seg.gather_rows_ad(inputs["events"], r["src"]),
        "time": r["time"],
        "pos_id": r["pos_id"],
        "lengths": r["lengths"],
        "h": f // ow,
        "w": f % ow,
        "batch_id": fid // n_rf,
        "batch_size": inputs["batch_size"],
    }
