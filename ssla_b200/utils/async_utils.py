"""MoS-attention routing with the interface of the reference's utils/async_utils.py."""
from __future__ import annotations

from typing import Dict, Tuple

import torch

from ..ops import segment as _seg
from .routing import group_events as _group_events
from .routing import receptive_field_lut, replicate_to_fields


def group_events(inputs, frame_size: Tuple[int, int], max_events_per_px: int = 512) -> Dict[str, torch.Tensor]:
    """utils/async_utils.py:10-84 (asserts of the reference kept)."""
    assert isinstance(inputs, tuple) and len(inputs) == 2, "inputs should be a tuple of (events, lengths)"
    assert isinstance(frame_size, tuple) and len(frame_size) == 2, "frame_size should be a tuple of (H, W)"
    events, lengths = inputs
    assert events.dim() == 3 and events.size(2) >= 4, "events should be a (B, N, C) tensor"
    assert lengths.dim() == 1 and lengths.size(0) == events.size(0), "lengths should be a (B,) tensor"
    return _group_events(inputs, frame_size, max_events_per_px)


def get_patch2pixel_lut(frame_size, kernel_size, stride) -> torch.Tensor:
    """[num_patches, kh*kw] pixel ids with -1 padding, 'same' padding (utils/async_utils.py:96-122)."""
    return receptive_field_lut(frame_size, kernel_size, stride)[0]


def scatter_group_events_to_patch(pixel_inputs: Dict[str, torch.Tensor], frame_size, patch2pixel_lut,
                                  kernel_size=None, stride=(1, 1)) -> Dict[str, torch.Tensor]:
    """Pixel-grouped events -> per-patch time-ordered event sequences
    (utils/async_utils.py:125-240).  Returns events, pos_id, lengths, batch_size, orig_event_idx.
    The kernel size is read from the look-up table (square kernels, as the reference builds)
    unless given."""
    if kernel_size is None:
        k = int(round(patch2pixel_lut.shape[1] ** 0.5))
        kernel_size = (k, k)
    r = replicate_to_fields(pixel_inputs["batch_id"], pixel_inputs["h"], pixel_inputs["w"],
                            pixel_inputs["lengths"], pixel_inputs["time"], frame_size, kernel_size, stride,
                            batch_size=pixel_inputs.get("batch_size"))
    return {
        "events": _seg.gather_rows_ad(pixel_inputs["events"], r["src"]),
        "pos_id": r["pos_id"],
        "lengths": r["lengths"],
        "batch_size": pixel_inputs["batch_size"],
        "orig_event_idx": r["src"],
    }


def gather_patch_events_to_group(patch_events: torch.Tensor, patch_event_to_pixel_event_idx: torch.Tensor,
                                 num_pixel_events: int) -> torch.Tensor:
    """Sum patch-level rows back onto their pixel events (utils/async_utils.py:243-264):
    zeros(E, C) fp32 index_add_, here with a fixed ascending-source summation order."""
    return _seg.index_add_rows_ad(patch_events.float(), patch_event_to_pixel_event_idx, int(num_pixel_events))
