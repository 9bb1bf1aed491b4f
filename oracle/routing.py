"""CPU restatement of the reference's pixel grouping (test infrastructure only).

``group_events`` follows utils/farsecnn_utils.py:130-174 (stable sort of the events by
(sample, pixel) id, unique_consecutive, the last ``max_events_per_px`` events of each pixel);
``preprocess`` follows MosModel.preprocess_inputs (model_mos.py:173-209): the duplicated
timestamp becomes the per-pixel delay min((t - t_prev) / 1e5, 1) with 1 at each pixel's first
event, then truncate_packed_sequence (utils/farsecnn_utils.py:8-33) keeps the first
``hot_pixel_thres`` events of every pixel.
"""
from __future__ import annotations

import torch


def group_events(events, lengths, frame_size, max_events_per_px=512):
    events = events.float()
    B, Nmax, C = events.shape
    H, W = int(frame_size[0]), int(frame_size[1])
    mask = torch.arange(Nmax).unsqueeze(0) < lengths.unsqueeze(1)
    ev = events[mask]
    batch_id = torch.arange(B).repeat_interleave(lengths)
    ids = batch_id * H * W + ev[:, 1].long() * W + ev[:, 0].long()
    order = torch.sort(ids, stable=True)[1]
    uniq, inv, counts = ids[order].unique_consecutive(return_inverse=True, return_counts=True)
    skip = (counts - max_events_per_px).clamp(min=0)
    kept_len = counts.clamp(max=max_events_per_px)
    start = torch.cumsum(counts, 0) - counts
    rows = torch.cat([torch.arange(int(s + k), int(s + c)) for s, k, c in zip(start, skip, counts)]) \
        if len(counts) else torch.zeros(0, dtype=torch.int64)
    sel = ev[order][rows]
    return {
        "events": sel[:, 3:], "time": sel[:, 2].long(), "batch_id": uniq // (H * W), "h": (uniq % (H * W)) // W,
        "w": uniq % W, "lengths": kept_len, "batch_size": B,
    }


def preprocess(events, lengths, frame_size, hot_pixel_thres=50):
    x = torch.cat([events[..., :3], events[..., 2:3], events[..., 3:]], dim=-1)
    g = group_events(x, lengths, frame_size)
    t = g["events"][:, 0].clone()
    dt = torch.empty_like(t)
    if t.numel():
        dt[0] = t[0]
        dt[1:] = t[1:] - t[:-1]
    dt = torch.clamp(dt / torch.full_like(dt, 1e5), max=1)
    first = torch.cumsum(g["lengths"], 0) - g["lengths"]
    dt[first] = 1
    feats = g["events"].clone()
    feats[:, 0] = dt
    if hot_pixel_thres > 0:
        starts = torch.cumsum(g["lengths"], 0) - g["lengths"]
        pos = torch.arange(feats.shape[0]) - torch.repeat_interleave(starts, g["lengths"])
        keep = pos < hot_pixel_thres
        feats, g["time"] = feats[keep], g["time"][keep]
        g["lengths"] = g["lengths"].clamp(max=hot_pixel_thres)
    g["events"] = feats
    return g
