"""Sparse event routing on the GPU: pixel grouping, receptive-field / patch look-up tables and
the pixel -> patch (or receptive field) event replication used by MoS attention and sparse
pooling.

Semantics follow the reference (utils/async_utils.py:10-264, utils/farsecnn_utils.py:8-265):
the same dictionaries in and out, the same orderings and dtypes.  Where the reference uses an
unstable ``torch.sort`` to order the events of a patch by time (utils/async_utils.py:221-222,
utils/farsecnn_utils.py:246), ties are broken deterministically here by (look-up-table
position, event order), i.e. the order the reference builds before sorting.

On CUDA tensors ``replicate_to_fields`` runs the routing kernels of ``csrc/routing.cu``: a
dense pixel -> group map, per-field event counts, and a per-field merge of the time-ordered
pixel lists (no sort).  The PyTorch formulation below it (pairs expanded from the active
groups, ordered by (field, position), then a stable time sort) is kept for windows larger than
32 pixels and for groups whose events are not in time order; both give the same output.
"""
from __future__ import annotations

import math
from typing import Dict, Tuple

import torch

from .. import _lib


def compute_padding_1d(in_size: int, kernel_size: int, stride: int, mode: str = "same") -> int:
    """Total padding so that out = ceil(in / stride) ('same') or so that every input is covered
    at least once ('minimal') (utils/farsecnn_utils.py:67-73)."""
    if mode == "same":
        return math.ceil((math.ceil(in_size / stride) - 1) * stride + kernel_size - in_size)
    if mode == "minimal":
        return math.ceil((in_size - kernel_size) / stride) * stride - in_size + kernel_size
    raise ValueError(f"unknown padding mode {mode!r}")


def _geometry(frame_size, kernel_size, stride):
    H, W = int(frame_size[0]), int(frame_size[1])
    kh, kw = int(kernel_size[0]), int(kernel_size[1])
    sh, sw = int(stride[0]), int(stride[1])
    ph, pw = compute_padding_1d(H, kh, sh), compute_padding_1d(W, kw, sw)
    oh = (H + ph - kh) // sh + 1
    ow = (W + pw - kw) // sw + 1
    return H, W, kh, kw, sh, sw, ph // 2, pw // 2, oh, ow


def receptive_field_lut(frame_size, kernel_size, stride) -> Tuple[torch.Tensor, torch.Tensor]:
    """([oh*ow, kh*kw] pixel ids (y*W + x, -1 outside the frame), [oh*ow, 2] output coords <x, y>)
    with 'same' padding split floor/ceil before/after (utils/farsecnn_utils.py:95-128,
    utils/async_utils.py:96-122)."""
    H, W, kh, kw, sh, sw, pt, pl, oh, ow = _geometry(frame_size, kernel_size, stride)
    oy = torch.arange(oh).view(oh, 1, 1, 1)
    ox = torch.arange(ow).view(1, ow, 1, 1)
    dy = torch.arange(kh).view(1, 1, kh, 1)
    dx = torch.arange(kw).view(1, 1, 1, kw)
    y = oy * sh - pt + dy
    x = ox * sw - pl + dx
    inside = (y >= 0) & (y < H) & (x >= 0) & (x < W)
    lut = torch.where(inside, y * W + x, torch.full_like(y * W + x, -1)).reshape(oh * ow, kh * kw)
    outcoord = torch.stack(torch.meshgrid(torch.arange(ow), torch.arange(oh), indexing="xy"), -1)
    return lut.to(torch.int64), outcoord.reshape(oh * ow, 2).to(torch.int64)


def group_events(inputs, frame_size, max_events_per_px: int = 512, keep_first=None,
                 delay_col=None) -> Dict[str, torch.Tensor]:
    """Group events [B, N, C] (rows <x, y, t, features...>, per-sample lengths) by pixel
    (utils/farsecnn_utils.py:130-174, utils/async_utils.py:10-84): groups in ascending
    (sample, pixel) order, a group's events in input order, at most the last
    ``max_events_per_px`` events of a pixel kept.  With ``keep_first`` only the first
    ``keep_first`` of those are kept, which is the grouping followed by
    ``truncate_packed_sequence`` (model_mos.py:173-209) in one pass; with ``delay_col`` that
    feature column is replaced by the per-pixel delay min((t - t_prev) / 1e5, 1), 1 for a
    group's first event (model_mos.py:190-200).

    Runs the grouping kernels of ``csrc/group.cu`` (counts, scans, placement, per-pixel
    ordering; no sort) and reads the device once, for the group and kept-event counts."""
    events, lengths = inputs
    B, Nmax, C = events.shape
    H, W = int(frame_size[0]), int(frame_size[1])
    _lib.require_cuda(events, what="group_events")
    dev = events.device
    ev = events.float().contiguous()
    ln = lengths.to(device=dev, dtype=torch.int64).contiguous()
    L, st = _lib.load(), _lib.stream_of(ev)
    big = (1 << 62)
    kf = big if keep_first is None else int(keep_first)
    nb = L.ssla_group_events_workspace_bytes(B, Nmax, H, W)
    ws = torch.empty(max(nb, 1), device=dev, dtype=torch.uint8)
    totals = torch.empty(3, device=dev, dtype=torch.int32)
    _lib.check(L.ssla_group_events_count(ev.data_ptr(), B, Nmax, C, ln.data_ptr(), H, W, int(max_events_per_px), kf,
                                         ws.data_ptr(), nb, totals.data_ptr(), st), "group_events")
    _, G, K = totals.tolist()
    i64 = lambda n: torch.empty(n, device=dev, dtype=torch.int64)
    batch_id, gh, gw, glen, time = i64(G), i64(G), i64(G), i64(G), i64(K)
    feats = torch.empty((K, C - 3), device=dev, dtype=torch.float32)
    _lib.check(L.ssla_group_events_emit(ev.data_ptr(), B, Nmax, C, H, W, int(max_events_per_px), kf, ws.data_ptr(),
                                        G, K, -1 if delay_col is None else int(delay_col), batch_id.data_ptr(),
                                        gh.data_ptr(), gw.data_ptr(), glen.data_ptr(), time.data_ptr(),
                                        feats.data_ptr(), st), "group_events")
    return {
        "events": feats,
        "time": time,
        "batch_id": batch_id,
        "h": gh,
        "w": gw,
        "lengths": glen,
        "batch_size": B,
    }


def truncate_packed_sequence(data: torch.Tensor, seqlens: torch.Tensor, threshold: int, others=None):
    """Keep the first `threshold` rows of every packed sequence (utils/farsecnn_utils.py:8-33)."""
    dev = data.device
    starts = torch.cumsum(seqlens, 0) - seqlens
    pos = torch.arange(data.shape[0], device=dev) - torch.repeat_interleave(starts, seqlens)
    keep = pos < threshold
    new_lengths = seqlens.clamp(max=threshold)
    if others is not None:
        return data[keep], new_lengths, others[keep]
    return data[keep], new_lengths


def _replicate_gpu(gr_batch_id, gr_h, gr_w, gr_lengths, gr_time, geo, batch_size):
    """The routing kernels; None when they do not apply (the caller falls back)."""
    H, W, kh, kw, sh, sw, pt, pl, oh, ow = geo
    if kh * kw > 32 or not gr_lengths.is_cuda:
        return None
    dev = gr_lengths.device
    G = gr_lengths.numel()
    i64 = lambda t: t.to(torch.int64).contiguous()
    bid, hh, ww, glen, gtime = i64(gr_batch_id), i64(gr_h), i64(gr_w), i64(gr_lengths), i64(gr_time)
    B = int(batch_size) if batch_size is not None else (int(bid.max()) + 1 if G else 0)
    L, st = _lib.load(), _lib.stream_of(glen)
    gstart = torch.cumsum(glen, 0) - glen
    flags = torch.zeros(2, dtype=torch.int32, device=dev)  # [0] groups outside the frame, [1] unsorted times
    pmap = torch.full((max(B * H * W, 1),), -1, dtype=torch.int32, device=dev)
    _lib.check(L.ssla_route_pixel_map(bid.data_ptr(), hh.data_ptr(), ww.data_ptr(), G, B, H, W, pmap.data_ptr(),
                                      flags.data_ptr(), st), "route_pixel_map")
    _lib.check(L.ssla_route_groups_time_sorted(gstart.data_ptr(), glen.data_ptr(), gtime.data_ptr(), G,
                                               flags.data_ptr() + 4, st), "route_groups_time_sorted")
    flen = torch.empty(max(B * oh * ow, 1), dtype=torch.int64, device=dev)
    _lib.check(L.ssla_route_field_lengths(pmap.data_ptr(), glen.data_ptr(), B, H, W, kh, kw, sh, sw, pt, pl, oh, ow,
                                          flen.data_ptr(), st), "route_field_lengths")
    # non-empty fields in ascending id order with their lengths and event offsets (compaction
    # kernels), then the one host read of the routing: flags, field count and event count
    nf_all = B * oh * ow
    fid_buf = torch.empty(max(nf_all, 1), dtype=torch.int64, device=dev)
    len_buf = torch.empty(max(nf_all, 1), dtype=torch.int64, device=dev)
    off_buf = torch.empty(nf_all + 1, dtype=torch.int64, device=dev)
    stats = torch.empty(4, dtype=torch.int64, device=dev)
    nws = L.ssla_route_compact_fields_workspace_bytes(nf_all)
    ws = torch.empty(max(nws, 8), dtype=torch.uint8, device=dev)
    _lib.check(L.ssla_route_compact_fields(flen.data_ptr(), nf_all, flags.data_ptr(), fid_buf.data_ptr(),
                                           len_buf.data_ptr(), off_buf.data_ptr(), stats.data_ptr(), ws.data_ptr(),
                                           nws, st), "route_compact_fields")
    bad_coord, unsorted, F, n_ev = stats.tolist()
    if bad_coord or unsorted:
        return None
    field_ids, lengths, off = fid_buf[:F], len_buf[:F], off_buf[:F + 1]
    src = torch.empty(n_ev, dtype=torch.int64, device=dev)
    pos = torch.empty(n_ev, dtype=torch.int64, device=dev)
    t = torch.empty(n_ev, dtype=torch.int64, device=dev)
    _lib.check(L.ssla_route_fill(pmap.data_ptr(), gstart.data_ptr(), glen.data_ptr(), gtime.data_ptr(), B, H, W, kh,
                                 kw, sh, sw, pt, pl, oh, ow, field_ids.data_ptr(), off.data_ptr(), field_ids.numel(),
                                 src.data_ptr(), pos.data_ptr(), t.data_ptr(), st), "route_fill")
    return {"field_id": field_ids, "lengths": lengths.to(gr_lengths.dtype), "src": src, "pos_id": pos,
            "time": t.to(gr_time.dtype)}


def replicate_to_fields(
    gr_batch_id: torch.Tensor,
    gr_h: torch.Tensor,
    gr_w: torch.Tensor,
    gr_lengths: torch.Tensor,
    gr_time: torch.Tensor,
    frame_size,
    kernel_size,
    stride,
    batch_size=None,
):
    """Replicate the events of pixel groups into every receptive field (patch) containing the
    pixel, and order each field's events by time.

    Returns a dict with
      field_id   [F]  global field index b * num_fields + f of each non-empty field (ascending)
      lengths    [F]  events per non-empty field
      src        [P]  index into the group-ordered event array of each replicated event
      pos_id     [P]  look-up-table position (0 .. kh*kw-1) the event was taken from
      time       [P]  its timestamp
    with events sorted by (field, time, position, source order).  ``batch_size`` (samples in
    the batch) sizes the GPU pixel map; without it the largest batch id is read back."""
    geo = _geometry(frame_size, kernel_size, stride)
    r = _replicate_gpu(gr_batch_id, gr_h, gr_w, gr_lengths, gr_time, geo, batch_size)
    if r is not None:
        return r
    H, W, kh, kw, sh, sw, pt, pl, oh, ow = geo
    dev = gr_lengths.device
    nf = oh * ow
    G = gr_lengths.numel()
    area = kh * kw
    # candidate (group, position) pairs: field coordinate that sees pixel (y, x) at (dy, dx)
    dy = torch.arange(kh, device=dev).repeat_interleave(kw)
    dx = torch.arange(kw, device=dev).repeat(kh)
    ny = gr_h.view(G, 1) + pt - dy.view(1, area)
    nx = gr_w.view(G, 1) + pl - dx.view(1, area)
    ok = (ny >= 0) & (nx >= 0) & (ny % sh == 0) & (nx % sw == 0)
    oy, ox = ny // sh, nx // sw
    ok &= (oy < oh) & (ox < ow)
    gidx = torch.arange(G, device=dev).view(G, 1).expand(G, area)[ok]
    pos = torch.arange(area, device=dev).view(1, area).expand(G, area)[ok]
    fid = (gr_batch_id.view(G, 1) * nf + oy * ow + ox)[ok]
    # order pairs by (field, position); pairs of one group with distinct positions are distinct
    key = fid * area + pos
    order = torch.sort(key, stable=True)[1]
    gidx, pos, fid = gidx[order], pos[order], fid[order]
    field_ids, per_pair_field = torch.unique_consecutive(fid, return_inverse=True)
    reps = gr_lengths[gidx]
    lengths = torch.zeros(field_ids.numel(), dtype=gr_lengths.dtype, device=dev)
    lengths.scatter_add_(0, per_pair_field, reps)
    # expand pairs to events (group order within a pair)
    gstart = torch.cumsum(gr_lengths, 0) - gr_lengths
    n_ev = int(reps.sum())
    pair_of_ev = torch.repeat_interleave(torch.arange(gidx.numel(), device=dev), reps)
    pair_start = torch.cumsum(reps, 0) - reps
    within = torch.arange(n_ev, device=dev) - pair_start[pair_of_ev]
    src = gstart[gidx][pair_of_ev] + within
    t = gr_time[src]
    fld = per_pair_field[pair_of_ev]
    # stable time sort inside each field (pre-order: field, position, event)
    stride_t = (t.max() + 1) if n_ev else torch.tensor(1, device=dev)
    order = torch.sort(fld.to(torch.int64) * stride_t + t, stable=True)[1]
    return {
        "field_id": field_ids,
        "lengths": lengths,
        "src": src[order],
        "pos_id": pos[pair_of_ev][order],
        "time": t[order],
    }
