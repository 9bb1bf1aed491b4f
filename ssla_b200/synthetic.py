"""Seeded synthetic event data with the shapes and distributions of the benchmark configs
(Gen1-like 240x304 frames; the Gen1 dataset itself is not used).

* ``event_stream``: one 100 ms sample of 20 bins x 5 ms; per bin round(0.02 * H * W) events,
  half at uniform pixels, half around 20 Gaussian blobs (sigma 8 px, centres fixed per
  sample); timestamps uniform within the bin (microseconds), polarity +-1; sorted by time.
* ``event_batch``: B such samples padded into [B, Nmax, 4] rows <x, y, t, p> plus lengths.
* ``pooling_rows``: BASELINE config 4 — per (batch, polarity) plane ~5% active pixels (half
  uniform, half blob), Poisson(3) events per pixel, rows sorted by flat pixel index, bf16
  features; cell ids for k x k pooling compacted to consecutive segment ids.
"""
from __future__ import annotations

import torch


def event_stream(seed: int, frame=(240, 304), bins: int = 20, bin_us: int = 5000, occupancy: float = 0.02,
                 blobs: int = 20, sigma: float = 8.0) -> torch.Tensor:
    H, W = frame
    g = torch.Generator().manual_seed(seed)
    per_bin = int(occupancy * H * W)
    centres = torch.stack([torch.rand(blobs, generator=g) * W, torch.rand(blobs, generator=g) * H], 1)
    rows = []
    for b in range(bins):
        nu = per_bin // 2
        nb = per_bin - nu
        xu = torch.randint(0, W, (nu,), generator=g)
        yu = torch.randint(0, H, (nu,), generator=g)
        which = torch.randint(0, blobs, (nb,), generator=g)
        pb = centres[which] + torch.randn(nb, 2, generator=g) * sigma
        xb = pb[:, 0].round().clamp(0, W - 1).long()
        yb = pb[:, 1].round().clamp(0, H - 1).long()
        x = torch.cat([xu, xb])
        y = torch.cat([yu, yb])
        t = b * bin_us + torch.randint(0, bin_us, (per_bin,), generator=g)
        p = torch.randint(0, 2, (per_bin,), generator=g) * 2 - 1
        rows.append(torch.stack([x, y, t, p], 1))
    ev = torch.cat(rows).float()
    return ev[torch.sort(ev[:, 2], stable=True)[1]]


def event_batch(B: int, seed: int = 0, **kw):
    streams = [event_stream(seed * 1000 + i, **kw) for i in range(B)]
    lengths = torch.tensor([s.shape[0] for s in streams])
    out = torch.zeros(B, int(lengths.max()), 4)
    for i, s in enumerate(streams):
        out[i, : s.shape[0]] = s
    return out, lengths


def pooling_rows(seed: int = 0, B: int = 16, frame=(240, 304), C: int = 64, active: float = 0.05, blobs: int = 20,
                 sigma: float = 8.0, mean_count: float = 3.0, dtype=torch.bfloat16):
    """(features [R, C], flat pixel index [R] sorted, dict of k -> (segment ids [R], n_segments))."""
    H, W = frame
    g = torch.Generator().manual_seed(seed)
    flat = []
    n_act = round(active * H * W)
    for plane in range(B * 2):
        nu = n_act // 2
        uni = torch.randperm(H * W, generator=g)[:nu]
        centres = torch.stack([torch.rand(blobs, generator=g) * W, torch.rand(blobs, generator=g) * H], 1)
        which = torch.randint(0, blobs, (n_act - nu,), generator=g)
        pb = centres[which] + torch.randn(n_act - nu, 2, generator=g) * sigma
        blob = pb[:, 1].round().clamp(0, H - 1).long() * W + pb[:, 0].round().clamp(0, W - 1).long()
        pix = torch.unique(torch.cat([uni, blob]))
        cnt = torch.poisson(torch.full((pix.numel(),), mean_count), generator=g).long()
        keep = cnt > 0
        flat.append((plane * H * W + pix[keep]).repeat_interleave(cnt[keep]))
    idx = torch.cat(flat)
    feats = torch.randn(idx.numel(), C, generator=g).to(dtype)
    cells = {}
    for k in (2, 4):
        plane = idx // (H * W)
        rem = idx % (H * W)
        y, x = rem // W, rem % W
        cell = (plane * (H // k) + y // k) * (W // k) + x // k
        uniq, inv = torch.unique(cell, return_inverse=True)
        cells[k] = (inv, uniq.numel())
    return feats, idx, cells


def seeded_parameters(model: torch.nn.Module, seed: int) -> None:
    """Overwrite every parameter with seeded values, in sorted-name order, so that two models with
    the same parameter names and shapes get identical weights (used to compare implementations
    without shipping checkpoints).  Scales: Xavier for the per-position projections
    (sqrt(2 / (in + hidden))), 1/sqrt(fan_in) for other weights, 1 + 0.1 N(0,1) for
    normalisation scales, 0.05 N(0,1) for biases."""
    g = torch.Generator().manual_seed(seed)
    mods = dict(model.named_modules())
    with torch.no_grad():
        for name, p in sorted(model.named_parameters()):
            owner, _, leaf = name.rpartition(".")
            m = mods.get(owner)
            x = torch.randn(p.shape, generator=g)
            if leaf in ("scatter_conv_weights", "gather_conv_weights"):
                fan = m.input_size if leaf == "scatter_conv_weights" else m.hidden_size
                x *= (2.0 / (fan + m.hidden_size)) ** 0.5
            elif leaf == "bias":
                x *= 0.05
            elif isinstance(m, (torch.nn.LayerNorm, torch.nn.BatchNorm2d)):
                x = 1.0 + 0.1 * x
            else:
                fan_in = p[0].numel() if p.dim() > 1 else p.numel()
                x *= fan_in ** -0.5
            p.copy_(x.to(p.dtype))


def dat_recording(seed: int, events: int, duration_us: int, frame=(240, 304)):
    """Seeded Event2D payload words (uint32 [2 * events]: t, x | y << 14 | p << 28) of a
    recording with `events` events, timestamps uniform in [0, duration_us) and sorted (equal
    timestamps occur when events > duration_us / few), uniform pixels and polarities."""
    import numpy as np

    g = torch.Generator().manual_seed(seed)
    t = torch.sort(torch.randint(0, max(int(duration_us), 1), (events,), generator=g))[0]
    x = torch.randint(0, frame[1], (events,), generator=g)
    y = torch.randint(0, frame[0], (events,), generator=g)
    p = torch.randint(0, 2, (events,), generator=g)
    words = torch.stack([t, x | (y << 14) | (p << 28)], 1).reshape(-1)
    return words.numpy().astype(np.uint32)
