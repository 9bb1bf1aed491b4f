"""Prophesee .dat (Event2D) input, B200 side (utils/io/dat_events_tools.py,
utils/io/psee_loader.py, dataset/gen1.py:179-206 and the Gen1 collation of
model_base.py:82-117).

The host parses the text header and reads each recording's payload once (two little-endian
32-bit words per event: t and x | y << 14 | p << 28).  ``EventStore`` keeps the payloads of
many recordings resident in one device buffer (a Gen1 split is a few tens of GB, well inside
one GPU's HBM), and ``EventStore.windows`` builds a model batch on the GPU: one kernel
reproduces the loader's cursor arithmetic (``seek_time(ts - window)`` then
``load_delta_t(window + 1)``) per sample, one host read sizes the batch, and one kernel decodes
the events into the padded [B, Nmax, 4] float32 <x, y, t, 2p - 1> tensor the model takes.
The train-split augmentations of the dataset (random thinning, horizontal flip) are random
draws of the host's numpy generator and stay outside.
"""
from __future__ import annotations

import os
from typing import Iterable, List, Optional, Sequence, Tuple, Union

import numpy as np
import torch

from ... import _lib

EV_TYPE = [("t", "u4"), ("_", "i4")]  # Event2D
EV_STRING = "Event2D"


def parse_header(f):
    """(first payload byte, event type, event size in bytes, (height, width)) of an open .dat
    file (utils/io/dat_events_tools.py:141-196): '% ' comment lines, then, when there was a
    header, one byte of event type and one of event size."""
    f.seek(0, os.SEEK_SET)
    bod = None
    num_comment_line = 0
    size = [None, None]
    while True:
        bod = f.tell()
        line = f.readline()
        if line.decode("latin-1")[:2] != "% ":
            break
        words = line.split()
        if len(words) > 1:
            if words[1] in ("Height", b"Height"):
                size[0] = int(words[2])
            if words[1] in ("Width", b"Width"):
                size[1] = int(words[2])
        num_comment_line += 1
    f.seek(bod, os.SEEK_SET)
    if num_comment_line > 0:
        ev_type = int(np.frombuffer(f.read(1), dtype=np.uint8)[0])  # Python ints: numpy 2 keeps uint8
        ev_size = int(np.frombuffer(f.read(1), dtype=np.uint8)[0])   # arithmetic in uint8
    else:
        ev_type = 0
        ev_size = sum(int(n[-1]) for _, n in EV_TYPE)
    bod = f.tell()
    return bod, ev_type, ev_size, size


def count_events(filename) -> int:
    """Number of events of a .dat file (utils/io/dat_events_tools.py:125-138)."""
    with open(filename, "rb") as f:
        bod, _, ev_size, _ = parse_header(f)
        f.seek(0, os.SEEK_END)
        eod = f.tell()
    if (eod - bod) % ev_size != 0:
        raise Exception("unexpected format !")
    return (eod - bod) // ev_size


def read_payload(filename, ev_count: int = -1, ev_start: int = 0) -> np.ndarray:
    """The raw event words of a .dat file as a uint32 array [2 * events]."""
    with open(filename, "rb") as f:
        _, ev_type, ev_size, _ = parse_header(f)
        if int(ev_size) != 8:
            raise ValueError(f"{filename}: event size {int(ev_size)} is not the 8-byte Event2D layout")
        if ev_start > 0:
            f.seek(ev_start * 8, 1)
        words = np.fromfile(f, dtype="<u4", count=-1 if ev_count < 0 else 2 * ev_count)
    return words[: words.shape[0] // 2 * 2]


def write_dat(filename, t, x, y, p, height: int = 240, width: int = 304) -> None:
    """Write Event2D events in the .dat layout the loader reads (a '% ' text header with height
    and width, event type 0 and size 8, then (t, x | y << 14 | (p == 1) << 28) words; the
    layout of utils/io/dat_events_tools.py:199-254)."""
    if max(height, width) > 2 ** 14 - 1:
        raise ValueError("coordinates exceed the 14-bit range of the .dat format")
    t = np.asarray(t, dtype=np.uint32)
    packed = (np.asarray(x, np.int64) + (np.asarray(y, np.int64) << 14) +
              ((np.asarray(p) == 1).astype(np.int64) << 28)).astype(np.int32)
    data = np.empty(t.shape[0], dtype=[("t", "<u4"), ("_", "<i4")])
    data["t"] = t
    data["_"] = packed
    with open(filename, "wb") as f:
        f.write(b"% Data file containing Event2D events.\n% Version 2\n")
        f.write(f"% Height {height:d}\n% Width {width:d}\n".encode())
        f.write(np.array([0, 8], dtype=np.uint8).tobytes())
        data.tofile(f)


class EventStore:
    """Payloads of many recordings resident in one device buffer, sliced into model batches on
    the GPU.  ``add`` appends a recording (a .dat path or a uint32 word array) and returns its
    id; ``windows`` returns the padded Gen1 batch for labels at ``ts`` of the given recordings."""

    def __init__(self, device: Union[str, torch.device] = "cuda", capacity_events: int = 0):
        self.device = torch.device(device)
        _lib.require_cuda(torch.empty(0, device=self.device), what="EventStore")
        self._words = torch.empty(2 * max(int(capacity_events), 1), dtype=torch.int32, device=self.device)
        self._used = 0  # events
        self._start: List[int] = []
        self._count: List[int] = []

    def __len__(self) -> int:
        return len(self._start)

    @property
    def num_events(self) -> int:
        return self._used

    def add(self, recording: Union[str, os.PathLike, np.ndarray]) -> int:
        words = read_payload(recording) if isinstance(recording, (str, os.PathLike)) else \
            np.ascontiguousarray(recording, dtype=np.uint32)
        n = words.shape[0] // 2
        need = 2 * (self._used + n)
        if need > self._words.numel():
            grown = torch.empty(max(need, 2 * self._words.numel()), dtype=torch.int32, device=self.device)
            grown[: 2 * self._used].copy_(self._words[: 2 * self._used])
            self._words = grown
        if n:
            host = torch.from_numpy(words[: 2 * n].view(np.int32)).pin_memory()
            self._words[2 * self._used: 2 * (self._used + n)].copy_(host, non_blocking=True)
            torch.cuda.current_stream(self.device).synchronize()  # the pinned staging buffer is freed next
        self._start.append(self._used)
        self._count.append(n)
        self._used += n
        return len(self._start) - 1

    def ranges(self, rec_ids: Sequence[int], ts: Sequence[int], window_us, term_criterion: int = 100000):
        """([B, 2] [begin, end) event ranges relative to each recording, [B] lengths) on the device."""
        window = _integral_us(window_us)
        B = len(rec_ids)
        ids = list(rec_ids)
        meta = torch.tensor([[self._start[i] for i in ids], [self._count[i] for i in ids], [int(t) for t in ts]],
                            dtype=torch.int64).reshape(3, B).pin_memory().to(self.device, non_blocking=True)
        rng = torch.empty((B, 2), dtype=torch.int64, device=self.device)
        lengths = torch.empty(B, dtype=torch.int64, device=self.device)
        L = _lib.load()
        _lib.check(L.ssla_dat_window_ranges(self._words.data_ptr(), meta[0].data_ptr(), meta[1].data_ptr(),
                                            meta[2].data_ptr(), B, window, int(term_criterion), rng.data_ptr(),
                                            lengths.data_ptr(), _lib.stream_of(rng)), "dat_window_ranges")
        return rng, lengths, meta

    def windows(self, rec_ids: Sequence[int], ts: Sequence[int], window_us, term_criterion: int = 100000,
                max_len: Optional[int] = None) -> Tuple[torch.Tensor, torch.Tensor]:
        """Padded events [B, Nmax, 4] float32 <x, y, t, 2p - 1> and lengths [B] for labels at ts[b]
        of recordings rec_ids[b] (Gen1 val/test sample + collation).  Nmax is the longest window
        (one host read) unless ``max_len`` (>= every length) is given."""
        rng, lengths, meta = self.ranges(rec_ids, ts, window_us, term_criterion)
        B = len(rec_ids)
        nmax = int(lengths.max()) if (max_len is None and B) else int(max_len or 0)
        out = torch.empty((B, nmax, 4), dtype=torch.float32, device=self.device)
        _lib.check(_lib.load().ssla_dat_decode_windows(self._words.data_ptr(), meta[0].data_ptr(), rng.data_ptr(), B,
                                                       nmax, out.data_ptr(), _lib.stream_of(out)),
                   "dat_decode_windows")
        return out, lengths


def _integral_us(window_us) -> int:
    w = float(window_us)
    if not w.is_integer() or w < 0:
        raise ValueError(f"window of {window_us} us: whole non-negative microseconds are required")
    return int(w)


def load_td_data(filename, ev_count: int = -1, ev_start: int = 0, device="cuda"):
    """Events of a .dat file decoded on the GPU: dict of device tensors t (int64), x, y (int16),
    p (int8) (utils/io/dat_events_tools.py:20-46 returns the same fields as a structured
    array)."""
    words = torch.from_numpy(read_payload(filename, ev_count, ev_start).view(np.int32)).to(device)
    store_t = words[0::2].to(torch.int64) & 0xFFFFFFFF
    packed = words[1::2]
    return {"t": store_t, "x": (packed & 16383).to(torch.int16), "y": ((packed & 268419072) >> 14).to(torch.int16),
            "p": ((packed & 268435456) >> 28).to(torch.int8)}
