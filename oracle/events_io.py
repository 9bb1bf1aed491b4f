"""CPU restatement of the Gen1 event input path (test infrastructure only).

Follows, on a numpy array of .dat payload words (two uint32 per event: t, packed
x | y << 14 | p << 28):
  * the stream loader's cursor arithmetic: ``seek_time`` (utils/io/psee_loader.py:177-219:
    bisection over events until at most ``term_criterion`` remain, an exact timestamp hit
    leaving the cursor one event past it because the probe read advanced the file, then a
    searchsorted of the remaining interval; ``seek_event`` clamping, :153-175) and
    ``load_delta_t`` (:109-151: 100000-event buffers read until one ends at or after the
    target, the last cut by searchsorted);
  * the Event2D decode (utils/io/dat_events_tools.py:14, :89-107: x = w & 16383,
    y = (w & 268419072) >> 14, p = (w & 268435456) >> 28);
  * the Gen1 window of a label at ts (dataset/gen1.py:190-193: seek_time(ts - window),
    load_delta_t(window + 1)) and the batch collation (model_base.py:82-117: float32 <t, x, y,
    p> zero-padded, reordered to <x, y, t, p>, p -> 2p - 1 on every row).
Pinned against the reference's own ``PSEELoader`` on synthetic .dat files
(``tests/golden/make_golden_events.py`` → ``tests/golden/events_io.pt``).
"""
from __future__ import annotations

import numpy as np

LOAD_BATCH = 100000


def _bisect_left(t: np.ndarray, lo: int, hi: int, key: int) -> int:
    """numpy.searchsorted(t[lo:hi], key) + lo for one key (plain bisection)."""
    while lo < hi:
        mid = lo + ((hi - lo) >> 1)
        if int(t[mid]) < key:
            lo = mid + 1
        else:
            hi = mid
    return lo


def seek_time(t: np.ndarray, final_time: int, term_criterion: int = 100000):
    """(cursor event index, current_time, done) after PSEELoader.seek_time (psee_loader.py:177-219)."""
    n = t.shape[0]
    total = int(t[n - 1]) if n else 0
    if final_time > total:
        return n, total + 1, True
    if final_time <= 0:
        return 0, 0, False
    low, high = 0, n
    while high - low > term_criterion:
        middle = (low + high) // 2
        mid = int(t[middle])
        if mid > final_time:
            high = middle
        elif mid < final_time:
            low = middle + 1
        else:
            pos = middle + 1
            return pos, final_time, pos >= n
    pos = min(max(_bisect_left(t, low, high, final_time), 0), n)
    return pos, final_time, pos >= n


def load_delta_t(t: np.ndarray, pos: int, current_time: int, done: bool, delta_t: int):
    """[begin, end) event range returned by PSEELoader.load_delta_t (psee_loader.py:109-151)."""
    n = t.shape[0]
    if delta_t < 1:
        raise ValueError("delta_t must be at least 1 micro-second")
    if done or pos >= n:
        return pos, pos
    final_time = current_time + delta_t
    tmp, p = current_time, pos
    last_lo = last_hi = pos
    while tmp < final_time and p < n:
        hi = min(n, p + LOAD_BATCH)
        tmp = int(t[hi - 1])
        last_lo, last_hi, p = p, hi, hi
    return pos, _bisect_left(t, last_lo, last_hi, final_time)


def window_range(words: np.ndarray, ts: int, window: int, term_criterion: int = 100000):
    t = words[0::2]
    pos, cur, done = seek_time(t, ts - window, term_criterion)
    return load_delta_t(t, pos, cur, done, window + 1)


def decode(words: np.ndarray):
    """(t, x, y, p) of Event2D words, in the loader's dtypes (u4, u2, u2, u1)."""
    t = words[0::2].astype(np.uint32)
    w = words[1::2].astype(np.uint32)
    return (t, (w & 16383).astype(np.uint16), ((w & 268419072) >> 14).astype(np.uint16),
            ((w & 268435456) >> 28).astype(np.uint8))


def gen1_batch(recordings, ts, window: int, term_criterion: int = 100000):
    """Padded [B, Nmax, 4] float32 <x, y, t, 2p - 1> batch and lengths for labels at ts[b] of
    recording words recordings[b] (dataset/gen1.py:179-206 without the train augmentations,
    model_base.py:82-117)."""
    samples = []
    for words, t_end in zip(recordings, ts):
        b, e = window_range(words, int(t_end), window, term_criterion)
        t, x, y, p = decode(words[2 * b:2 * e])
        samples.append(np.stack([t.astype(np.float32), x.astype(np.float32), y.astype(np.float32),
                                 p.astype(np.float32)], axis=-1).reshape(-1, 4))
    lens = [s.shape[0] for s in samples]
    nmax = max(lens) if lens else 0
    ev = np.stack([np.pad(s, ((0, nmax - s.shape[0]), (0, 0))) for s in samples], 0) if samples else \
        np.zeros((0, 0, 4), np.float32)
    ev = ev[:, :, [1, 2, 0, 3]]
    ev[:, :, -1] = ev[:, :, -1] * 2 - 1
    return ev, np.asarray(lens, dtype=np.int64)
