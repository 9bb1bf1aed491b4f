"""Golden fixture for the event-input parity tests, produced by the reference's own stream
loader and collation on the CPU.

    python tests/golden/make_golden_events.py /path/to/ssla

Synthetic recordings (``ssla_b200.synthetic.dat_recording``, seeded, so only their checksums
are stored) are written as .dat files with ``ssla_b200.utils.io.write_dat``; for every case the
reference ``PSEELoader`` runs ``seek_time(ts - window)`` and ``load_delta_t(window + 1)`` (the
calls of dataset/gen1.py:190-193) and the cursor position and returned events are recorded;
``BaseModel.pad_batches`` (model_base.py:82-117, lightning stubbed) collates one batch per
window size (stored as its shape, lengths and the SHA-256 of its float32 bytes).  Cases cover
windows reaching before the stream start, an exact timestamp hit of the bisection, targets at and past the last timestamp, short and empty recordings and a small
bisection stop.  Harness-side shims only: lightning stubs, and the header's uint8 event size
handed back as a Python int (numpy 2 would keep the loader's byte arithmetic in uint8).
"""
from __future__ import annotations

import hashlib
import sys
import tempfile
from pathlib import Path

import numpy as np
import torch

OUT = Path(__file__).resolve().parent
ROOT = OUT.parent.parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(OUT))

from ssla_b200.synthetic import dat_recording  # noqa: E402
from ssla_b200.utils.io import write_dat  # noqa: E402

RECORDINGS = [  # (seed, events, duration_us)
    (1, 300000, 2000000),
    (2, 5000, 1000000),
    (3, 0, 1),
    (4, 250000, 500000),
]


def cases(words_list):
    out = []
    for r, words in enumerate(words_list):
        t = words[0::2]
        n = t.shape[0]
        total = int(t[-1]) if n else 0
        for window in (100000, 50000, 1):
            ts = [window // 2, window, window + 1, total + window, total + window + 1, total + 3 * window]
            if n:
                ts += [int(t[n // 2]) + window, int(t[n // 4]) + window, int(t[(3 * n) // 4]) + window]
                rs = np.random.default_rng(1000 * r + window)
                ts += [int(v) for v in rs.integers(0, total + 2 * window, 6)]
            for term in (100000, 1000):
                out += [(r, int(v), window, term) for v in ts]
    return out


def main(ref_root: str):
    sys.path.insert(0, ref_root)
    from make_golden_model import install_shims

    install_shims()
    from utils.io import dat_events_tools as dat_tools
    from utils.io.psee_loader import PSEELoader

    # numpy 2 keeps the header's uint8 event size in uint8 arithmetic (the loader's byte counts
    # overflow); the reference ran under numpy 1, where they promote: hand back Python ints.
    parse = dat_tools.parse_header

    def parse_header_ints(f):
        bod, ev_type, ev_size, size = parse(f)
        return bod, int(ev_type), int(ev_size), size

    dat_tools.parse_header = parse_header_ints
    import model_base

    recs = [dat_recording(s, n, d) for s, n, d in RECORDINGS]
    with tempfile.TemporaryDirectory() as tmp:
        paths = []
        for i, w in enumerate(recs):
            path = str(Path(tmp) / f"rec{i}_td.dat")
            t = w[0::2]
            packed = w[1::2].astype(np.int64)
            write_dat(path, t, packed & 16383, (packed >> 14) & 16383, (packed >> 28) & 1)
            paths.append(path)
        rows = []
        windows = {}
        for r, ts, window, term in cases(recs):
            loader = PSEELoader(paths[r])
            loader.seek_time(ts - window, term_criterion=term)
            begin = (loader._file.tell() - loader._start) // loader._ev_size
            ev = loader.load_delta_t(window + 1)
            rows.append([r, ts, window, term, begin, len(ev)])
            if term == 100000:
                windows.setdefault(window, []).append((ev, np.zeros((0, 5), np.float32)))
        fake = type("Fake", (), {"dataset": "Gen1"})()
        batches = {}
        for window, data in windows.items():
            batch = model_base.BaseModel.pad_batches(fake, data[:24])
            ev = batch["events"].contiguous().numpy()
            batches[window] = {"shape": tuple(ev.shape), "sha256": hashlib.sha256(ev.tobytes()).hexdigest(),
                               "lengths": batch["lengths"].clone()}
    torch.save({
        "recordings": RECORDINGS,
        "checksums": [int(w.astype(np.int64).sum()) for w in recs],
        "cases": torch.tensor(rows, dtype=torch.int64),
        "batches": batches,
    }, OUT / "events_io.pt")
    print("cases", len(rows), "batches", {k: v["shape"] for k, v in batches.items()})


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")
