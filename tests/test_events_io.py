"""Event input (Gen1 .dat windows): the oracle against the reference loader's golden cases,
the host-side .dat handling, and the GPU window slicing + collation against the oracle."""
from __future__ import annotations

import hashlib
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import events_io as oev
from ssla_b200.synthetic import dat_recording
from ssla_b200.utils.io import count_events, parse_header, read_payload, write_dat

GOLDEN = Path(__file__).parent / "golden" / "events_io.pt"


@pytest.fixture(scope="module")
def golden():
    g = torch.load(GOLDEN, weights_only=False)
    recs = [dat_recording(s, n, d) for s, n, d in g["recordings"]]
    assert [int(w.astype(np.int64).sum()) for w in recs] == g["checksums"], "synthetic recordings drifted"
    return g, recs


def _sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a, dtype=np.float32).tobytes()).hexdigest()


def test_oracle_matches_reference_loader(golden):
    g, recs = golden
    hits = 0
    for r, ts, window, term, begin, length in g["cases"].tolist():
        t = recs[r][0::2]
        pos, cur, done = oev.seek_time(t, ts - window, term)
        b, e = oev.load_delta_t(t, pos, cur, done, window + 1)
        assert (b, e - b) == (begin, length), (r, ts, window, term)
        ft = ts - window
        if 0 < ft <= (int(t[-1]) if t.shape[0] else 0):
            hits += int(pos != oev._bisect_left(t, 0, t.shape[0], ft))  # the cursor skipped a hit
    assert hits > 0  # the exact-hit branch of the bisection is exercised


def test_oracle_collation_matches_reference(golden):
    g, recs = golden
    cases = [c for c in g["cases"].tolist() if c[3] == 100000]
    for window, ref in g["batches"].items():
        sel = [c for c in cases if c[2] == window][:24]
        ev, lens = oev.gen1_batch([recs[c[0]] for c in sel], [c[1] for c in sel], window)
        assert tuple(ev.shape) == ref["shape"]
        assert np.array_equal(lens, ref["lengths"].numpy())
        assert _sha(ev) == ref["sha256"]


def test_dat_file_roundtrip(tmp_path):
    words = dat_recording(7, 1234, 10000)
    t, packed = words[0::2], words[1::2].astype(np.int64)
    path = tmp_path / "x_td.dat"
    write_dat(path, t, packed & 16383, (packed >> 14) & 16383, (packed >> 28) & 1, height=240, width=304)
    with open(path, "rb") as f:
        bod, ev_type, ev_size, size = parse_header(f)
    assert (ev_type, ev_size, size) == (0, 8, [240, 304])
    assert count_events(path) == 1234
    assert np.array_equal(read_payload(path), words)
    assert np.array_equal(read_payload(path, ev_count=10, ev_start=5), words[10:30])


@pytest.mark.gpu
def test_gpu_windows_match_golden_cases(golden):
    from ssla_b200.utils.io import EventStore

    g, recs = golden
    store = EventStore("cuda")
    ids = [store.add(w) for w in recs]
    cases = g["cases"]
    for term in (100000, 1000):
        sel = cases[cases[:, 3] == term]
        for window in sel[:, 2].unique().tolist():
            c = sel[sel[:, 2] == window]
            rng, lengths, _ = store.ranges([ids[r] for r in c[:, 0].tolist()], c[:, 1].tolist(), window, term)
            assert torch.equal(rng[:, 0].cpu(), c[:, 4]), (term, window)
            assert torch.equal(lengths.cpu(), c[:, 5]), (term, window)


@pytest.mark.gpu
def test_gpu_batches_bit_exact(golden):
    from ssla_b200.utils.io import EventStore

    g, recs = golden
    store = EventStore("cuda")
    ids = [store.add(w) for w in recs]
    cases = [c for c in g["cases"].tolist() if c[3] == 100000]
    for window, ref in g["batches"].items():
        sel = [c for c in cases if c[2] == window][:24]
        ev, lens = store.windows([ids[c[0]] for c in sel], [c[1] for c in sel], window)
        assert tuple(ev.shape) == ref["shape"]
        assert torch.equal(lens.cpu(), ref["lengths"])
        assert _sha(ev.cpu().numpy()) == ref["sha256"]


@pytest.mark.gpu
def test_gpu_windows_large_recording_vs_oracle():
    """A 4M-event recording with dense duplicate timestamps, many random labels: ranges and the
    collated batch equal the oracle's; a fixed max_len pads past the longest window."""
    from ssla_b200.utils.io import EventStore

    words = dat_recording(11, 4_000_000, 3_000_000)
    store = EventStore("cuda")
    rid = store.add(words)
    rs = np.random.default_rng(5)
    ts = [int(v) for v in rs.integers(0, 3_200_000, 64)]
    ev, lens = store.windows([rid] * 64, ts, 50000)
    ref, rlens = oev.gen1_batch([words] * 64, ts, 50000)
    assert np.array_equal(lens.cpu().numpy(), rlens)
    assert np.array_equal(ev.cpu().numpy(), ref)
    ev2, _ = store.windows([rid] * 3, ts[:3], 50000, max_len=int(rlens.max()) + 5)
    assert torch.equal(ev2[:, : ev.shape[1]].cpu(), ev[:3].cpu()) or ev.shape[1] == 0
    assert torch.equal(ev2[:, ev.shape[1]:].cpu(), torch.tensor([0., 0., 0., -1.]).expand(3, ev2.shape[1] - ev.shape[1], 4))


def test_window_must_be_whole_microseconds():
    from ssla_b200.utils.io.dat_events_tools import _integral_us

    assert _integral_us(0.1 * 1e6) == 100000  # the Gen1 configs' 0.1 s window
    with pytest.raises(ValueError):
        _integral_us(1000.5)
    with pytest.raises(ValueError):
        _integral_us(-1)
