"""Host-side logic of the multi-GPU path on CPU ranks (gloo, world size 2): sample sharding and
the output gather; a rank failure surfaces as an error on the other rank instead of a hang."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import datetime

    from ssla_b200.distributed import gather_outputs, shard_range

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    a, b = shard_range(7, rank, world)
    x = torch.arange(a, b, dtype=torch.float32).view(-1, 1).repeat(1, 3)
    y = gather_outputs(x)
    q.put((rank, y[:, 0].tolist()))
    dist.destroy_process_group()


def _failing_worker(rank, world, port, q):
    import datetime

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        os._exit(3)  # a rank that dies between steps
    try:
        dist.all_reduce(torch.ones(1))
        q.put((rank, "no error"))
    except Exception as e:  # noqa: BLE001
        q.put((rank, type(e).__name__))


def test_shard_range_covers_everything():
    from ssla_b200.distributed import shard_range

    for n in (0, 1, 7, 64):
        for w in (1, 2, 3, 8):
            parts = [shard_range(n, r, w) for r in range(w)]
            assert parts[0][0] == 0 and parts[-1][1] == n
            assert all(parts[i][1] == parts[i + 1][0] for i in range(w - 1))


def test_gather_outputs_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=60) for _ in ps)
    for p in ps:
        p.join(30)
    assert res[0] == res[1] == [float(i) for i in range(7)]


def test_dead_rank_is_reported_not_hung():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_failing_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    rank, what = q.get(timeout=60)
    for p in ps:
        p.join(30)
        if p.is_alive():
            p.kill()
    assert rank == 0 and what != "no error"
