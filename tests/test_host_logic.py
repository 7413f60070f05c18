"""Host-side logic of the multi-GPU benchmark on CPU: image sharding over
ranks (world size 2, gloo) and the max-over-ranks timing reduction."""
import os
import socket
import sys

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import ROOT

sys.path.insert(0, ROOT)
import bench  # noqa: E402


def test_image_shard_covers_every_image_once():
    for world in (1, 2, 4, 8):
        seen = []
        for r in range(world):
            first, count = bench.image_shard(r, world, 64)
            seen.extend(range(first, first + count))
        assert sorted(seen) == list(range(64))
    with pytest.raises(ValueError):
        bench.image_shard(0, 3, 64)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    first, count = bench.image_shard(rank, world, 64)
    owned = torch.zeros(64, dtype=torch.int64)
    owned[first:first + count] = 1
    dist.all_reduce(owned)  # every image owned by exactly one rank
    t = torch.tensor([10.0 * (rank + 1)], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)  # the job time is the slowest rank's
    out[rank] = (int(owned.min()), int(owned.max()), float(t.item()))
    dist.destroy_process_group()


def test_two_rank_gloo_sharding_and_max_reduction():
    port = _free_port()
    # the manager's server process is spawned, not forked: this process may
    # already run threads (torch), and a fork of a threaded process can hang
    with mp.get_context("spawn").Manager() as m:
        out = m.dict()
        mp.spawn(_worker, args=(2, port, out), nprocs=2, join=True)
        res = dict(out)
    assert res[0] == res[1] == (1, 1, 20.0)


def _dying_rank_worker(rank, port, q):
    import datetime
    import time
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2,
                            timeout=datetime.timedelta(seconds=10))
    if rank == 1:
        os._exit(3)  # leaves between steps: nothing of it is in flight
    t0 = time.monotonic()
    try:
        dist.barrier()
        q.put(("completed", time.monotonic() - t0))
    except Exception as e:  # the surviving rank learns of it at its next collective
        q.put((type(e).__name__, time.monotonic() - t0))
    q.close()
    q.join_thread()  # the message reaches the pipe before the hard exit
    os._exit(0)


def test_rank_that_dies_ends_the_others_next_collective_with_an_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dying_rank_worker, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=90)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung instead of failing"
    outcome, seconds = q.get(timeout=5)
    assert outcome != "completed" and seconds < 60
    assert procs[1].exitcode == 3 and procs[0].exitcode == 0
