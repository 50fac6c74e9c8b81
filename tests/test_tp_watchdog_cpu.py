"""Failure detection for tensor-parallel decoding, on CPU with gloo ranks
(no GPU fault is involved): a rank that leaves between steps is noticed by
the others through the heartbeat store before they enter the next
collective (woolly_b200/tp.py).  Three ranks run steps of an all-reduce;
rank 2 stops after step 1.  Ranks 0 and 1 must raise WoollyError
(WL_ERR_NCCL) naming rank 2 at step 2, within the heartbeat timeout, and
must not have entered step 2's collective."""
import os
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, leave_after, q):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    from woolly_b200 import _lib
    from woolly_b200.tp import RankWatch
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    store = dist.TCPStore("127.0.0.1", port + 1, world, rank == 0, timeout=__import__("datetime").timedelta(seconds=30))
    dist.init_process_group("gloo", rank=rank, world_size=world, store=dist.PrefixStore("pg", store))
    watch = RankWatch(store, rank, world, timeout_s=1.5)
    done = []
    try:
        for step in range(4):
            if rank == leave_after[0] and step > leave_after[1]:
                watch.leave()
                q.put((rank, "left", done))
                return
            watch.guard(step)
            x = torch.ones(4) * (rank + 1)
            dist.all_reduce(x)  # the collective a missing rank would block forever
            done.append(step)
        q.put((rank, "ok", done))
    except _lib.WoollyError as e:
        q.put((rank, f"error {e.code}: {e.message}", done))
    finally:
        time.sleep(0.2)
        os._exit(0)  # no destroy_process_group: a peer is gone


@pytest.mark.parametrize("world", [3])
def test_rank_that_leaves_is_detected_before_the_collective(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, (2, 1), q)) for r in range(world)]
    t0 = time.time()
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, status, done = q.get(timeout=60)
        res[r] = (status, done)
    for p in procs:
        p.join(timeout=30)
    assert time.time() - t0 < 45
    assert res[2][0] == "left" and res[2][1] == [0, 1]
    for r in (0, 1):
        status, done = res[r]
        assert status.startswith("error 14"), status  # WL_ERR_NCCL
        assert "[2]" in status
        assert done == [0, 1]  # step 2's collective was never entered


def test_all_ranks_present_passes():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, (-1, 99), q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict((r, (s, d)) for r, s, d in (q.get(timeout=60) for _ in range(2)))
    for p in procs:
        p.join(timeout=30)
    assert all(s == "ok" and d == [0, 1, 2, 3] for s, d in res.values())
