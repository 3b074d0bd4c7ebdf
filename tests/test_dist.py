"""Frame sharding host logic on the CPU with gloo, world size 2 (the GPU path is the same code over NCCL)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from promptmoge_b200.dist import frame_range, gather_frame_states


@pytest.mark.parametrize("n,world", [(256, 8), (10, 3), (2, 4), (0, 2), (7, 1)])
def test_frame_ranges_partition(n, world):
    seen = []
    sizes = []
    for r in range(world):
        b, e = frame_range(n, r, world)
        seen += list(range(b, e))
        sizes.append(e - b)
    assert seen == list(range(n))
    assert max(sizes) - min(sizes) <= 1


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, n_frames, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=60))
    try:
        b, e = frame_range(n_frames, rank, world)
        # frame f's state: 18 words, word 0 = f, word 1 = rank
        local = torch.zeros((e - b, 18), dtype=torch.int32)
        local[:, 0] = torch.arange(b, e, dtype=torch.int32)
        local[:, 1] = rank
        out = gather_frame_states(local, n_frames)
        q.put((rank, out[:, 0].tolist(), out[:, 1].tolist()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n_frames", [9, 8])
def test_gather_frame_states_gloo_world2(n_frames):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, n_frames, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, frames, owners in res:
        assert frames == list(range(n_frames))
        assert owners == [0 if f < frame_range(n_frames, 0, 2)[1] else 1 for f in range(n_frames)]


def _failing_worker(rank, world, port, q):
    """Rank 1 fails on the host before the gather (its frames raise); rank 0's gather must end with an error within
    the process group's short timeout instead of waiting for good."""
    import datetime
    import time
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
    if rank == 1:
        q.put((rank, "failed", 0.0))
        q.close()
        q.join_thread()
        os._exit(3)
    t0 = time.monotonic()
    try:
        gather_frame_states(torch.zeros((4, 18), dtype=torch.int32), 8)
        q.put((rank, "completed", time.monotonic() - t0))
    except RuntimeError:
        q.put((rank, "error", time.monotonic() - t0))
    q.close()
    q.join_thread()
    os._exit(0)


def test_peer_failure_ends_gather_with_error_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict((r, (what, dt)) for r, what, dt in (q.get(timeout=120) for _ in procs))
    for p in procs:
        p.join(timeout=60)
    assert res[1][0] == "failed" and procs[1].exitcode == 3
    assert res[0][0] == "error" and res[0][1] < 30.0
    assert procs[0].exitcode == 0
