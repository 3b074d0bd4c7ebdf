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
