"""Fused multi-frame scene (config 5) host logic on the CPU: Morton codes, the scene generator, count-balanced
Morton shards, and the halo plan + all-to-all exchange over gloo at world sizes 2 and 3.  The per-layer conv here is
the numpy oracle, so the test checks that a sharded stack of convs equals the single-device stack voxel by voxel;
the GPU run (tests/test_gpu_fused.py, bench.py --fused-scene) uses the same plan with the tcgen05 kernel."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import refiner as oref
from oracle import structure as ost
from promptmoge_b200 import fused

EXT = [1, 1 << 21, 1 << 21, 1 << 21]


def test_morton_roundtrip_and_order():
    rng = np.random.default_rng(0)
    xyz = torch.from_numpy(rng.integers(0, 1 << 21, (5000, 3)))
    code = fused.morton3(xyz[:, 0], xyz[:, 1], xyz[:, 2])
    x, y, z = fused.demorton3(code)
    assert torch.equal(torch.stack([x, y, z], 1), xyz)
    # children of one parent (coords >> 1) are one contiguous code range: code >> 3 == parent's code
    par = fused.morton3(xyz[:, 0] >> 1, xyz[:, 1] >> 1, xyz[:, 2] >> 1)
    assert torch.equal(code >> 3, par)
    # bit layout: x in the lowest bit of each triple
    assert int(fused.morton3(torch.tensor([1]), torch.tensor([0]), torch.tensor([0]))) == 1
    assert int(fused.morton3(torch.tensor([0]), torch.tensor([1]), torch.tensor([0]))) == 2
    assert int(fused.morton3(torch.tensor([0]), torch.tensor([0]), torch.tensor([1]))) == 4


def _small_scene():
    coords, info = fused.make_fused_scene(3, n_poses=4, H=12, W=16, voxel=0.05, room_size=(4.0, 4.0, 3.0))
    return coords, info


def test_scene_unique_sorted_deterministic():
    coords, info = _small_scene()
    again, _ = _small_scene()
    assert torch.equal(coords, again)
    assert info["voxels"] == coords.shape[0] > 100
    code = fused.morton3(coords[:, 1], coords[:, 2], coords[:, 3])
    assert bool((code[1:] > code[:-1]).all())          # unique and in Morton order
    assert int(coords[:, 1:].min()) >= 0


@pytest.mark.parametrize("M,world", [(10, 3), (1000, 8), (5, 5), (0, 2)])
def test_shard_bounds_partition(M, world):
    b = fused.shard_bounds(M, world)
    assert b[0][0] == 0 and b[-1][1] == M
    assert all(b[i][1] == b[i + 1][0] for i in range(world - 1))
    sizes = [hi - lo for lo, hi in b]
    assert max(sizes) - min(sizes) <= 1


def test_tile_mask_of():
    rng = np.random.default_rng(1)
    nm = rng.integers(-3, 5, (27, 70)).astype(np.int32)
    nm[nm < 0] = -1
    got = fused.tile_mask_of(torch.from_numpy(nm)).numpy().view(np.uint32)
    for g in range(3):
        rows = nm[:, 32 * g:32 * (g + 1)]
        want = sum(1 << v for v in range(27) if (rows[v] >= 0).any())
        assert int(got[g]) == want


def _layers_np(n, C, seed):
    rng = np.random.default_rng(seed)
    return [(rng.integers(-127, 128, (C, 3, 3, 3, C)).astype(np.int8), rng.uniform(1e-4, 5e-4, C).astype(np.float32),
             (rng.standard_normal(C) * 0.1).astype(np.float32)) for _ in range(n)]


def _oracle_layer(q, nmap_rm, layer):
    """int8 conv -> dequant -> SiLU -> requantise with the reference's rules (the oracle's arithmetic)."""
    w, ws, b = layer
    acc = oref.conv_acc(q, nmap_rm, w)
    y = oref.dequant(acc, np.float32(0.05), ws, b)
    return np.clip(np.rint(oref.silu(y) / np.float32(0.04)), -127, 127).astype(np.int8)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=60))
    try:
        coords, _ = _small_scene()
        M = coords.shape[0]
        nmap_rm = ost.nmap_sorted(coords.numpy(), EXT)               # [M, 27] global ids
        bounds = fused.shard_bounds(M, world)
        lo, hi = bounds[rank]
        nmap_owned = torch.from_numpy(np.ascontiguousarray(nmap_rm[lo:hi].T))
        plan = fused.ShardPlan(nmap_owned, bounds, rank)
        C = 16
        rng = np.random.default_rng(5)
        q0 = rng.integers(-127, 128, (M, C)).astype(np.int8)
        layers = _layers_np(3, C, 9)

        def conv(q_local, nmap_tm, mask, layer):
            return torch.from_numpy(_oracle_layer(q_local.numpy(), nmap_tm.numpy().T, layer))

        out = fused.run_layers(plan, torch.from_numpy(q0[lo:hi]), layers, conv)
        parts = [None] * world
        dist.all_gather_object(parts, out.numpy())
        q.put((rank, np.concatenate(parts, axis=0), plan.n_halo, plan.send_splits, plan.recv_splits))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_layers_equal_single_device_gloo(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=180) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # single device: the same three layers over the whole voxel set
    coords, _ = _small_scene()
    nmap_rm = ost.nmap_sorted(coords.numpy(), EXT)
    C = 16
    qv = np.random.default_rng(5).integers(-127, 128, (coords.shape[0], C)).astype(np.int8)
    for layer in _layers_np(3, C, 9):
        qv = _oracle_layer(qv, nmap_rm, layer)
    recv_total = {r: sum(rs) for r, _, _, _, rs in res}
    send_total = {r: sum(ss) for r, _, _, ss, _ in res}
    for rank, got, n_halo, send_splits, recv_splits in res:
        np.testing.assert_array_equal(got, qv)
        assert n_halo == sum(recv_splits) > 0
        assert recv_splits[rank] == 0 and send_splits[rank] == 0
    assert sum(recv_total.values()) == sum(send_total.values())


@pytest.mark.parametrize("world", [1, 4])
def test_in_process_emulation_equals_single_device(world):
    """Every rank's plan built in one process, halo rows moved by exchange_in_process: same result as one device."""
    coords, _ = _small_scene()
    M = coords.shape[0]
    nmap_rm = ost.nmap_sorted(coords.numpy(), EXT)
    nmap_tm = torch.from_numpy(np.ascontiguousarray(nmap_rm.T))
    bounds = fused.shard_bounds(M, world)
    plans = fused.plans_in_process(nmap_tm, bounds)
    C = 8
    q0 = np.random.default_rng(2).integers(-127, 128, (M, C)).astype(np.int8)
    layers = _layers_np(2, C, 4)
    bufs = [p.local_buffer(C) for p in plans]
    for p, b, (lo, hi) in zip(plans, bufs, bounds):
        b[:p.n_own] = torch.from_numpy(q0[lo:hi])
    for layer in layers:
        fused.exchange_in_process(plans, bufs)
        for p, b in zip(plans, bufs):
            b[:p.n_own] = torch.from_numpy(_oracle_layer(b.numpy(), p.nmap.numpy().T, layer))
    got = np.concatenate([b[:p.n_own].numpy() for p, b in zip(plans, bufs)])
    want = q0
    for layer in layers:
        want = _oracle_layer(want, nmap_rm, layer)
    np.testing.assert_array_equal(got, want)
