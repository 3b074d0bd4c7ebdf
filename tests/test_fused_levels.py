"""A fused scene sharded without a global view (every rank back-projects its own poses; voxels go to their Morton-range
owners; neighbours across a boundary are looked up at their owner; coarser levels are parents, code >> 3) and the
sharded U-Net encoder over it (halo exchange before every conv, children moved to their parent's owner before the
mean pool), on the CPU with gloo at world sizes 2 and 3: every level's structure and every level's int8
output equal the single-rank run voxel by voxel.  The per-layer arithmetic is the oracle's."""
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
from promptmoge_b200.dist import frame_range

WIDTHS = [16, 32, 32]
POSES = 6
EXT = [1, 1 << 21, 1 << 21, 1 << 21]


def _layout():
    return fused.scene_layout(5, POSES, (4.0, 4.0, 3.0))


def _codes(pose_ids):
    return fused.scene_codes(5, _layout(), pose_ids, H=12, W=16, voxel=0.05)


def nmap_cpu(coords, ext):
    nm = ost.nmap_sorted(coords.numpy(), ext)
    return torch.from_numpy(np.ascontiguousarray(nm.T)).to(torch.int32)


def conv_cpu(q_local, nmap, mask, layer):
    w, ws, b, sa, s_out = layer
    Co, Ci = w.shape[1], w.shape[2]
    qw = w.permute(1, 0, 2).reshape(Co, 3, 3, 3, Ci).numpy()
    acc = oref.conv_acc(q_local.numpy(), nmap.t().contiguous().numpy(), qw).astype(np.int64)
    y = oref.dequant(acc, np.float32(sa), ws.numpy(), b.numpy())
    return torch.from_numpy(np.clip(np.rint(oref.silu(y) / np.float32(s_out)), -127, 127).astype(np.int8))


def link_cpu(pooled, layer):
    w, ws, b, sa, s_out = layer
    qp = np.clip(np.rint(pooled.numpy() / np.float32(sa)), -127, 127).astype(np.int8)
    y = oref.dequant(oref.linear_acc(qp, w.numpy()), np.float32(sa), ws.numpy(), b.numpy())
    return torch.from_numpy(np.clip(np.rint(oref.silu(y) / np.float32(s_out)), -127, 127).astype(np.int8))


def _run(local_codes, group, overlap=False, aligned=False):
    levels = fused.build_levels(local_codes, len(WIDTHS), nmap_cpu, group, aligned=aligned)
    convs, links = fused.encoder_layers(WIDTHS, 2, seed=9, device="cpu")
    rng = np.random.default_rng(17)
    n0 = levels[0].offset
    # level-0 input: a deterministic function of the voxel's global index
    g_all = torch.from_numpy(rng.integers(-127, 128, (200000, WIDTHS[0])).astype(np.int8))
    q0 = g_all[n0:n0 + levels[0].plan.n_own]
    outs = fused.encoder_forward(levels, q0, convs, links, conv_cpu, link_cpu, group, overlap=overlap)
    return levels, outs


def fused_pools(levels):
    return [fused.PoolPlan(levels[k], levels[k + 1], None) for k in range(len(levels) - 1)]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=120))
    try:
        b, e = frame_range(POSES, rank, world)
        levels, outs = _run(_codes(range(b, e)), None)
        _, plain = _run(_codes(range(b, e)), None, overlap=True)      # exchanges beside the interior rows' conv
        assert all(torch.equal(a, p) for a, p in zip(outs, plain))
        # every level balanced on its own count (the default run above): parents of whole child groups pooled where
        # the children are; the aligned ranges (coarser levels cut at the parents of level 0's boundaries) as well
        lv_b = levels
        _, outs_b = _run(_codes(range(b, e)), None, aligned=True)
        n_pooled = sum(pp.n_pool_send for pp in fused_pools(lv_b))
        # numpy arrays travel by value: shared-memory tensors would need this process alive while the parent reads
        q.put((rank, [l.codes.numpy() for l in levels], [l.offset for l in levels], [o.numpy() for o in outs],
               [l.plan.n_halo for l in levels], [l.plan.n_int for l in levels], [o.numpy() for o in outs_b],
               n_pooled))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_levels_and_encoder_equal_single_rank(world):
    whole = _codes(range(POSES))
    ref_levels, ref_outs = _run(whole, fused.LOCAL)
    assert len(ref_levels) == len(WIDTHS) and all(l.plan.n_halo == 0 for l in ref_levels)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted((q.get(timeout=300) for _ in range(world)), key=lambda r: r[0])
    res = [(r[0], [torch.from_numpy(c) for c in r[1]], r[2], [torch.from_numpy(o) for o in r[3]], r[4], r[5],
            [torch.from_numpy(o) for o in r[6]], r[7]) for r in res]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert sum(r[4][0] for r in res) > 0                      # the shards really exchanged halo rows
    assert all(0 < r[5][0] < r[1][0].numel() for r in res)     # level 0 has interior and boundary rows on every rank
    for k in range(len(WIDTHS)):
        codes = torch.cat([r[1][k] for r in res])
        assert torch.equal(codes, ref_levels[k].codes), k     # ranges partition the level in Morton order
        assert [r[2][k] for r in res] == list(np.cumsum([0] + [r[1][k].numel() for r in res])[:-1])
        out = torch.cat([r[3][k] for r in res])
        assert torch.equal(out, ref_outs[k]), k
        # per-level balanced ranges (pooled rows and boundary children move between ranks): the same outputs
        assert torch.equal(torch.cat([r[6][k] for r in res]), ref_outs[k]), k
    assert sum(r[7] for r in res) > 0                          # some parents were pooled on another rank than theirs


def test_single_rank_levels_are_the_global_structure():
    """One rank: level 0 holds every back-projected voxel, its neighbour map is the oracle's over the whole set, and
    each coarser level is the set of parents (code >> 3)."""
    whole = _codes(range(POSES))
    levels = fused.build_levels(whole, len(WIDTHS), nmap_cpu, fused.LOCAL)
    assert torch.equal(levels[0].codes, whole)
    np.testing.assert_array_equal(levels[0].plan.nmap.t().numpy(),
                                  ost.nmap_sorted(fused.coords_of_codes(whole).numpy(), EXT))
    for k in range(1, len(WIDTHS)):
        assert torch.equal(levels[k].codes, torch.unique(levels[k - 1].codes >> 3))
