"""Fused multi-frame scene (config 5) on the GPU: the scene's neighbour map from the hash builder equals the oracle's,
and a stack of tcgen05 int8 convs over Morton shards (ranks emulated in one process, halo rows moved between their
buffers exactly as the all-to-all does) equals the single-device stack over the whole voxel set bit for bit."""
import numpy as np
import pytest
import torch

from oracle import structure as ost
from promptmoge_b200 import fused

pytestmark = pytest.mark.gpu

EXT = [1, 1 << 21, 1 << 21, 1 << 21]


def _scene():
    coords, _ = fused.make_fused_scene(11, n_poses=6, H=60, W=80, voxel=0.02, device="cuda")
    return coords


def test_fused_scene_neighbour_map_matches_oracle():
    from promptmoge_b200 import ops
    coords = _scene()
    nm, mask, st = ops.nmap_hash(coords, EXT)
    assert int(st.item()) == 0
    want = ost.nmap_sorted(coords.cpu().numpy(), EXT)
    np.testing.assert_array_equal(nm.cpu().numpy()[:, :coords.shape[0]].T, want)


@pytest.mark.parametrize("world", [2, 5])
def test_sharded_gpu_layers_equal_single_device(world):
    from promptmoge_b200 import ops
    coords = _scene()
    M = coords.shape[0]
    nm, mask, st = ops.nmap_hash(coords, EXT)
    nm = nm[:, :M].contiguous()
    C = 32
    layers = fused.random_layers(3, C, seed=7, device="cuda")
    q0 = torch.randint(-127, 128, (M, C), dtype=torch.int8, generator=torch.Generator().manual_seed(3)).cuda()
    # single device
    want = q0.clone()
    full = fused.plans_in_process(nm, fused.shard_bounds(M, 1))[0]
    want = fused.run_layers(full, want, layers, fused.gpu_conv)
    # emulated shards
    bounds = fused.shard_bounds(M, world)
    plans = fused.plans_in_process(nm, bounds)
    bufs = [p.local_buffer(C) for p in plans]
    for p, b, (lo, hi) in zip(plans, bufs, bounds):
        b[:p.n_own] = q0[lo:hi]
    for layer in layers:
        fused.exchange_in_process(plans, bufs)
        outs = [fused.gpu_conv(b, p.nmap, p.mask, layer) for p, b in zip(plans, bufs)]
        for p, b, o in zip(plans, bufs, outs):
            b[:p.n_own] = o
    got = torch.cat([b[:p.n_own] for p, b in zip(plans, bufs)])
    torch.cuda.synchronize()
    assert sum(p.n_halo for p in plans) > 0
    assert torch.equal(got, want)
