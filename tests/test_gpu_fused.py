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
    for i, layer in enumerate(layers):
        fused.exchange_in_process(plans, bufs)
        outs = [fused.gpu_conv(b, p.nmap, p.mask, layer) for p, b in zip(plans, bufs)]
        # the overlapped form (ShardPlan.conv): interior rows, then boundary rows, written back in row order
        for p, b, o in zip(plans, bufs, outs):
            parts = [fused.gpu_conv(b, p.nmap_int, p.mask_int, layer), fused.gpu_conv(b, p.nmap_bnd, p.mask_bnd, layer)]
            split = torch.empty_like(o)
            split.index_copy_(0, p.perm, torch.cat(parts))
            assert torch.equal(split, o), i
        for p, b, o in zip(plans, bufs, outs):
            b[:p.n_own] = o
    got = torch.cat([b[:p.n_own] for p, b in zip(plans, bufs)])
    torch.cuda.synchronize()
    assert sum(p.n_halo for p in plans) > 0
    assert all(0 < p.n_int < p.n_own for p in plans)
    assert torch.equal(got, want)


def test_sharded_levels_on_device_equal_oracle_structure():
    """The sharded level build as the only rank on the GPU (hash neighbour maps): every level's voxels are the parents
    of the level below, every neighbour map equals the oracle's over that level, and the encoder's level-0 output
    equals the oracle's conv arithmetic (up to one-step SiLU requantise flips from CUDA's exp)."""
    import numpy as np
    from oracle import structure as ost
    from promptmoge_b200 import fused, ops
    from test_fused_levels import conv_cpu
    layout = fused.scene_layout(11, 6)
    codes = fused.scene_codes(11, layout, range(6), H=60, W=80, voxel=0.02, device="cuda")

    def nmap_fn(coords, ext):
        nm, _, st = ops.nmap_hash(coords, ext)
        assert int(st.item()) == 0
        return nm

    widths = [32, 64, 128]
    levels = fused.build_levels(codes, len(widths), nmap_fn, fused.LOCAL)
    ext = [1, 1 << 21, 1 << 21, 1 << 21]
    for k, lv in enumerate(levels):
        if k:
            assert torch.equal(lv.codes, torch.unique(levels[k - 1].codes >> 3))
        want = ost.nmap_sorted(fused.coords_of_codes(lv.codes).cpu().numpy(), ext)
        np.testing.assert_array_equal(lv.plan.nmap.t().cpu().numpy(), want)
    convs, links = fused.encoder_layers(widths, 2, seed=3, device="cuda")
    q0 = torch.randint(-127, 128, (levels[0].plan.n_own, widths[0]), dtype=torch.int8,
                       generator=torch.Generator().manual_seed(1)).cuda()
    outs = fused.encoder_forward(levels, q0, convs, links, fused.gpu_conv, fused.gpu_link, fused.LOCAL)
    assert [o.shape[0] for o in outs] == [lv.plan.n_own for lv in levels]
    cpu_layers = [tuple(t.cpu() if torch.is_tensor(t) else t for t in layer) for layer in convs[0]]
    q = q0.cpu()
    nm = levels[0].plan.nmap.cpu()
    for layer in cpu_layers:
        q = conv_cpu(q, nm, None, layer)
    d = (outs[0].cpu().to(torch.int32) - q.to(torch.int32)).abs()
    assert int(d.max()) <= 1 and float((d > 0).float().mean()) < 1e-3
