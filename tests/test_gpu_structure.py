"""Voxelisation, dedup and neighbour maps on the GPU against the oracle and the reference's own fixtures:
bit-exact coordinates, neighbour maps, parents and CSR segments."""
import numpy as np
import pytest
import torch

from conftest import sha

pytestmark = pytest.mark.gpu

SMALL = ["B_small", "A_small"]


def _widths(g):
    from promptmoge_b200 import synth
    return synth.MODELS[g.config["model"]]["model_channels"]


def _pc_for_step(g, scene, step):
    pc = scene.point_coord.copy()
    for s in range(step):
        pc[..., 2] = (g[f"s{s}_logz_in"] + g[f"s{s}_delta"]).astype(np.float32)
    return pc


def _levels(pc_np, L):
    from promptmoge_b200.levels import build_levels
    pc = torch.from_numpy(pc_np).cuda()
    lv, pools = build_levels(pc, L)
    torch.cuda.synchronize()
    return lv, pools


@pytest.mark.parametrize("name", SMALL)
def test_levels_match_reference_fixture(golden, name):
    g = golden(name)
    scene = g.scene()
    L = len(_widths(g))
    for step in range(g.config["K"]):
        lv, pools = _levels(_pc_for_step(g, scene, step), L)
        for k in range(L):
            np.testing.assert_array_equal(lv[k]["coords"].cpu().numpy(), g[f"s{step}_L{k}_coords"], err_msg=f"L{k}")
            np.testing.assert_array_equal(lv[k]["nmap"].cpu().numpy(), g[f"s{step}_L{k}_nmap"], err_msg=f"L{k}")
        for k, p in enumerate(pools):
            for key in ("parent", "seg_indices", "seg_offsets"):
                ref = g[f"s{step}_P{k}_{key}"]
                np.testing.assert_array_equal(p[key].cpu().numpy().astype(ref.dtype), ref, err_msg=f"P{k} {key}")


@pytest.mark.parametrize("name", ["B_full", "A_full"])
def test_full_size_levels_match_reference_digests(golden, name):
    """At the benchmark sizes (240x320, 480x640) every level array hashes to the reference's SHA-256."""
    g = golden(name)
    scene = g.scene()
    L = len(_widths(g))
    lv, pools = _levels(scene.point_coord, L)
    for k in range(L):
        assert sha(lv[k]["coords"].cpu().numpy().astype(np.int32)) == g.digests[f"s0_L{k}_coords"], f"L{k} coords"
        assert sha(np.ascontiguousarray(lv[k]["nmap"].cpu().numpy())) == g.digests[f"s0_L{k}_nmap"], f"L{k} nmap"
    for k, p in enumerate(pools):
        assert sha(p["parent"].cpu().numpy()) == g.digests[f"s0_P{k}_parent"]
        assert sha(p["seg_indices"].cpu().numpy()) == g.digests[f"s0_P{k}_seg_indices"]
        assert sha(p["seg_offsets"].cpu().numpy().astype(np.int64)) == g.digests[f"s0_P{k}_seg_offsets"]


def test_tile_masks_are_the_or_of_occupied_taps(golden):
    g = golden("A_small")
    lv, _ = _levels(g.scene().point_coord, 5)
    for l in lv:
        nm = l["nmap"].cpu().numpy()
        M = nm.shape[0]
        occ = (nm >= 0)
        bits = (occ * (1 << np.arange(27))).astype(np.int64)
        for t in range((M + 31) // 32):
            want = int(np.bitwise_or.reduce(bits[t * 32:(t + 1) * 32].ravel()))
            assert int(l["mask"][t].item()) & 0x7FFFFFF == want


@pytest.mark.parametrize("name", ["conv_20k_c32", "conv_100k_c16"])
def test_hash_nmap_matches_reference(golden, name):
    """Generic voxel sets (surface shells in a 2^21 grid): the hash neighbour map equals the reference's."""
    from promptmoge_b200 import ops, synth
    g = golden(name)
    c = g.config
    coords = torch.from_numpy(synth.make_surface_voxels(c["N"], c["seed"])).cuda()
    ext = [1, 1 << 21, 1 << 21, 1 << 21]
    nmap_rm, _, st = ops.nmap_hash(coords, ext, row_major=True)
    nmap_tm, mask, st2 = ops.nmap_hash(coords, ext, row_major=False)
    torch.cuda.synchronize()
    assert int(st.item()) == 0 and int(st2.item()) == 0
    a = nmap_rm.cpu().numpy()
    assert sha(a) == str(g["nmap_sha"])
    np.testing.assert_array_equal(nmap_tm.cpu().numpy().T, a)


def test_hash_nmap_equals_frame_nmap_on_refiner_levels(golden):
    """The generic hash builder and the column builder agree on every refiner level (and with the oracle)."""
    from promptmoge_b200 import ops
    from oracle import structure as ost
    g = golden("A_small")
    lv, _ = _levels(g.scene().point_coord, 5)
    for k, l in enumerate(lv):
        coords = l["coords"].contiguous()
        c = coords.cpu().numpy()
        ext = [int(c[:, 0].max()) + 1, l["H"], l["W"], int(c[:, 3].max()) + 1]
        nm, _, st = ops.nmap_hash(coords, ext, row_major=True)
        torch.cuda.synchronize()
        assert int(st.item()) == 0
        np.testing.assert_array_equal(nm.cpu().numpy(), l["nmap"].cpu().numpy())
        np.testing.assert_array_equal(nm.cpu().numpy(), ost.nmap_sorted(c, ext))


def test_hash_nmap_range_errors_are_reported(golden):
    from promptmoge_b200 import ops
    coords = torch.tensor([[0, 1, 2, 3], [0, 5, 2, 3], [0, 99, 0, 0]], dtype=torch.int32).cuda()
    nm, _, st = ops.nmap_hash(coords, [1, 16, 16, 16], row_major=True)
    torch.cuda.synchronize()
    assert int(st.item()) == 6          # PMG_ERR_RANGE: x = 99 outside the 16-wide grid


def test_pool_overflow_sets_status_and_stays_in_bounds(golden):
    from promptmoge_b200 import ops
    g = golden("B_small")
    pc = torch.from_numpy(g.scene().point_coord).cuda()
    B, H, W, _ = pc.shape
    zq, zmin, zmax, _, _ = ops.voxelize_l0(pc)
    p = ops.pool_frames(B, H, W, None, zq, zmin, cap=64)
    torch.cuda.synchronize()
    assert int(p["status"].item()) == 4            # PMG_ERR_OVERFLOW
    assert int(p["count"][0].item()) == 64
    assert int(p["count"][1].item()) > 64
    par = p["parent"].cpu().numpy()
    assert par.min() >= 0 and par.max() < 64
