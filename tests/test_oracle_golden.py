"""The oracle against the reference's own outputs (fixtures from tests/golden/make_golden.py).  CPU only."""
import numpy as np
import pytest

from conftest import sha
from oracle import fit as ofit
from oracle import refiner as oref
from oracle import structure as ost

SMALL = ["B_small", "A_small"]


def _pc_for_step(g, scene, step):
    """The point map the reference refined at `step` (its own refined logz of the previous step)."""
    pc = scene.point_coord.copy()
    for s in range(step):
        pc[..., 2] = (g[f"s{s}_logz_in"] + g[f"s{s}_delta"]).astype(np.float32)
    return pc


@pytest.mark.parametrize("name", SMALL)
def test_structure_bit_exact(golden, name):
    g = golden(name)
    scene = g.scene()
    factors = [2] * (len(ost_levels_widths(g)) - 1)
    for step in range(g.config["K"]):
        pc = _pc_for_step(g, scene, step)
        if step > 0:
            np.testing.assert_array_equal(pc[..., 2], g[f"s{step}_logz_in"])
        feats, coords, shape, _ = ost.voxelize(pc)
        assert tuple(shape[:4]) == tuple(g[f"s{step}_shape"])
        levels, pools = ost.build_levels(coords, shape, factors)
        for k, lv in enumerate(levels):
            np.testing.assert_array_equal(lv["coords"], g[f"s{step}_L{k}_coords"])
            np.testing.assert_array_equal(lv["nmap"], g[f"s{step}_L{k}_nmap"])
        for k, p in enumerate(pools):
            np.testing.assert_array_equal(p["parent"], g[f"s{step}_P{k}_parent"])
            np.testing.assert_array_equal(p["seg_indices"], g[f"s{step}_P{k}_seg_indices"])
            np.testing.assert_array_equal(p["seg_offsets"], g[f"s{step}_P{k}_seg_offsets"])


def ost_levels_widths(g):
    from promptmoge_b200 import synth
    return synth.MODELS[g.config["model"]]["model_channels"]


def test_column_and_sorted_backends_agree(golden):
    """The two reference nmap backends are exact and interchangeable at level 0 (_core.py:24-29)."""
    g = golden("A_small")
    _, coords, shape, _ = ost.voxelize(g.scene().point_coord)
    np.testing.assert_array_equal(ost.nmap_column(coords, shape[:4]), ost.nmap_sorted(coords, shape[:4]))


@pytest.mark.parametrize("name", SMALL)
def test_layer_accumulators_and_dequant(golden, name):
    """Given the reference's int8 input of each quantised layer, the oracle's int32 accumulators equal the reference
    operators' exact accumulators (SHA-256 over the whole tensor), and its dequantised output matches the reference
    fake-quant layer within 1e-3 relative."""
    g = golden(name)
    model = g.config["model"]
    widths = ost_levels_widths(g)
    qr = oref.QuantRefiner(g.weights(), g.clips, widths, [2] * (len(widths) - 1))
    levels_nmap = {}
    k = 0
    while f"s0_L{k}_nmap" in g:
        levels_nmap[k] = g[f"s0_L{k}_nmap"]
        k += 1
    names = g.layer_names(0)
    assert len(names) == (31 if model == "A" else 25)
    for n in names:
        key = f"s0_Q_{n}"
        q = g[key + "_q"]
        assert sha(q) == g.digests[key + "_q"]
        qw, sw = qr.qw[n]
        if ".conv" in n:
            M = q.shape[0]
            lv = _level_for_conv(n, widths)
            nmap = levels_nmap[lv]
            assert nmap.shape[0] == M
            acc = oref.conv_acc(q, nmap, qw)
        else:
            acc = oref.linear_acc(q, qw)
        acc32 = acc.astype(np.int32)
        assert np.array_equal(acc32.astype(np.int64), acc)
        assert sha(acc32) == g.digests[key + "_acc"], n
        rows = g[key + "_rows"]
        np.testing.assert_array_equal(acc32[rows], g[key + "_acc_rows"])
        y = oref.dequant(acc[rows], oref.act_scale(g.clips[n]), sw, qr.w[n + ".bias"])
        yr = g[key + "_y_rows"]
        rel = np.abs(y - yr).max() / max(np.abs(yr).max(), 1e-30)
        assert rel <= 1e-3, (n, rel)


@pytest.mark.parametrize("name", SMALL)
def test_seeded_conv_accumulators(golden, name):
    """Each conv layer on its seeded int8 input (synth.seeded_conv_input): the oracle's accumulators over the
    reference's neighbour maps hash to the reference's (the digests the GPU tests also check at full size)."""
    from promptmoge_b200 import synth
    g = golden(name)
    widths = ost_levels_widths(g)
    qr = oref.QuantRefiner(g.weights(), g.clips, widths, [2] * (len(widths) - 1))
    keys = sorted(k for k in g.digests if k.startswith("s0_S_"))
    assert len(keys) == (20 if g.config["model"] == "A" else 16)
    for key in keys:
        n = key[len("s0_S_"):-len("_acc")]
        nmap = g[f"s0_L{_level_for_conv(n, widths)}_nmap"]
        qw, _ = qr.qw[n]
        q = synth.seeded_conv_input(n, nmap.shape[0], qw.shape[-1])
        acc = oref.conv_acc(q, nmap, qw)
        assert sha(acc.astype(np.int32)) == g.digests[key], n


def _level_for_conv(name, widths):
    L = len(widths)
    if name.startswith("down_stages."):
        return int(name.split(".")[1])
    if name.startswith("bottleneck_stage"):
        return L - 1
    if name.startswith("up_stages."):
        return L - 2 - int(name.split(".")[1])
    raise ValueError(name)


@pytest.mark.parametrize("name", SMALL)
def test_fit_and_prompt_features(golden, name):
    g = golden(name)
    scene = g.scene()
    for step in range(g.config["K"]):
        pc = _pc_for_step(g, scene, step)
        pf, s, t = ofit.prompt_feats(pc[..., 2], scene.lidar_depth, scene.lidar_conf)
        st = g[f"s{step}_fit_st"]
        # The reference solves s = (n Sxy - Sx Sy) / (n Sxx - Sx^2) in fp32; the denominator cancels ~7 digits, so a
        # one-ulp change of any sum (summation order) moves s by ~1e-5 relative.  Tolerances reflect that
        # conditioning: 1e-4 relative on s and 1e-4 m on t (0.01 % of a metre-scale depth).
        np.testing.assert_allclose(s, st[:, 0], rtol=1e-4)
        np.testing.assert_allclose(t, st[:, 1], rtol=0, atol=1e-4)
        np.testing.assert_allclose(pf, g[f"s{step}_prompt_feats"], rtol=1e-3, atol=1e-4)


@pytest.mark.parametrize("name", SMALL)
def test_refine_step_end_to_end(golden, name):
    """The oracle's whole refine step against the reference's: structure bit-exact, refined depth within 0.2 %
    AbsRel-delta, and the per-pixel log-depth update within 2e-3 absolute."""
    g = golden(name)
    scene = g.scene()
    widths = ost_levels_widths(g)
    qr = oref.QuantRefiner(g.weights(), g.clips, widths, [2] * (len(widths) - 1))
    pc = scene.point_coord.copy()
    enc = scene.encoder_feature.astype(np.float32)
    for step in range(g.config["K"]):
        new_pc, info = oref.refine_step(qr, pc, scene.lidar_depth, scene.lidar_conf, enc, scene.uv_bias)
        ref_logz = (g[f"s{step}_logz_in"] + g[f"s{step}_delta"]).astype(np.float32)
        d_o, d_r = np.exp(new_pc[..., 2].astype(np.float64)), np.exp(ref_logz.astype(np.float64))
        absrel = np.mean(np.abs(d_o - d_r) / d_r)
        assert absrel < 2e-3, absrel
        assert np.abs(info["delta"].reshape(ref_logz.shape) - g[f"s{step}_delta"]).max() < 2e-3
        pc = new_pc
        pc[..., 2] = ref_logz          # continue from the reference's state, so each step is compared alone


@pytest.mark.parametrize("name", SMALL)
def test_final_fit(golden, name):
    g = golden(name)
    scene = g.scene()
    depth = np.exp(g["final_logz"].astype(np.float32)).astype(np.float32)
    d_lr = ofit.area_resize(depth, *scene.lidar_depth.shape[-2:])
    # exp() differs by an ulp between numpy and torch; the resampler itself is checked bit-exact against torch below.
    np.testing.assert_allclose(d_lr, g["final_d_lr"], rtol=1e-6)
    _, s, t = ofit.final_fit(depth, scene.lidar_depth, scene.lidar_conf)
    np.testing.assert_allclose(s, g["final_fit_st"][:, 0], rtol=1e-4)
    np.testing.assert_allclose(t, g["final_fit_st"][:, 1], rtol=0, atol=1e-4)


def test_conv_sweep_case(golden):
    g = golden("conv_20k_c32")
    from promptmoge_b200 import synth
    c = g.config
    coords = synth.make_surface_voxels(c["N"], c["seed"])
    shape = (1, 1 << 21, 1 << 21, 1 << 21)
    nmap = ost.nmap_sorted(coords, shape)
    assert sha(nmap) == str(g["nmap_sha"])
    rng = np.random.default_rng(c["seed"] + 100)
    q = rng.integers(-127, 128, (coords.shape[0], c["C"])).astype(np.int8)
    qw = rng.integers(-127, 128, (c["C"], 3, 3, 3, c["C"])).astype(np.int8)
    acc = oref.conv_acc(q, nmap, qw).astype(np.int32)
    assert sha(acc) == str(g["acc_sha"])


def test_trim_count_matches_torch():
    torch = pytest.importorskip("torch")
    counts = np.concatenate([np.arange(0, 5000), np.array([49152, 307200, 2 ** 24 - 3])])
    mask_sum = torch.from_numpy(counts.astype(np.int64))
    ref = ((1 - 0.2) * mask_sum).long().clamp_min(32).numpy()
    np.testing.assert_array_equal(ofit.trim_count(counts), ref)


@pytest.mark.parametrize("src,dst", [((192, 256), (480, 640)), ((192, 256), (240, 320)), ((192, 256), (48, 64)),
                                     ((192, 256), (384, 512)), ((192, 256), (32, 48))])
def test_resamplers_match_torch(src, dst):
    torch = pytest.importorskip("torch")
    F = torch.nn.functional
    rng = np.random.default_rng(0)
    x = rng.random((1, 1) + src).astype(np.float32)
    ref = F.interpolate(torch.from_numpy(x), dst, mode="nearest").numpy()
    np.testing.assert_array_equal(ofit.nearest_resize(x, *dst), ref)
    y = rng.random((1,) + dst).astype(np.float32)
    ref = F.interpolate(torch.from_numpy(y).unsqueeze(1), src, mode="area").squeeze(1).numpy()
    np.testing.assert_array_equal(ofit.area_resize(y, *src), ref)
