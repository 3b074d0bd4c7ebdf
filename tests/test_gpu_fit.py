"""The robust metric fit on the GPU against the oracle and the reference fixtures."""
import numpy as np
import pytest
import torch

from oracle import fit as ofit

pytestmark = pytest.mark.gpu


def _fit_np(z, y, m, trace):
    return ofit.fit_scale_shift(z, y, m, trace=trace)


@pytest.mark.parametrize("name", ["B_small", "A_small", "B_full", "A_full"])
def test_prompt_fit_and_features(golden, name):
    from promptmoge_b200 import ops
    g = golden(name)
    sc = g.scene()
    pc = torch.from_numpy(sc.point_coord).cuda()
    ld = torch.from_numpy(sc.lidar_depth).cuda()
    lc = torch.from_numpy(sc.lidar_conf).cuda()
    z, y, fl = ops.fit_prep_prompt(pc, ld, lc)
    st = ops.fit_solve(z, y, fl)
    torch.cuda.synchronize()
    s = ops.fit_state_view(st)[0]
    # the oracle on the GPU's own prepared inputs: same trims, same solution (fp64 sums -> fp32)
    zn, yn, fn = z.cpu().numpy(), y.cpu().numpy(), fl.cpu().numpy()
    B, H, W = sc.point_coord.shape[:3]
    d = ofit.nearest_resize(sc.lidar_depth, H, W)[:, 0].reshape(B, -1)
    np.testing.assert_array_equal(yn, d)
    c = np.clip(ofit.nearest_resize(sc.lidar_conf, H, W)[:, 0] / np.float32(2), 0, 1).reshape(B, -1)
    np.testing.assert_array_equal((fn & 2) > 0, np.isfinite(d) & (d > 0) & (c >= np.float32(0.999)))
    trace = []
    so, to = _fit_np(zn, yn, (fn & 2) > 0, trace)
    assert s["thr"] == trace[-2][2][0]
    assert s["s"] == so[0] and s["t"] == to[0]
    # against the reference's own fit (fp32 sums; the 2x2 solve cancels ~7 digits, see test_oracle_golden)
    st_ref = g["s0_fit_st"][0]
    assert abs(s["s"] - st_ref[0]) <= 1e-4 * abs(st_ref[0])
    assert abs(s["t"] - st_ref[1]) <= 1e-4
    logz = pc[..., 2].contiguous()
    pf = ops.prompt_feats(logz, ld, lc, st).cpu().numpy()
    pf_o, _, _ = ofit.prompt_feats(sc.point_coord[..., 2], sc.lidar_depth, sc.lidar_conf)
    np.testing.assert_allclose(pf, pf_o, rtol=1e-3, atol=1e-4)
    if name.endswith("small"):
        np.testing.assert_allclose(pf, g["s0_prompt_feats"], rtol=1e-3, atol=1e-4)


@pytest.mark.parametrize("name", ["B_small", "A_small"])
def test_final_fit(golden, name):
    from promptmoge_b200 import ops
    g = golden(name)
    sc = g.scene()
    depth_np = np.exp(g["final_logz"].astype(np.float32)).astype(np.float32)
    depth = torch.from_numpy(depth_np).cuda()
    ld = torch.from_numpy(sc.lidar_depth).cuda()
    lc = torch.from_numpy(sc.lidar_conf).cuda()
    z, y, fl = ops.fit_prep_final(depth, ld, lc)
    np.testing.assert_array_equal(z.cpu().numpy().reshape(sc.lidar_depth.shape[0], 192, 256),
                                  ofit.area_resize(depth_np, 192, 256))
    st = ops.fit_solve(z, y, fl)
    s = ops.fit_state_view(st)[0]
    _, so, to = ofit.final_fit(depth_np, sc.lidar_depth, sc.lidar_conf)
    assert s["s"] == so[0] and s["t"] == to[0]
    out = ops.apply_affine(depth.clone(), st).cpu().numpy()
    np.testing.assert_array_equal(out, (np.float32(s["s"]) * depth_np + np.float32(s["t"])).astype(np.float32))


def test_fit_edge_cases():
    """Fewer than min_points masked -> (1, 0); all masked; a frame batch with different counts per frame."""
    from promptmoge_b200 import ops
    rng = np.random.default_rng(0)
    B, N = 3, 5000
    z = rng.uniform(0.5, 4, (B, N)).astype(np.float32)
    y = (1.7 * z + 0.3 + 0.01 * rng.standard_normal((B, N))).astype(np.float32)
    m = np.zeros((B, N), bool)
    m[0, :20] = True          # < 32 points: no fit
    m[1] = True               # everything
    m[2, ::3] = True
    fl = torch.from_numpy((m.astype(np.uint8) * 3)).cuda()
    st = ops.fit_solve(torch.from_numpy(z).cuda(), torch.from_numpy(y).cuda(), fl)
    got = ops.fit_state_view(st)
    so, to = ofit.fit_scale_shift(z, y, m)
    for b in range(B):
        assert got[b]["s"] == so[b] and got[b]["t"] == to[b], b
    assert got[0]["s"] == 1.0 and got[0]["t"] == 0.0 and got[0]["ok"] == 0
