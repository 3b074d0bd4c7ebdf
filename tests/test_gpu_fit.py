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


def _fused_vs_multi(pc, ld, lc, soft=True):
    from promptmoge_b200 import ops
    st_f, pf_f = ops.fit_prompt_fused(pc[..., 2], ld, lc, soft_gate=soft)
    z, y, fl = ops.fit_prep_prompt(pc, ld, lc)
    st_m = ops.fit_solve(z, y, fl)
    pf_m = ops.prompt_feats(pc[..., 2].contiguous(), ld, lc, st_m, soft_gate=soft)
    torch.cuda.synchronize()
    return ops.fit_state_view(st_f), pf_f, ops.fit_state_view(st_m), pf_m


@pytest.mark.parametrize("name", ["B_small", "A_small", "B_full", "A_full"])
def test_one_launch_fit_equals_multi_launch_fit(golden, name):
    """The 16-CTA cluster fit (one launch: prep, 4 trimmed iterations, prompt features) reaches the multi-launch
    fit's state and prompt features bit for bit, and the reference's (s, t)."""
    g = golden(name)
    sc = g.scene()
    pc = torch.from_numpy(sc.point_coord).cuda()
    ld = torch.from_numpy(sc.lidar_depth).cuda()
    lc = torch.from_numpy(sc.lidar_conf).cuda()
    f, pf_f, m, pf_m = _fused_vs_multi(pc, ld, lc)
    for key in ("s", "t", "thr", "count", "k", "ok"):
        assert f[0][key] == m[0][key], key
    assert f[0]["sums"] == m[0]["sums"]
    assert torch.equal(pf_f, pf_m)
    st_ref = g["s0_fit_st"][0]
    assert abs(f[0]["s"] - st_ref[0]) <= 1e-4 * abs(st_ref[0]) and abs(f[0]["t"] - st_ref[1]) <= 1e-4


def test_one_launch_fit_batch_and_edge_cases():
    """Three frames in one launch (three clusters): an ordinary frame, one with fewer than 32 confident pixels
    (no fit: s = 1, t = 0), and one where every pixel is confident; each equals the multi-launch fit, hard and soft
    gate."""
    from promptmoge_b200 import synth
    scs = [synth.make_scene(s, 120, 160, 8, 256) for s in (51, 52, 53)]
    pc = torch.from_numpy(np.concatenate([s.point_coord for s in scs])).cuda()
    ld = np.concatenate([s.lidar_depth for s in scs])
    lc = np.concatenate([s.lidar_conf for s in scs])
    lc[1] = 0.0
    lc[1, 0, 0, :10] = 2.0
    lc[2] = 2.0
    ld[2] = np.where(ld[2] > 0, ld[2], 1.5)
    ld, lc = torch.from_numpy(ld).cuda(), torch.from_numpy(lc).cuda()
    for soft in (True, False):
        f, pf_f, m, pf_m = _fused_vs_multi(pc, ld, lc, soft)
        for b in range(3):
            for key in ("s", "t", "thr", "count", "k", "ok"):
                assert f[b][key] == m[b][key], (b, key)
        assert f[1]["ok"] == 0 and f[1]["s"] == 1.0 and f[1]["t"] == 0.0
        assert torch.equal(pf_f, pf_m)


def test_one_launch_fit_refuses_frames_beyond_its_shared_memory():
    from promptmoge_b200 import _lib
    lib = _lib.load()
    t = torch.zeros(8, dtype=torch.float32, device="cuda")
    st = torch.zeros((1, 18), dtype=torch.int32, device="cuda")
    # 4096 x 4096 pixels: a 1,048,576-pixel slice per CTA (4 MB of residuals) cannot sit in shared memory
    ws = torch.empty(lib.pmg_fit_prompt_fused_workspace_bytes(1, 4096, 4096), dtype=torch.uint8, device="cuda")
    rc = lib.pmg_fit_prompt_fused(t.data_ptr(), 1, t.data_ptr(), t.data_ptr(), 1, 4096, 4096, 192, 256, 4, 0.2, 32, 1,
                                  st.data_ptr(), t.data_ptr(), None, None, ws.data_ptr(), ws.numel(), None)
    assert rc == 5      # PMG_ERR_UNSUPPORTED, nothing launched
