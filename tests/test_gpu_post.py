"""Post-refinement output on the GPU (csrc/post.cu through the C ABI) against the reference's recover_focal_shift
outputs (tests/golden/post.npz), torch's own bilinear resize, and the oracle composition of infer's output path
(resize + 'exp' remap, focal / shift, shifted depth, final LiDAR fit, point map, mask, gauge).  Tolerances: focal and
shift 2e-6 relative of the reference (its LM stops within ~1e-7 of the minimiser; the fixed-focal case 2e-3, where it
stops early); resize 1e-5 relative plus 4e-6 of the largest value (torch's CPU kernel orders the weighted terms
differently); end to end 1e-5 relative."""
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import fit as ofit
from oracle import gauge as ogauge
from oracle import post as opost

sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
import make_post as mp  # noqa: E402

pytestmark = pytest.mark.gpu
G = np.load(Path(__file__).resolve().parent / "golden" / "post.npz")


@pytest.mark.parametrize("name", list(mp.CASES))
def test_focal_shift_against_reference(name):
    from promptmoge_b200 import post
    pts, mask, focal = mp.case(name)
    f, s = post.recover_focal_shift(torch.from_numpy(pts).cuda(),
                                    None if mask is None else torch.from_numpy(mask).cuda(),
                                    None if focal is None else torch.from_numpy(focal).cuda())
    f, s = f.cpu().numpy(), s.cpu().numpy()
    of, os_ = opost.recover_focal_shift(pts, mask, focal)
    np.testing.assert_allclose(f, of, rtol=1e-6, atol=0)
    np.testing.assert_allclose(s, os_, rtol=1e-6, atol=1e-7)
    np.testing.assert_allclose(f, G[f"{name}_focal"], rtol=2e-6, atol=0)
    tol = 2e-3 if name == "focal_given" else 2e-6
    np.testing.assert_allclose(s, G[f"{name}_shift"], rtol=tol, atol=tol / 10)


def test_focal_shift_deterministic_and_batched():
    from promptmoge_b200 import post
    pts, mask, _ = mp.case("masked")
    t = torch.from_numpy(pts).cuda()
    m = torch.from_numpy(mask).cuda()
    a = post.recover_focal_shift(t, m)
    b = post.recover_focal_shift(t, m)
    one = post.recover_focal_shift(t[1:2], m[1:2])
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
    assert torch.equal(a[0][1:2], one[0]) and torch.equal(a[1][1:2], one[1])


@pytest.mark.parametrize("h,w,H,W", [(48, 64, 480, 640), (240, 320, 480, 640), (60, 80, 37, 53), (30, 40, 30, 40)])
def test_resize_remap_equals_torch(h, w, H, W):
    from promptmoge_b200 import post
    rng = np.random.default_rng(h + W)
    c = np.stack([rng.uniform(-1, 1, (2, h, w)), rng.uniform(-1, 1, (2, h, w)), rng.uniform(-0.5, 2, (2, h, w))],
                 -1).astype(np.float32)
    got = post.resize_remap(torch.from_numpy(c).cuda(), (H, W)).cpu().numpy()
    r = F.interpolate(torch.from_numpy(c).movedim(-1, -3), (H, W), mode="bilinear", align_corners=False,
                      antialias=False).movedim(-3, -1).numpy()
    want = opost.remap_exp(r)
    # torch's CPU kernel orders (and may fuse) the four weighted terms differently: a few ulps of the operands, which
    # near a sign change of x or y is a large relative error of a small result
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=4e-6 * float(np.abs(want).max()))


def _oracle_post(coords, H, W, ld, lc, mask, gauge):
    r = F.interpolate(torch.from_numpy(coords).movedim(-1, -3), (H, W), mode="bilinear", align_corners=False,
                      antialias=False).movedim(-3, -1).numpy()
    pts = opost.remap_exp(r)
    f, s = opost.recover_focal_shift(pts, mask)
    depth = (pts[..., 2] + s[:, None, None]).astype(np.float32)
    depth, fs, ft = ofit.final_fit(depth, ld, lc, None if mask is None else mask.astype(np.float32))
    fx, fy = zip(*[opost.focal_to_fxfy(np.float32(x), W, H) for x in f])
    points = opost.depth_to_points(depth, fx, fy)
    if mask is not None:
        m = mask & (depth > 0)
        points = np.where(m[..., None], points, np.inf).astype(np.float32)
        depth = np.where(m, depth, np.inf).astype(np.float32)
    if gauge:
        corr = ogauge.prompt_gauge_poly(depth, ld[:, 0], lc[:, 0], degree=2)
        depth = (depth * corr).astype(np.float32)
        points = (points * corr[..., None]).astype(np.float32)
    return points, depth, f, s, fs, ft


@pytest.mark.parametrize("masked,gauge", [(False, False), (True, False), (True, True)])
def test_postprocess_equals_oracle(masked, gauge):
    from promptmoge_b200 import post, synth
    sc = synth.make_scene(8, 240, 320, 8, 256, batch=2)
    coords = sc.point_coord.astype(np.float32)                   # (x/z, y/z, log z) at the refiner's grid
    H, W = 480, 640
    mask = None
    if masked:
        rng = np.random.default_rng(3)
        mask = np.ones((2, H, W), bool)
        mask[:, :40] = False
        mask[1, rng.random((H, W)) < 0.05] = False
    out = post.postprocess(torch.from_numpy(coords).cuda(), (H, W), torch.from_numpy(sc.lidar_depth).cuda(),
                           torch.from_numpy(sc.lidar_conf).cuda(),
                           None if mask is None else torch.from_numpy(mask).cuda(), gauge_poly=2 if gauge else 0)
    points, depth, f, s, fs, ft = _oracle_post(coords, H, W, sc.lidar_depth, sc.lidar_conf, mask, gauge)
    np.testing.assert_allclose(out["focal"].cpu().numpy(), f, rtol=1e-6)
    np.testing.assert_allclose(out["shift"].cpu().numpy(), s, rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(out["metric_fit"].cpu().numpy()[:, 0], fs, rtol=1e-4)
    d = out["depth"].cpu().numpy()
    assert np.array_equal(np.isinf(d), np.isinf(depth))
    fin = np.isfinite(depth)
    np.testing.assert_allclose(d[fin], depth[fin], rtol=1e-4 if gauge else 1e-5)
    p = out["points"].cpu().numpy()
    np.testing.assert_allclose(p[fin], points[fin], rtol=1e-4 if gauge else 1e-5, atol=1e-6)
    K = out["intrinsics"].cpu().numpy()
    assert K.shape == (2, 3, 3) and np.allclose(K[:, :2, 2], 0.5)


def test_post_graph_equals_eager():
    from promptmoge_b200 import post, synth
    sc = synth.make_scene(9, 240, 320, 8, 256, batch=1)
    c = torch.from_numpy(sc.point_coord.astype(np.float32)).cuda()
    ld, lc = torch.from_numpy(sc.lidar_depth).cuda(), torch.from_numpy(sc.lidar_conf).cuda()
    eager = post.postprocess(c, (480, 640), ld, lc)
    pg = post.PostGraph(1, (240, 320), (480, 640))
    for _ in range(2):
        got = pg.run(c, ld, lc)
        for k in ("points", "depth", "focal", "shift", "metric_fit"):
            assert torch.equal(got[k], eager[k]), k
