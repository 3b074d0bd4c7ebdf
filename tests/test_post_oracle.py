"""The post-refinement oracle (oracle/post.py) against the reference's own recover_focal_shift and
normalized_view_plane_uv outputs (tests/golden/post.npz, made by tests/golden/make_post.py), and torch.linspace."""
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import fit as ofit
from oracle import post as opost

sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
import make_post as mp  # noqa: E402

G = np.load(Path(__file__).resolve().parent / "golden" / "post.npz")


@pytest.mark.parametrize("name", [n for n in mp.CASES if n != "focal_given"])
def test_focal_shift_matches_reference(name):
    pts, mask, focal = mp.case(name)
    f, s = opost.recover_focal_shift(pts, mask, focal)
    np.testing.assert_allclose(f, G[f"{name}_focal"], rtol=2e-6, atol=0)
    np.testing.assert_allclose(s, G[f"{name}_shift"], rtol=2e-6, atol=2e-7)


def test_focal_given_shift_near_reference():
    """With a fixed focal the reference's scipy LM stops at ftol 1e-3 short of the minimiser; the oracle returns the
    minimiser, within 2e-3 of the reference's shift, and its cost is never higher."""
    pts, mask, focal = mp.case("focal_given")
    f, s = opost.recover_focal_shift(pts, mask, focal)
    np.testing.assert_array_equal(f, G["focal_given_focal"])
    np.testing.assert_allclose(s, G["focal_given_shift"], rtol=0, atol=2e-3)
    uv = opost.normalized_view_plane_uv(pts.shape[2], pts.shape[1])
    hi, wi = ofit.nearest_index(64, pts.shape[1]), ofit.nearest_index(64, pts.shape[2])
    for b in range(pts.shape[0]):
        p = pts[b][hi][:, wi].reshape(-1, 3).astype(np.float64)
        u = uv[hi][:, wi].reshape(-1, 2).astype(np.float64)

        def cost(sh):
            return float(((focal[b] * p[:, :2] / (p[:, 2:] + sh) - u) ** 2).sum())
        assert cost(float(s[b])) <= cost(float(G["focal_given_shift"][b])) + 1e-12


@pytest.mark.parametrize("w,h", mp.UV_SIZES)
def test_view_plane_uv_bit_exact(w, h):
    np.testing.assert_array_equal(opost.normalized_view_plane_uv(w, h), G[f"uv_{w}x{h}"])


def test_linspace_fma_form_equals_torch():
    rng = np.random.default_rng(0)
    for _ in range(200):
        n = int(rng.integers(1, 700))
        a = float(rng.uniform(-3, 3))
        b = float(rng.uniform(-3, 3))
        np.testing.assert_array_equal(ofit.linspace_f32(a, b, n),
                                      torch.linspace(a, b, n, dtype=torch.float32).numpy())


def test_depth_to_points_conventions():
    d = np.full((1, 4, 6), 2.0, np.float32)
    fx, fy = opost.focal_to_fxfy(np.float32(1.2), 6, 4)
    p = opost.depth_to_points(d, [fx], [fy])
    assert p.shape == (1, 4, 6, 3)
    # the principal point sits between the two central pixel columns / rows: symmetric x, y
    np.testing.assert_allclose(p[0, :, :, 0], -p[0, :, ::-1, 0], rtol=1e-6)
    np.testing.assert_allclose(p[0, :, :, 1], -p[0, ::-1, :, 1], rtol=1e-6)
    assert (p[0, :, 3:, 0] > 0).all() and (p[0, 2:, :, 1] > 0).all()
    np.testing.assert_array_equal(p[..., 2], d)
