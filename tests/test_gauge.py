"""Polynomial prompt gauge (moge/model/v3.py:151-183): the numpy oracle against the reference's own outputs
(tests/golden/gauge.npz, made by tests/golden/make_gauge.py), and the GPU kernels against both."""
import sys
from pathlib import Path

import numpy as np
import pytest

sys.path.insert(0, str(Path(__file__).parent / "golden"))
from make_gauge import CASES, case, input_sha  # noqa: E402

from oracle import gauge as ogauge  # noqa: E402

GOLD = np.load(Path(__file__).parent / "golden" / "gauge.npz")


def _inputs(name):
    d, l, c, deg = case(*CASES[name])
    assert GOLD[f"{name}_inputs_sha"].item().decode() == input_sha(d, l, c), "synthetic inputs changed"
    return d, l, c, deg


@pytest.mark.parametrize("name", sorted(CASES))
def test_oracle_matches_reference(name):
    d, l, c, deg = _inputs(name)
    got = ogauge.prompt_gauge_poly(d, l, c, deg)
    # the reference solves in fp32 LAPACK, the oracle in float64: a few ulp
    np.testing.assert_allclose(got, GOLD[f"{name}_corr"], rtol=1e-6)


def test_too_few_points_means_no_correction():
    d, l, c, deg = _inputs("few")
    assert np.all(GOLD["few_corr"][0] == 1.0)
    _, ok, n = ogauge.gauge_coefficients(d, l, c, deg)
    assert not ok[0] and n[0] < 200 and ok[1]


def test_lower_median_and_linspace():
    assert ogauge.lower_median(np.array([4, 1, 3, 2], np.float32)) == 2
    ls = ogauge.linspace(5)
    assert ls.tolist() == [-1.0, -0.5, 0.0, 0.5, 1.0]


@pytest.mark.gpu
@pytest.mark.parametrize("name", sorted(CASES))
def test_gpu_gauge_matches_reference(name):
    import torch
    from promptmoge_b200 import ops
    d, l, c, deg = _inputs(name)
    pts = np.random.default_rng(0).standard_normal(d.shape + (3,)).astype(np.float32)
    pts_t = torch.from_numpy(pts).cuda()
    depth = torch.from_numpy(d).cuda()
    corr, out, coef = ops.gauge_poly(depth, torch.from_numpy(l).cuda(), torch.from_numpy(c).cuda(), degree=deg,
                                     points=pts_t)
    corr = corr.cpu().numpy()
    ref = GOLD[f"{name}_corr"]
    # fp64 normal equations vs the reference's fp32 least squares: ~1e-6 relative
    np.testing.assert_allclose(corr, ref, rtol=2e-5)
    _, ok, n = ogauge.gauge_coefficients(d, l, c, deg)
    cf = coef.cpu().numpy()
    np.testing.assert_array_equal(cf[:, 6] != 0, ok)
    np.testing.assert_array_equal(cf[:, 7].astype(np.int64), n)
    # applied in place / out of place exactly as depth * corr, points * corr in fp32
    np.testing.assert_array_equal(out.cpu().numpy(), (d * corr).astype(np.float32))
    np.testing.assert_array_equal(pts_t.cpu().numpy(), (pts * corr[..., None]).astype(np.float32))
    for b in range(d.shape[0]):
        if not ok[b]:
            assert np.all(corr[b] == 1.0)
