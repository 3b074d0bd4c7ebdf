"""Oracle (test infrastructure): the per-frame polynomial prompt gauge in numpy.

Restates MoGeModel.prompt_gauge_poly (moge/model/v3.py:151-183): the prediction's depth is area-averaged onto the
sensor grid over finite positive pixels only (two area resamplings, v3.py:156-158), the log ratio
log(lidar) - log(z_lr) on confident pixels (conf >= 2, lidar > 0, z_lr > 0; at least 200 of them, v3.py:170-172) is
fitted by a degree-1 (1, u, v) or degree-2 (1, u, v, u^2, uv, v^2) polynomial over u, v = linspace(-1, 1) of the
sensor grid with three iteratively reweighted least-squares solves (weights min(2 * 1.4826 * median|r| / |r|, 1),
the median being torch's lower median, v3.py:175-177), and the correction is exp(poly) over the image grid
(v3.py:178-182); a frame with too few points or a non-finite solution gets 1.

Elementwise steps are fp32 in the reference's order; each least-squares solve is done in float64 (numpy lstsq), where
the reference solves the fp32 system with LAPACK; the two agree to ~1e-6 relative, which the tests' tolerances cover.
Parity is pinned by tests/golden/gauge.npz (the reference's own outputs, tests/golden/make_gauge.py).
"""
from __future__ import annotations

import numpy as np

from .fit import area_resize, linspace_f32

f32 = np.float32


def linspace(n: int) -> np.ndarray:
    """torch.linspace(-1, 1, n) in fp32 (fused multiply-add form, see fit.linspace_f32)."""
    return linspace_f32(-1.0, 1.0, n)


def basis(uu: np.ndarray, vv: np.ndarray, degree: int) -> np.ndarray:
    cols = [np.ones_like(uu), uu, vv]
    if degree >= 2:
        cols += [(uu * uu).astype(f32), (uu * vv).astype(f32), (vv * vv).astype(f32)]
    return np.stack(cols, -1).astype(f32)


def lower_median(x: np.ndarray) -> f32:
    """torch.median: the lower of the two middle values for an even count."""
    return f32(np.partition(x, (x.size - 1) // 2)[(x.size - 1) // 2])


def gauge_coefficients(depth: np.ndarray, lidar: np.ndarray, conf: np.ndarray | None, degree: int = 2,
                       iters: int = 3):
    """Per frame: (coef [B, 3 or 6] float64, ok [B] bool, n [B] confident pixels)."""
    depth = depth.astype(f32)
    B, H, W = depth.shape
    h, w = lidar.shape[-2:]
    ok = np.isfinite(depth) & (depth > 0)
    num = area_resize(np.where(ok, depth, f32(0)).astype(f32), h, w)
    den = area_resize(ok.astype(f32), h, w)
    z_lr = np.where(den > f32(0.5), (num / np.maximum(den, f32(1e-6))).astype(f32), f32(0)).astype(f32)
    ld = lidar.reshape(B, h, w).astype(f32)
    cf = conf.reshape(B, h, w).astype(f32) if conf is not None else np.full_like(ld, 2.0)
    vv, uu = np.meshgrid(linspace(h), linspace(w), indexing="ij")
    Bm = basis(uu, vv, degree).reshape(-1, 3 if degree < 2 else 6)
    ncoef = Bm.shape[1]
    coefs = np.zeros((B, ncoef))
    oks = np.zeros(B, dtype=bool)
    ns = np.zeros(B, dtype=np.int64)
    for b in range(B):
        m = ((cf[b] >= 2) & (ld[b] > 0) & (z_lr[b] > 0)).reshape(-1)
        ns[b] = int(m.sum())
        if ns[b] < 200:
            continue
        A = Bm[m]
        y = (np.log(np.maximum(ld[b], f32(1e-3))).astype(f32)
             - np.log(np.maximum(z_lr[b], f32(1e-3))).astype(f32)).astype(f32).reshape(-1)[m]
        wgt = np.ones_like(y)
        coef = np.zeros(ncoef)
        for _ in range(iters):
            coef = np.linalg.lstsq((A * wgt[:, None]).astype(np.float64), (y * wgt).astype(np.float64),
                                   rcond=None)[0]
            r = (y - (A.astype(np.float64) @ coef)).astype(f32)
            sc = (f32(1.4826) * lower_median(np.abs(r)) + f32(1e-4)).astype(f32)
            wgt = np.minimum((f32(2) * sc) / np.maximum(np.abs(r), f32(1e-6)), f32(1.0)).astype(f32)
        if not np.all(np.isfinite(coef)):
            continue
        coefs[b] = coef
        oks[b] = True
    return coefs, oks, ns


def prompt_gauge_poly(depth: np.ndarray, lidar: np.ndarray, conf: np.ndarray | None, degree: int = 2,
                      iters: int = 3) -> np.ndarray:
    """[B, H, W] fp32 correction exp(poly(u, v)) per frame (1 where the fit is skipped)."""
    B, H, W = depth.shape
    coefs, oks, _ = gauge_coefficients(depth, lidar, conf, degree, iters)
    VV, UU = np.meshgrid(linspace(H), linspace(W), indexing="ij")
    full = basis(UU, VV, degree).astype(np.float64)
    out = np.ones((B, H, W), dtype=f32)
    for b in range(B):
        if oks[b]:
            out[b] = np.exp(full @ coefs[b]).astype(f32)
    return out
