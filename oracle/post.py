"""Oracle (test infrastructure): the post-refinement output path of MoGeModel.infer in numpy.

Restates
  * normalized_view_plane_uv (moge/utils/geometry_torch.py:43-55): u, v = torch.linspace(-+span (n - 1) / n, n) in
    fp32, span_x = a / sqrt(1 + a^2), span_y = 1 / sqrt(1 + a^2), a = W / H;
  * recover_focal_shift (geometry_torch.py:118-170 with geometry_numpy.py:82-119): the point map and uv grid
    nearest-downsampled to 64 x 64 (the mask by 'nearest' of its float form, > 0), then per frame the shift that
    minimises sum |f xy / (z + shift) - uv|^2 with the focal f in closed form (f = sum(p . uv) / sum |p|^2,
    p = xy / (z + shift)), or with the given focal; fewer than two samples give focal 1, shift 0.  The reference runs
    scipy's MINPACK Levenberg-Marquardt from shift 0 with ftol 1e-3; on these smooth one-dimensional objectives it
    stops within ~1e-7 of the minimiser, which this oracle (and the GPU kernel) find by damped Gauss-Newton in
    float64 from the same start; the focal then follows in float32 as the reference computes it;
  * the 'exp' output remap (moge/model/v2.py:172-187) and intrinsics_from_focal_center / depth_map_to_point_map of
    utils3d (the utils3d_moge dependency, pinned to commit 62f09d5 in pyproject.toml, is not available here: its
    published convention -- normalised intrinsics, pixel centres at ((j + 0.5) / W, (i + 0.5) / H) -- is restated,
    parity unpinned for that one function).
Parity of the focal / shift recovery and of the uv grid is pinned by tests/golden/post.npz (tests/golden/make_post.py).
"""
from __future__ import annotations

import math

import numpy as np

from .fit import linspace_f32, nearest_index

f32 = np.float32


def view_plane_spans(width: int, height: int, aspect_ratio: float | None = None):
    a = width / height if aspect_ratio is None else aspect_ratio
    return a / (1 + a ** 2) ** 0.5, 1 / (1 + a ** 2) ** 0.5


def normalized_view_plane_uv(width: int, height: int, aspect_ratio: float | None = None) -> np.ndarray:
    sx, sy = view_plane_spans(width, height, aspect_ratio)
    u = linspace_f32(-sx * (width - 1) / width, sx * (width - 1) / width, width)
    v = linspace_f32(-sy * (height - 1) / height, sy * (height - 1) / height, height)
    uu, vv = np.meshgrid(u, v, indexing="xy")
    return np.stack([uu, vv], -1).astype(f32)


def solve_shift(uv: np.ndarray, xyz: np.ndarray, focal: float | None = None, iters: int = 100):
    """Minimiser of sum |f p - uv|^2, p = xy / (z + s), over s from s = 0 (f closed-form when focal is None) by
    damped Gauss-Newton in float64.  Returns (shift fp32, focal fp32 as the reference computes it)."""
    uv = uv.reshape(-1, 2).astype(np.float64)
    xy = xyz[..., :2].reshape(-1, 2).astype(np.float64)
    z = xyz[..., 2].reshape(-1).astype(np.float64)
    U2 = float((uv * uv).sum())

    def terms(s):
        a = 1.0 / (z + s)
        p = xy * a[:, None]
        q = -p * a[:, None]
        S1, S2 = float((p * uv).sum()), float((p * p).sum())
        T1, T2, Q2 = float((q * uv).sum()), float((p * q).sum()), float((q * q).sum())
        if focal is None:
            f = S1 / S2
            df = (T1 * S2 - 2.0 * S1 * T2) / (S2 * S2)
        else:
            f, df = float(focal), 0.0
        cost = f * f * S2 - 2.0 * f * S1 + U2
        rj = f * df * S2 + f * f * T2 - df * S1 - f * T1
        jj = df * df * S2 + 2.0 * df * f * T2 + f * f * Q2
        return cost, rj, jj

    s, lam = 0.0, 0.0
    cost, rj, jj = terms(s)
    for _ in range(iters):
        if not (jj > 0.0):
            break
        step = -rj / (jj + lam)
        if abs(step) <= 1e-12 * max(1.0, abs(s)):
            break
        c2, rj2, jj2 = terms(s + step)
        if np.isfinite(c2) and c2 <= cost:
            s += step
            cost, rj, jj = c2, rj2, jj2
            lam *= 0.25
        else:
            lam = max(lam * 8.0, 1e-6 * jj)
    shift = f32(s)
    if focal is not None:
        return shift, f32(focal)
    xy32 = xyz[..., :2].reshape(-1, 2).astype(f32)
    z32 = xyz[..., 2].reshape(-1).astype(f32)
    xp = (xy32 / (z32 + shift)[:, None]).astype(f32)
    uv32 = uv.astype(f32)
    return shift, f32(f32((xp * uv32).sum(dtype=np.float64)) / f32(np.square(xp).sum(dtype=np.float64)))


def recover_focal_shift(points: np.ndarray, mask: np.ndarray | None = None, focal: np.ndarray | None = None,
                        downsample_size=(64, 64)):
    """points [B,H,W,3] fp32, mask [B,H,W] bool or None, focal [B] or None -> (focal [B] fp32, shift [B] fp32)."""
    B, H, W = points.shape[:3]
    uv = normalized_view_plane_uv(W, H)
    hi, wi = nearest_index(downsample_size[0], H), nearest_index(downsample_size[1], W)
    p_lr = points[:, hi][:, :, wi]
    uv_lr = uv[hi][:, wi]
    m_lr = None if mask is None else mask[:, hi][:, :, wi]
    fo, sh = np.empty(B, f32), np.empty(B, f32)
    for b in range(B):
        p = p_lr[b] if m_lr is None else p_lr[b][m_lr[b]]
        u = uv_lr if m_lr is None else uv_lr[m_lr[b]]
        if p.reshape(-1, 3).shape[0] < 2:
            fo[b], sh[b] = 1.0, 0.0
            continue
        s, f = solve_shift(u, p, None if focal is None else float(focal[b]))
        fo[b], sh[b] = f, s
    return fo, sh


def remap_exp(coords: np.ndarray) -> np.ndarray:
    """'exp' remap: (x, y, z) -> (x e^z, y e^z, e^z) in fp32."""
    ez = np.exp(coords[..., 2:3].astype(f32)).astype(f32)
    return np.concatenate([(coords[..., :2] * ez).astype(f32), ez], -1).astype(f32)


def focal_to_fxfy(focal, width: int, height: int):
    """fx, fy of infer (v3.py:741): focal / 2 * sqrt(1 + a^2) / a, focal / 2 * sqrt(1 + a^2), a = W / H."""
    a = width / height
    return focal / 2 * math.sqrt(1 + a ** 2) / a, focal / 2 * math.sqrt(1 + a ** 2)


def depth_to_points(depth: np.ndarray, fx, fy, cx: float = 0.5, cy: float = 0.5) -> np.ndarray:
    """depth [B,H,W] -> points [B,H,W,3] with normalised intrinsics, pixel centres ((j + 0.5)/W, (i + 0.5)/H)."""
    B, H, W = depth.shape
    u = ((np.arange(W) + 0.5) / W).astype(f32)
    v = ((np.arange(H) + 0.5) / H).astype(f32)
    fx = np.asarray(fx, f32).reshape(B, 1, 1)
    fy = np.asarray(fy, f32).reshape(B, 1, 1)
    x = ((u[None, None, :] - f32(cx)) / fx * depth).astype(f32)
    y = ((v[None, :, None] - f32(cy)) / fy * depth).astype(f32)
    return np.stack([x, y, depth.astype(f32)], -1)
