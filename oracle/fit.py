"""Oracle (test infrastructure): the closed-form robust metric fit and the LiDAR prompt features in numpy.

Restates moge/model/modules/prompt_stem.py:211-240 (fit_scale_shift), moge/model/v3.py:362-383
(_lidar_in_affine_frame with the soft residual gate), the final 'lidar_ls' fit of v3.py:768-778, and the two
resamplers they use (torch F.interpolate 'nearest' and 'area' on CPU).  Elementwise arithmetic is fp32 in the same
operation order as the reference (no fused multiply-add); the five fit sums are accumulated in float64 and rounded
to fp32 (the reference sums in fp32 with cascaded accumulation; the two agree to ~1e-7 relative).
"""
from __future__ import annotations

import numpy as np

f32 = np.float32


def linspace_f32(start: float, end: float, n: int) -> np.ndarray:
    """torch.linspace(start, end, n, dtype=float32): step = (end - start) / (n - 1) in fp32, then start + step * i
    below the midpoint and end - step * (n - 1 - i) above it, each a fused multiply-add (one rounding; the product
    and sum are formed exactly in float64 and rounded once)."""
    s, e = f32(start), f32(end)
    if n == 1:
        return np.array([s], f32)
    step = f32(e - s) / f32(n - 1)
    i = np.arange(n, dtype=np.float64)
    lo = (np.float64(s) + np.float64(step) * i).astype(f32)
    hi = (np.float64(e) - np.float64(step) * (n - 1 - i)).astype(f32)
    return np.where(np.arange(n) < n // 2, lo, hi).astype(f32)


def nearest_index(out_size: int, in_size: int) -> np.ndarray:
    """Source index of torch's 'nearest' resize on CPU: min(floor(dst * (float)in/out), in-1) in fp32; identity when
    sizes match, dst >> 1 when out == 2 in (aten UpSample.h nearest_idx)."""
    dst = np.arange(out_size)
    if out_size == in_size:
        return dst
    if out_size == 2 * in_size:
        return dst >> 1
    scale = f32(in_size) / f32(out_size)
    return np.minimum(np.floor(dst.astype(f32) * scale).astype(np.int64), in_size - 1)


def nearest_resize(x: np.ndarray, H: int, W: int) -> np.ndarray:
    """F.interpolate(x, (H, W), mode='nearest') for x [..., h, w]."""
    h, w = x.shape[-2:]
    return x[..., nearest_index(H, h)[:, None], nearest_index(W, w)[None, :]]


def area_resize(x: np.ndarray, h: int, w: int) -> np.ndarray:
    """F.interpolate(x, (h, w), mode='area') = adaptive_avg_pool2d on CPU: window [floor(o*in/out),
    ceil((o+1)*in/out)), summed in fp32 row by row in input order, then divided by the window height and then by
    the window width (two roundings, as aten's cpu_adaptive_avg_pool does)."""
    H, W = x.shape[-2:]
    out = np.empty(x.shape[:-2] + (h, w), dtype=f32)
    xs = x.astype(f32)
    for oh in range(h):
        h0 = (oh * H) // h
        h1 = -(-((oh + 1) * H) // h)
        for ow in range(w):
            w0 = (ow * W) // w
            w1 = -(-((ow + 1) * W) // w)
            acc = np.zeros(x.shape[:-2], dtype=f32)
            for ih in range(h0, h1):
                for iw in range(w0, w1):
                    acc = (acc + xs[..., ih, iw]).astype(f32)
            out[..., oh, ow] = ((acc / f32(h1 - h0)).astype(f32) / f32(w1 - w0)).astype(f32)
    return out


def _sum(x: np.ndarray) -> np.ndarray:
    return x.astype(np.float64).sum(axis=1).astype(f32)


def trim_count(count: np.ndarray, trim: float = 0.2, min_points: int = 32) -> np.ndarray:
    """k = ((1 - trim) * mask.sum(1)).long().clamp_min(min_points): a Python float times an int64 tensor promotes to
    fp32, so the product is fp32(0.8) * fp32(count) rounded to fp32, then truncated (prompt_stem.py:237)."""
    k = (f32(1.0 - trim) * count.astype(f32)).astype(f32).astype(np.int64)
    return np.maximum(k, min_points)


def fit_scale_shift(z, target, mask, iters: int = 4, trim: float = 0.2, min_points: int = 32, trace=None):
    """Batched trimmed least squares target ~= s * z + t on mask (prompt_stem.py:211-240).  z, target [B, N] fp32,
    mask [B, N] bool -> s, t [B] fp32.  (1, 0) when fewer than min_points are masked.  `trace`, if a list, receives
    per iteration the solved (s, t) and the trim threshold."""
    z = np.asarray(z, f32)
    target = np.asarray(target, f32)
    mask = np.asarray(mask, bool)
    B, N = z.shape
    w = mask.astype(f32)
    s = np.ones(B, f32)
    t = np.zeros(B, f32)
    ok = w.sum(1) >= min_points
    for it in range(iters + 1):
        n = np.maximum(_sum(w), f32(1))
        sx = _sum(w * z)
        sy = _sum(w * target)
        sxx = _sum((w * z) * z)
        sxy = _sum((w * z) * target)
        den = (n * sxx - sx * sx).astype(f32)
        s_new = np.where(den > f32(1e-12), ((n * sxy - sx * sy) / np.maximum(den, f32(1e-12))).astype(f32), f32(1))
        t_new = ((sy - s_new * sx) / n).astype(f32)
        s = np.where(ok, s_new, s).astype(f32)
        t = np.where(ok, t_new, t).astype(f32)
        if it == iters:
            if trace is not None:
                trace.append((s.copy(), t.copy(), None))
            break
        r = (np.abs((s[:, None] * z + t[:, None]) - target) / np.maximum(target, f32(1e-3))).astype(f32)
        r = np.where(mask, r, f32(np.inf))
        k = trim_count(mask.sum(1), trim, min_points)
        thr = np.array([np.partition(r[b], min(int(k[b]), N) - 1)[min(int(k[b]), N) - 1] for b in range(B)], f32)
        if trace is not None:
            trace.append((s.copy(), t.copy(), thr.copy()))
        w = (mask & (r <= thr[:, None])).astype(f32)
    return s, t


def lidar_in_affine_frame(logz, lidar_depth, lidar_conf, soft_gate: bool = True):
    """MoGeModel._lidar_in_affine_frame, v3.py:362-383.  logz [B, H, W]; lidar_depth, lidar_conf [B, 1, h, w].
    Returns (log_d_aff, gate, s, t)."""
    logz = np.asarray(logz, f32)
    B, H, W = logz.shape
    d = nearest_resize(np.asarray(lidar_depth, f32), H, W)[:, 0]
    c = np.clip(nearest_resize(np.asarray(lidar_conf, f32), H, W)[:, 0] / f32(2.0), f32(0), f32(1))
    valid = np.isfinite(d) & (d > 0)
    z = np.exp(logz).astype(f32)
    s, t = fit_scale_shift(z.reshape(B, -1), d.reshape(B, -1), (valid & (c >= f32(0.999))).reshape(B, -1))
    d_aff = ((d - t.reshape(-1, 1, 1)) / np.maximum(s.reshape(-1, 1, 1), f32(1e-6))).astype(f32)
    ok = valid & (d_aff > f32(1e-4))
    log_d_aff = np.where(ok, np.log(np.maximum(d_aff, f32(1e-4))).astype(f32), logz)
    if soft_gate:
        gate = ((f32(0.15) + f32(0.85) * c) * ok.astype(f32)).astype(f32)
    else:
        gate = (c * ok.astype(f32)).astype(f32)
    return log_d_aff, gate, s, t


def prompt_feats(logz, lidar_depth, lidar_conf):
    """The refiner's prompt channels (v3.py:552-555): residual = (log_d_aff - logz) * gate, gate.  [B*H*W, 2]."""
    log_d_aff, gate, s, t = lidar_in_affine_frame(logz, lidar_depth, lidar_conf, soft_gate=True)
    residual = ((log_d_aff - np.asarray(logz, f32)) * gate).astype(f32)
    return np.stack([residual, gate], axis=-1).reshape(-1, 2), s, t


def final_fit(depth, lidar_depth, lidar_conf, mask_area=None):
    """The final metric fit of infer(metric_from='lidar_ls'), v3.py:768-777: area-downsample depth to the LiDAR grid,
    mask = conf >= 2 & lidar > 0 & d_lr > 0 (& model-mask area > 0.99 when given), fit, depth = s * depth + t.
    depth [B, H, W] fp32.  Returns (metric depth, s, t)."""
    depth = np.asarray(depth, f32)
    ld = np.asarray(lidar_depth, f32)[:, 0]
    lc = np.asarray(lidar_conf, f32)[:, 0]
    h, w = ld.shape[-2:]
    d_lr = area_resize(depth, h, w)
    m = (lc >= 2) & (ld > 0) & (d_lr > 0)
    if mask_area is not None:
        m &= area_resize(np.asarray(mask_area, f32), h, w) > f32(0.99)
    B = depth.shape[0]
    s, t = fit_scale_shift(d_lr.reshape(B, -1), ld.reshape(B, -1), m.reshape(B, -1))
    return (s[:, None, None] * depth + t[:, None, None]).astype(f32), s, t
