"""Oracle (test infrastructure): the LiDAR prompt preparation that precedes the refiner, in numpy.

Restates
  * ``promptmoge.nearest_fill`` (promptmoge/model.py:61-72): every missing LiDAR pixel (depth <= 0, or NaN) takes the
    depth of its Euclidean-nearest valid pixel and confidence 1; a frame with no missing or no valid pixel is
    returned unchanged.  The reference finds the nearest pixel with scipy.ndimage.distance_transform_edt
    (return_indices), the separable exact algorithm of Maurer, Qi and Raghavan (2003): pass 1 along axis 0 (the
    nearest valid row of each column), pass 2 along axis 1 (the lower envelope of those candidates along each
    row), each pass moving to a later candidate only when it is strictly closer.  Among equidistant valid pixels
    it therefore returns the one with the smallest column, and within that column the smallest row; this oracle
    states that rule directly (column scan, then an argmin over columns whose first minimum is the smallest column).
  * ``build_prompt`` (moge/model/modules/prompt_stem.py:45-105), the 4-channel form the deployed models take
    (channels: clamp(log d - mu, +-4) on valid pixels, valid, conf / levels on valid pixels, uncertainty
    1 - c (1 - clamp((d - 3) / 2, 0, 1)), 1 where invalid), mu the lower median of log d over the confident pixels
    (conf / levels >= 0.999), else over all valid pixels, else 0 (masked_median, prompt_stem.py:33-40), resized to
    the token grid by torch's 'nearest' rule.

Elementwise arithmetic is fp32 in the reference's operation order.  ``log`` is numpy's; torch's may differ from it by
an ulp, which the tests' tolerance on channel 0 and mu covers.  Parity is pinned by tests/golden/prompt.npz, made
by tests/golden/make_prompt.py from the reference's own functions.
"""
from __future__ import annotations

import numpy as np

from .fit import nearest_resize

f32 = np.float32
LOG_CLAMP = f32(4.0)
RANGE_KNEE_M = f32(3.0)
RANGE_FULL_M = f32(5.0)


def nearest_valid_index(valid: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """(row, col) of the nearest valid pixel of every pixel of a 2-D mask with at least one valid pixel: minimum
    squared distance, ties to the smallest column, then the smallest row (scipy's exact EDT feature transform)."""
    h, w = valid.shape
    rows = np.arange(h)[:, None].repeat(w, 1)
    big = np.int64(1 << 40)
    # pass 1, per column: the last valid row at or above, the first at or below; a tie goes to the one above
    up = np.maximum.accumulate(np.where(valid, rows, -1), axis=0)
    down = np.minimum.accumulate(np.where(valid, rows, h + (1 << 20))[::-1], axis=0)[::-1]
    have_up, have_down = up >= 0, down < h
    use_up = have_up & (~have_down | (rows - up <= down - rows))
    near = np.where(use_up, up, np.where(have_down, down, -1))
    g = np.where(near >= 0, (rows - near).astype(np.int64) ** 2, big)          # [h, w'] squared column distance
    # pass 2, per row: argmin over candidate columns of g + (x - x')^2; argmin returns the first (smallest) column
    cols = np.arange(w)
    dx2 = (cols[:, None] - cols[None, :]).astype(np.int64) ** 2                 # [x, x']
    best = np.empty((h, w), np.int64)
    for i in range(h):
        best[i] = np.argmin(g[i][None, :] + dx2, axis=1)
    src_row = near[np.arange(h)[:, None], best]
    return src_row, best


def nearest_fill(depth: np.ndarray, conf: np.ndarray):
    """promptmoge.nearest_fill for one frame [h, w] (promptmoge/model.py:61-72)."""
    valid = depth > 0
    if valid.all() or not valid.any():
        return depth, conf
    r, c = nearest_valid_index(valid)
    return depth[r, c], np.where(valid, conf, 1).astype(conf.dtype)


def nearest_fill_batch(depth: np.ndarray, conf: np.ndarray):
    """nearest_fill applied to each frame of [B, h, w] (or [B, 1, h, w]) inputs."""
    shape = depth.shape
    d = depth.reshape(-1, *shape[-2:])
    c = conf.reshape(-1, *shape[-2:])
    out = [nearest_fill(d[b], c[b]) for b in range(d.shape[0])]
    return (np.stack([o[0] for o in out]).reshape(shape), np.stack([o[1] for o in out]).reshape(shape))


def lower_median(v: np.ndarray) -> np.float32:
    """torch.median of a 1-D tensor: the lower of the two middle values."""
    s = np.sort(v.astype(f32))
    return s[(s.size - 1) // 2]


def build_prompt(depth: np.ndarray, conf: np.ndarray, out_hw, conf_levels: float = 2.0):
    """build_prompt (prompt_stem.py:45-105) without the optional mono/prefill/phase channels.
    depth, conf [B, 1, h, w] -> prompt [B, 4, H, W] fp32, mu [B] fp32."""
    depth = depth.astype(f32)
    conf = conf.astype(f32)
    with np.errstate(invalid="ignore"):
        valid = np.isfinite(depth) & (depth > 0)
    depth = np.where(valid, depth, f32(1.0)).astype(f32)
    with np.errstate(divide="ignore"):
        logd = np.log(depth).astype(f32)
    c = np.clip((conf / f32(conf_levels)).astype(f32), f32(0), f32(1)).astype(f32)
    hi = valid & (c >= f32(0.999))
    B = depth.shape[0]
    mu = np.zeros(B, f32)
    for b in range(B):
        sel = hi[b] if hi[b].any() else valid[b]
        v = logd[b][sel]
        mu[b] = lower_median(v) if v.size else f32(0.0)
    vf = valid.astype(f32)
    nlog = (np.clip((logd - mu[:, None, None, None]).astype(f32), -LOG_CLAMP, LOG_CLAMP) * vf).astype(f32)
    rng = np.clip(((depth - RANGE_KNEE_M) / f32(RANGE_FULL_M - RANGE_KNEE_M)).astype(f32), f32(0), f32(1))
    unc = (f32(1.0) - (c * (f32(1.0) - rng).astype(f32)).astype(f32)).astype(f32)
    unc = np.where(valid, unc, f32(1.0)).astype(f32)
    prompt = np.concatenate([nlog, vf, (c * vf).astype(f32), unc], axis=1).astype(f32)
    H, W = out_hw
    if prompt.shape[-2:] != (H, W):
        prompt = nearest_resize(prompt, H, W)
    return np.ascontiguousarray(prompt), mu
