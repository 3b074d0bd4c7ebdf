"""Golden vectors for the post-refinement focal / shift recovery, produced by the reference's own
moge.utils.geometry_torch.recover_focal_shift (moge/utils/geometry_torch.py:118-170: nearest downsample to 64 x 64,
scipy least_squares 'lm' per frame, geometry_numpy.py:82-119) and normalized_view_plane_uv (geometry_torch.py:43-55).

    python tests/golden/make_post.py /path/to/PromptMoGe

Writes tests/golden/post.npz: per case the affine point map [B,H,W,3], the optional mask [B,H,W] and fixed focal
[B], and the reference's focal [B] and shift [B]; and the view-plane uv grids of a few sizes."""
import sys
import types
from pathlib import Path

import numpy as np

f32 = np.float32


def affine_points(seed: int, B: int, H: int, W: int, shifts, focal_scale: float = 0.9, noise: float = 0.002):
    """An affine point map (x, y, z - shift with x, y scaled by an unknown focal factor) of seeded smooth surfaces
    seen by a pinhole camera: what the network's 'exp' remap produces before the shift is known."""
    rng = np.random.default_rng(seed)
    aspect = W / H
    span_x = aspect / (1 + aspect ** 2) ** 0.5
    span_y = 1 / (1 + aspect ** 2) ** 0.5
    u = np.linspace(-span_x * (W - 1) / W, span_x * (W - 1) / W, W)
    v = np.linspace(-span_y * (H - 1) / H, span_y * (H - 1) / H, H)
    uu, vv = np.meshgrid(u, v, indexing="xy")
    out = np.empty((B, H, W, 3), f32)
    for b in range(B):
        z = 1.5 + 0.8 * uu + 0.5 * np.sin(3 * vv + rng.uniform(0, 3)) + rng.uniform(0, 1.5)
        z = z * np.exp(rng.normal(0, noise, z.shape))
        f_true = rng.uniform(0.9, 1.6)
        x = uu * z / f_true * focal_scale
        y = vv * z / f_true * focal_scale
        out[b] = np.stack([x, y, z - shifts[b]], -1)
    return out


# name -> (seed, B, H, W, shifts, mask kind, fixed focal)
CASES = {
    "plain": (1, 3, 96, 128, [0.0, 0.3, -0.2], None, None),
    "masked": (2, 2, 120, 160, [0.5, -0.1], "half", None),
    "focal_given": (3, 2, 60, 80, [0.2, 0.0], None, [1.3, 0.8]),
    "few_points": (4, 2, 48, 64, [0.1, 0.1], "one", None),       # frame 0 keeps a single sample: focal 1, shift 0
    "odd_size": (5, 1, 37, 53, [0.4], "rand", None),              # smaller than 64 on both axes (nearest upsample)
}


def case(name):
    seed, B, H, W, shifts, mk, focal = CASES[name]
    pts = affine_points(seed, B, H, W, shifts)
    mask = None
    if mk is not None:
        rng = np.random.default_rng(seed + 100)
        if mk == "half":
            mask = np.zeros((B, H, W), bool)
            mask[:, :, : W // 2 + 7] = True
        elif mk == "one":
            mask = np.ones((B, H, W), bool)
            mask[0] = False
            mask[0, 1, 5] = True          # row 1 of 48 is sampled once by the 64-row nearest grid
        else:
            mask = rng.random((B, H, W)) < 0.7
    return pts, mask, (np.array(focal, f32) if focal is not None else None)


UV_SIZES = [(160, 120), (53, 37), (1, 1), (64, 64), (300, 7)]


def main(ref: Path):
    sys.modules.setdefault("utils3d", types.ModuleType("utils3d"))
    sys.path.insert(0, str(ref))
    import torch
    from moge.utils.geometry_torch import normalized_view_plane_uv, recover_focal_shift

    out = {}
    for name in CASES:
        pts, mask, focal = case(name)
        f, s = recover_focal_shift(torch.from_numpy(pts), None if mask is None else torch.from_numpy(mask),
                                   focal=None if focal is None else torch.from_numpy(focal))
        out[f"{name}_focal"] = f.numpy().astype(f32)
        out[f"{name}_shift"] = s.numpy().astype(f32)
    for w, h in UV_SIZES:
        out[f"uv_{w}x{h}"] = normalized_view_plane_uv(w, h, dtype=torch.float32).numpy()
    dst = Path(__file__).resolve().parent / "post.npz"
    np.savez_compressed(dst, **out)
    print("wrote", dst)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {sys.argv[0]} /path/to/PromptMoGe")
    main(Path(sys.argv[1]))
