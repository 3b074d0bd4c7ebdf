"""Golden vectors for the optional refiner-side gates of the refine loop (moge/model/v3.py:565-573), produced with
the reference's own MoGeModel._lidar_uncertainty (v3.py:385-393) and _lidar_in_affine_frame (v3.py:362-383, which
runs prompt_stem.fit_scale_shift) on seeded synthetic frames:

    output gate      g = floor + (1 - floor) * u;  logz = cur + g * (refined - cur)
    elastic anchor   log_d_aff, gate = _lidar_in_affine_frame(logz);  logz = logz + beta * gate * (log_d_aff - logz)

    python tests/golden/make_gates.py /path/to/PromptMoGe

Writes tests/golden/gates.npz: per case the inputs (cur, refined [B,H,W], lidar / conf [B,1,192,256]), floor,
beta, and the reference's gated logz."""
import sys
import types
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(REPO))
from promptmoge_b200 import synth  # noqa: E402

# name -> (seed, B, H, W, floor or None, beta)
CASES = {"gate": (41, 2, 48, 64, 0.1, 0.0), "anchor": (42, 2, 48, 64, None, 0.3),
         "both": (43, 1, 120, 160, 0.25, 0.5)}


def case(name):
    seed, B, H, W, floor, beta = CASES[name]
    sc = synth.make_scene(seed, H, W, 8, 256, batch=B)
    cur = sc.point_coord[..., 2].astype(np.float32)
    rng = np.random.default_rng(seed)
    refined = (cur + rng.normal(0, 0.05, cur.shape)).astype(np.float32)
    return cur, refined, sc.lidar_depth.astype(np.float32), sc.lidar_conf.astype(np.float32), floor, beta


def main(ref: Path):
    sys.modules.setdefault("utils3d", types.ModuleType("utils3d"))
    sys.path.insert(0, str(ref / "promptmoge" / "_fallback"))
    sys.path.insert(0, str(ref))
    import torch
    from moge.model.v3 import MoGeModel

    out = {}
    for name in CASES:
        cur, refined, ld, lc, floor, beta = case(name)
        c, r = torch.from_numpy(cur), torch.from_numpy(refined)
        tl, tc = torch.from_numpy(ld), torch.from_numpy(lc)
        if floor is not None:
            u = MoGeModel._lidar_uncertainty(r.shape[-2:], tl, tc)
            g = floor + (1.0 - floor) * u
            r = c + g * (r - c)
        if beta > 0:
            log_d_aff, gate, _, _ = MoGeModel._lidar_in_affine_frame(r, tl, tc)
            r = r + beta * gate * (log_d_aff - r)
        out[f"{name}_out"] = r.numpy().astype(np.float32)
    dst = Path(__file__).resolve().parent / "gates.npz"
    np.savez_compressed(dst, **out)
    print("wrote", dst)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {sys.argv[0]} /path/to/PromptMoGe")
    main(Path(sys.argv[1]))
