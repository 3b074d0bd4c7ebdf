"""Golden vectors for the per-frame polynomial prompt gauge, produced by the reference's own
MoGeModel.prompt_gauge_poly (moge/model/v3.py:151-183) on seeded synthetic frames: a ray-cast room's depth with a
smooth multiplicative distortion and noise as the prediction, the scene's LiDAR and confidence as the prompt.

    python tests/golden/make_gauge.py /path/to/PromptMoGe

Writes tests/golden/gauge.npz: per case the inputs (depth [B,H,W], lidar [B,h,w], conf [B,h,w]), degree, and the
reference output corr [B,H,W] (fp32)."""
import sys
import types
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(REPO))
from promptmoge_b200 import synth  # noqa: E402


def import_reference(ref: Path):
    sys.modules.setdefault("utils3d", types.ModuleType("utils3d"))   # only used after refinement (v3.py:758-799)
    sys.path.insert(0, str(ref / "promptmoge" / "_fallback"))
    sys.path.insert(0, str(ref))
    from moge.model.v3 import MoGeModel
    return MoGeModel


def case(seed, B, H, W, degree, holes=0.0, few=False):
    """Inputs of one case: depth [B,H,W], lidar [B,h,w] (the scene's 192x256 LiDAR subsampled to h = 0.4 H, the
    sensor-to-image ratio of the benchmark configs), conf [B,h,w]."""
    sc = synth.make_scene(seed, H, W, 16, 8, batch=B)
    depth = np.exp(sc.point_coord[..., 2]).astype(np.float32)
    rng = np.random.default_rng(seed + 7)
    v, u = np.meshgrid(np.linspace(-1, 1, H), np.linspace(-1, 1, W), indexing="ij")
    for b in range(B):
        c = rng.normal(0, 0.05, 6)
        depth[b] *= np.exp(c[0] + c[1] * u + c[2] * v + c[3] * u * u + c[4] * u * v + c[5] * v * v).astype(np.float32)
    depth *= np.exp(rng.normal(0, 0.01, depth.shape)).astype(np.float32)
    if holes:
        m = rng.random(depth.shape) < holes
        depth[m] = np.where(rng.random(int(m.sum())) < 0.5, np.inf, 0.0)
    h, w = int(round(0.4 * H)), int(round(0.4 * W))
    li = (np.arange(h) * sc.lidar_depth.shape[-2]) // h
    lj = (np.arange(w) * sc.lidar_depth.shape[-1]) // w
    lidar = sc.lidar_depth.reshape(B, *sc.lidar_depth.shape[-2:])[:, li][:, :, lj].astype(np.float32)
    conf = sc.lidar_conf.reshape(B, *sc.lidar_conf.shape[-2:])[:, li][:, :, lj].astype(np.float32)
    if few:                                # fewer than 200 confident pixels in frame 0 -> no correction
        conf[0] = np.where(rng.random(conf[0].shape) < 0.02, conf[0], 0.0)
    return (np.ascontiguousarray(depth, dtype=np.float32), np.ascontiguousarray(lidar), np.ascontiguousarray(conf),
            degree)


# name -> case(seed, B, H, W, degree, holes, few)
CASES = {
    "q2": (21, 2, 120, 160, 2, 0.0, False),
    "q1": (22, 1, 120, 160, 1, 0.0, False),
    "holes": (23, 2, 120, 160, 2, 0.05, False),
    "few": (24, 2, 120, 160, 2, 0.0, True),
    "B240": (25, 1, 240, 320, 2, 0.0, False),
}


def input_sha(*arrays) -> str:
    import hashlib
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def main(ref):
    import torch
    MoGeModel = import_reference(Path(ref))
    out = {}
    for name, args in CASES.items():
        depth, lidar, conf, degree = case(*args)
        with torch.no_grad():
            corr = MoGeModel.prompt_gauge_poly(torch.from_numpy(depth), torch.from_numpy(lidar),
                                               torch.from_numpy(conf), degree=degree).numpy()
        out[f"{name}_inputs_sha"] = np.bytes_(input_sha(depth, lidar, conf))
        out[f"{name}_corr"] = corr.astype(np.float32)
        print(name, depth.shape, lidar.shape, float(corr.min()), float(corr.max()))
    np.savez_compressed(Path(__file__).with_name("gauge.npz"), **out)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {sys.argv[0]} /path/to/PromptMoGe")
    main(sys.argv[1])
