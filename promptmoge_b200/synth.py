"""Seeded synthetic inputs for the sparse 3-D refinement step.

There are no ARKitScenes frames and no trained checkpoints on this machine, so every workload is generated from a
seed with plain numpy arithmetic (an analytic ray cast, not a renderer):

* ``make_scene`` -- a 4 x 5 x 3 m room with 6-12 axis-aligned boxes and 2 spheres, a camera at a random interior
  pose, pinhole fx = fy = 0.8 W.  It returns the refiner's point map ``(x/z, y/z, log z)`` with 1 %-of-depth
  Gaussian noise, the 192 x 256 LiDAR prompt (2 % noise, 5 % holes set to 0, confidence {0,1,2} drawn with
  probabilities 0.1 / 0.2 / 0.7), the fp16 N(0,1) token feature ``[B, 1024, H/d, W/d]`` and the UV bias map.
* ``make_refiner_weights`` -- random-init weights of the refiner's layer list (``Sparse3DUNet`` of
  moge/model/modules/sparse_unet.py:33-120 with the widths of promptmoge/compress/make_refiner.py:21 (Model A) and
  make_model_b.py:45,59-60 (Model B)), keyed by the reference's own state-dict names so the same tensors load into
  the reference module for parity fixtures.
* ``make_surface_voxels`` -- the isolated-conv workload: voxels on 2-D surface shells in a 2^21-per-axis grid.

Nothing here touches a GPU.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

# Refiner geometry per model (sparse_unet.py:33-120; v3.py:126-143 with refiner_uv_fold -> 1024 encoder channels).
MODELS = {
    "A": dict(model_channels=[32, 64, 128, 256, 256], downsample_factors=[2, 2, 2, 2], encoder_downsample=16,
              H=480, W=640),
    "B": dict(model_channels=[32, 64, 128, 256], downsample_factors=[2, 2, 2], encoder_downsample=8,
              H=240, W=320),
}
ENC_CHANNELS = 1024
IN_CHANNELS = 3
PROMPT_CHANNELS = 2
OUT_CHANNELS = 1
LIDAR_HW = (192, 256)
DEPTH_RESOLUTION = 256.0


@dataclass
class Scene:
    point_coord: np.ndarray      # [B, H, W, 3] fp32  (x/z, y/z, log z)
    lidar_depth: np.ndarray      # [B, 1, 192, 256] fp32 metres, 0 = hole
    lidar_conf: np.ndarray       # [B, 1, 192, 256] fp32 in {0, 1, 2}
    encoder_feature: np.ndarray  # [B, 1024, H/d, W/d] fp16
    uv_bias: np.ndarray          # [B, C_last, H/d, W/d] fp32
    meta: dict = field(default_factory=dict)


def _rotation(yaw: float, pitch: float, roll: float) -> np.ndarray:
    """Camera-to-world rotation. Camera axes: x right, y down, z forward. World: z up."""
    # Base: camera looking along world +x, with camera y (down) = world -z and camera x (right) = world -y.
    base = np.array([[0.0, 0.0, 1.0], [-1.0, 0.0, 0.0], [0.0, -1.0, 0.0]])
    cy, sy = math.cos(yaw), math.sin(yaw)
    cp, sp = math.cos(pitch), math.sin(pitch)
    cr, sr = math.cos(roll), math.sin(roll)
    rz = np.array([[cy, -sy, 0], [sy, cy, 0], [0, 0, 1.0]])
    ry = np.array([[cp, 0, sp], [0, 1.0, 0], [-sp, 0, cp]])
    rx = np.array([[1.0, 0, 0], [0, cr, -sr], [0, sr, cr]])
    return rz @ ry @ rx @ base


def _raycast(origin: np.ndarray, dirs: np.ndarray, boxes: list, spheres: list, room: np.ndarray) -> np.ndarray:
    """Nearest positive hit parameter t along each direction (dirs: [N, 3] world, not normalised)."""
    inv = 1.0 / np.where(np.abs(dirs) < 1e-12, 1e-12, dirs)
    # Inside the room: the exit distance of the room box.
    t1 = (room[0] - origin) * inv
    t2 = (room[1] - origin) * inv
    t_exit = np.maximum(t1, t2).min(axis=1)
    t = t_exit.copy()
    for lo, hi in boxes:
        a = (lo - origin) * inv
        b = (hi - origin) * inv
        tn = np.minimum(a, b).max(axis=1)
        tf = np.maximum(a, b).min(axis=1)
        hit = (tn <= tf) & (tn > 1e-3)
        t = np.where(hit & (tn < t), tn, t)
    for c, r in spheres:
        oc = origin - c
        qa = np.einsum("ij,ij->i", dirs, dirs)
        qb = 2.0 * (dirs @ oc)
        qc = float(oc @ oc) - r * r
        disc = qb * qb - 4 * qa * qc
        ok = disc > 0
        sq = np.sqrt(np.where(ok, disc, 0.0))
        tn = (-qb - sq) / (2 * qa)
        hit = ok & (tn > 1e-3)
        t = np.where(hit & (tn < t), tn, t)
    return t


def _render_depth(rng_layout, H: int, W: int, origin, R, boxes, spheres, room):
    fx = fy = 0.8 * W
    cx, cy = W / 2.0, H / 2.0
    v, u = np.meshgrid(np.arange(H, dtype=np.float64) + 0.5, np.arange(W, dtype=np.float64) + 0.5, indexing="ij")
    xn = (u - cx) / fx
    yn = (v - cy) / fy
    d_cam = np.stack([xn, yn, np.ones_like(xn)], axis=-1).reshape(-1, 3)
    d_world = d_cam @ R.T
    t = _raycast(origin, d_world, boxes, spheres, room)
    # d_cam has unit z, so the hit parameter IS the depth along the optical axis.
    return t.reshape(H, W), xn, yn


def make_scene(seed: int, H: int = 480, W: int = 640, encoder_downsample: int = 16, c_last: int = 256,
               batch: int = 1) -> Scene:
    """Seeded synthetic frames (one independent room per batch entry, seeds seed, seed+1, ...)."""
    pcs, lds, lcs, encs, uvbs = [], [], [], [], []
    for b in range(batch):
        rng = np.random.default_rng(seed + b)
        room = np.array([[0.0, 0.0, 0.0], [4.0, 5.0, 3.0]])
        origin = np.array([rng.uniform(1.0, 3.0), rng.uniform(1.0, 4.0), rng.uniform(1.0, 2.0)])
        R = _rotation(rng.uniform(-math.pi, math.pi), rng.uniform(-0.35, 0.35), rng.uniform(-0.1, 0.1))
        clear = 0.6                                  # free space kept around the camera
        boxes = []
        n_boxes = int(rng.integers(6, 13))
        while len(boxes) < n_boxes:
            size = rng.uniform([0.3, 0.3, 0.3], [1.4, 1.4, 1.6])
            lo = rng.uniform(room[0], room[1] - size)
            if rng.random() < 0.6:
                lo[2] = 0.0                          # furniture stands on the floor
            if np.all(origin > lo - clear) and np.all(origin < lo + size + clear):
                continue
            boxes.append((lo, lo + size))
        spheres = []
        while len(spheres) < 2:
            r = float(rng.uniform(0.2, 0.6))
            c = rng.uniform(room[0] + r, room[1] - r)
            if np.linalg.norm(c - origin) < r + clear:
                continue
            spheres.append((c, r))

        depth, xn, yn = _render_depth(rng, H, W, origin, R, boxes, spheres, room)
        z = depth * (1.0 + 0.01 * rng.standard_normal(depth.shape))
        z = np.maximum(z, 1e-3)
        pc = np.stack([xn, yn, np.log(z)], axis=-1).astype(np.float32)

        lh, lw = LIDAR_HW
        ldep, _, _ = _render_depth(rng, lh, lw, origin, R, boxes, spheres, room)
        ldep = ldep * (1.0 + 0.02 * rng.standard_normal(ldep.shape))
        holes = rng.random(ldep.shape) < 0.05
        ldep = np.where(holes, 0.0, ldep).astype(np.float32)
        conf = rng.choice(np.array([0.0, 1.0, 2.0], dtype=np.float32), size=ldep.shape, p=[0.1, 0.2, 0.7])

        th, tw = H // encoder_downsample, W // encoder_downsample
        enc = rng.standard_normal((ENC_CHANNELS, th, tw)).astype(np.float16)
        # UV half of the encoder conditioning (v3.py:541-545): a fixed 1x1 projection of the view-plane UV grid.
        u = np.linspace(-1.0, 1.0, tw, dtype=np.float64)
        v = np.linspace(-0.75, 0.75, th, dtype=np.float64)
        vv, uu = np.meshgrid(v, u, indexing="ij")
        w_uv = rng.normal(0.0, 0.5, (c_last, 2))
        uvb = (w_uv[:, 0, None, None] * uu[None] + w_uv[:, 1, None, None] * vv[None]).astype(np.float32)

        pcs.append(pc); lds.append(ldep[None]); lcs.append(conf[None]); encs.append(enc); uvbs.append(uvb)
    return Scene(
        point_coord=np.stack(pcs), lidar_depth=np.stack(lds).astype(np.float32),
        lidar_conf=np.stack(lcs).astype(np.float32), encoder_feature=np.stack(encs), uv_bias=np.stack(uvbs),
        meta=dict(seed=seed, H=H, W=W, batch=batch, encoder_downsample=encoder_downsample),
    )


def scene_for_model(model: str, seed: int, batch: int = 1, scale: int = 1) -> Scene:
    """The scene a model's refiner consumes; ``scale`` > 1 shrinks H, W (and the token grid) for small tests."""
    m = MODELS[model]
    return make_scene(seed, m["H"] // scale, m["W"] // scale, m["encoder_downsample"], m["model_channels"][-1],
                      batch=batch)


def refiner_layer_shapes(model: str) -> dict:
    """State-dict names and shapes of a narrowed QAT refiner (sparse_unet.py:77-120, flex_sparse_blocks.py:50-105)."""
    ch = MODELS[model]["model_channels"]
    L = len(ch)
    shapes = {
        "input_proj.weight": (ch[0], IN_CHANNELS), "input_proj.bias": (ch[0],),
        "prompt_proj.weight": (ch[0], PROMPT_CHANNELS), "prompt_proj.bias": (ch[0],),
        "encoder_fuse.weight": (ch[-1], ENC_CHANNELS), "encoder_fuse.bias": (ch[-1],),
        "fuse_proj.0.weight": (ch[-1], 2 * ch[-1]), "fuse_proj.0.bias": (ch[-1],),
        "fuse_proj.2.weight": (ch[-1], ch[-1]), "fuse_proj.2.bias": (ch[-1],),
        "out_proj.weight": (OUT_CHANNELS, ch[0]), "out_proj.bias": (OUT_CHANNELS,),
    }

    def block(prefix, c):
        shapes[f"{prefix}.norm1.weight"] = (c,)
        shapes[f"{prefix}.norm1.bias"] = (c,)
        for cv in ("conv1", "conv2"):
            shapes[f"{prefix}.{cv}.weight"] = (c, 3, 3, 3, c)
            shapes[f"{prefix}.{cv}.bias"] = (c,)

    for k in range(L):
        block(f"down_stages.{k}.0", ch[k])
        if k < L - 1:
            shapes[f"downsample_blocks.{k}.linear.weight"] = (ch[k + 1], ch[k])
            shapes[f"downsample_blocks.{k}.linear.bias"] = (ch[k + 1],)
    block("bottleneck_stage.0", ch[-1])
    for i in range(L - 1):
        src, dst = L - 1 - i, L - 2 - i
        shapes[f"upsample_blocks.{i}.linear.weight"] = (ch[dst], ch[src])
        shapes[f"upsample_blocks.{i}.linear.bias"] = (ch[dst],)
        block(f"up_stages.{i}.0", ch[dst])
    return shapes


def make_refiner_weights(model: str, seed: int = 0) -> dict:
    """Random-init refiner weights (uniform +-1/sqrt(fan_in), the scale of nn.Linear / SubmanifoldConv3d's default
    init).  The prompt projection, zero-initialised in the reference (sparse_unet.py:78-80), gets a random init here
    so the LiDAR residual path is exercised; the output projection is kept small so one step is a small update."""
    rng = np.random.default_rng(1_000_003 + seed)
    out = {}
    for name, shp in refiner_layer_shapes(model).items():
        if name.endswith("norm1.weight"):
            out[name] = (1.0 + 0.1 * rng.uniform(-1, 1, shp)).astype(np.float32)
            continue
        if name.endswith("norm1.bias"):
            out[name] = (0.1 * rng.uniform(-1, 1, shp)).astype(np.float32)
            continue
        wname = name[:-len(".bias")] + ".weight" if name.endswith(".bias") else name
        wshape = refiner_layer_shapes(model)[wname]
        fan_in = int(np.prod(wshape[1:]))
        bound = 1.0 / math.sqrt(fan_in)
        if name.startswith("out_proj"):
            bound *= 0.05
        out[name] = rng.uniform(-bound, bound, shp).astype(np.float32)
    return out


def make_surface_voxels(n: int, seed: int = 0, axis_bits: int = 21) -> np.ndarray:
    """~n unique voxels (b=0, x, y, z) on 2-D surface shells in a 2^axis_bits-per-axis grid, lexicographically
    sorted, as int32 [M, 4].  Each shell is a wavy height field z = h(x, y) over a square patch, rasterised one voxel
    per (x, y) and thickened where the surface is steep so that neighbourhoods stay connected (about 9 occupied taps
    per voxel on average)."""
    rng = np.random.default_rng(seed)
    extent = 1 << axis_bits
    chunks = []
    total = 0
    while total < n:
        side = int(min(max(64, math.isqrt(max(n - total, 1))), 2048))
        x0, y0, z0 = (int(v) for v in rng.integers(0, extent - 4 * side, 3))
        ax, ay = rng.uniform(0.05, 0.25, 2)
        fx, fy = rng.uniform(0.01, 0.05, 2)
        ph = rng.uniform(0, 2 * math.pi, 2)
        yy, xx = np.meshgrid(np.arange(side), np.arange(side), indexing="ij")
        h = side * (ax * np.sin(fx * xx + ph[0]) + ay * np.cos(fy * yy + ph[1])) + 0.35 * (xx + yy)
        zi = np.floor(h).astype(np.int64)
        pts = [np.stack([xx.ravel(), yy.ravel(), zi.ravel()], 1)]
        # Fill vertical gaps to the lower neighbour so the shell is 26-connected.
        zmin_nb = np.minimum(np.roll(zi, 1, 0), np.roll(zi, 1, 1))
        gap = zi - zmin_nb
        for d in range(1, 3):
            m = (gap > d).ravel()
            pts.append(np.stack([xx.ravel()[m], yy.ravel()[m], zi.ravel()[m] - d], 1))
        p = np.concatenate(pts)
        p[:, 0] += x0; p[:, 1] += y0; p[:, 2] += z0
        chunks.append(p)
        total += p.shape[0]
    p = np.concatenate(chunks)
    p = np.unique(p, axis=0)
    if p.shape[0] > n:
        p = p[np.sort(rng.choice(p.shape[0], n, replace=False))]
    coords = np.zeros((p.shape[0], 4), np.int32)
    coords[:, 1:] = p
    return coords


def seeded_conv_input(layer: str, rows: int, channels: int) -> np.ndarray:
    """Seeded int8 input [rows, channels], uniform in [-127, 127], for pinning one conv layer's int32 accumulators
    at full size: the fixture generator feeds it to the reference's own submanifold_conv on the reference-built
    neighbour cache, the GPU tests feed the same array to the library's conv kernels.  The seed is derived from the
    layer's reference module name, so every layer gets its own input."""
    seed = int.from_bytes(layer.encode(), "little") % (2 ** 61 - 1)
    rng = np.random.default_rng(seed)
    return rng.integers(-127, 128, size=(rows, channels)).astype(np.int8)
