"""The deployed int8 refiner format: ``refiner.bin`` (named blocks back to back) + ``refiner.json`` (geometry and the
block index), as written by the reference's exporter (promptmoge/export/refiner.py:28-111) and read by its Metal
engine (ios/.../Refiner.swift:65-116).

Blocks, in file order (export/refiner.py:87-103), for a refiner of L levels:
  input_proj, prompt_proj, out_proj     ``.w`` weight^T [in][out] fp16, ``.b`` fp16            (unquantised linears)
  down{k} (k < L), pool{k} (k < L-1)    resblock / quantised linear
  encoder_fuse, fuse0, fuse2            quantised linears
  bott                                  resblock
  up{i}, dec{i} (i < L-1)               quantised linear / resblock
  uv_bias                               [C_last, R, C] fp32, the UV half of the encoder conditioning, baked
A quantised linear is ``.w8`` int8 q^T [in][out], ``.ws`` fp32 per-output-channel scale, ``.b`` fp16 bias, ``.clip``
fp32 [1] (the activation clip of its input); a resblock is ``.n1w``/``.n1b`` fp16 LayerNorm affine and, per conv c1 /
c2, ``.{c}w8`` int8 [27][Cin][Cout], ``.{c}ws``, ``.{c}b`` fp16, ``.{c}clip``.  int8 values and scales follow the
training quantiser (q = clamp(round(w / s), +-127), s = max(amax / 127, 1e-12) per output channel).

``write_refiner_dir`` produces the same bytes as the reference exporter for the same weights and clips (checked in
tests/test_refiner_bin.py against the exporter's own output); ``read_refiner_dir`` turns a directory back into the
weights dictionary the engine loads, with the int8 weights and scales taken as stored (not re-quantised) and the
fp16 parameters widened to fp32 exactly.
"""
from __future__ import annotations

import json
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from .engine import quantise_weight

ROWS, COLS = 30, 40          # the token grid the exporter bakes the UV conditioning for (export/coreml.py:24)


def block_layout(levels: int) -> list:
    """(tag, kind, reference module name) in the exporter's order; kind in {"linear", "qlinear", "res"}."""
    out = [("input_proj", "linear", "input_proj"), ("prompt_proj", "linear", "prompt_proj"),
           ("out_proj", "linear", "out_proj")]
    for k in range(levels):
        out.append((f"down{k}", "res", f"down_stages.{k}.0"))
        if k < levels - 1:
            out.append((f"pool{k}", "qlinear", f"downsample_blocks.{k}.linear"))
    out += [("encoder_fuse", "qlinear", "encoder_fuse"), ("fuse0", "qlinear", "fuse_proj.0"),
            ("fuse2", "qlinear", "fuse_proj.2"), ("bott", "res", "bottleneck_stage.0")]
    for i in range(levels - 1):
        out += [(f"up{i}", "qlinear", f"upsample_blocks.{i}.linear"), (f"dec{i}", "res", f"up_stages.{i}.0")]
    return out


class _Writer:
    def __init__(self, path: Path):
        self.f = open(path, "wb")
        self.index = {}
        self.offset = 0

    def put(self, name: str, a, dtype):
        if name in self.index:
            raise ValueError(f"duplicate block {name}")
        x = np.ascontiguousarray(np.asarray(a, dtype=np.float32), dtype=dtype)
        self.f.write(x.tobytes())
        self.index[name] = {"offset": self.offset, "count": int(x.size), "shape": list(x.shape),
                            "dtype": np.dtype(dtype).name}
        self.offset += x.nbytes


def write_refiner_dir(out_dir, weights: dict, clips: dict, channels, uv_bias: np.ndarray,
                      encoder_downsample: int | None = None, depth_resolution: float = 256.0) -> Path:
    """Write refiner.bin / refiner.json for fp32 master weights (reference module names) and activation clips."""
    out = Path(out_dir)
    out.mkdir(parents=True, exist_ok=True)
    L = len(channels)
    down = encoder_downsample if encoder_downsample is not None else 2 ** (L - 1)
    w = _Writer(out / "refiner.bin")
    try:
        for tag, kind, layer in block_layout(L):
            if kind == "linear":
                w.put(f"{tag}.w", np.asarray(weights[layer + ".weight"], np.float32).T, np.float16)
                w.put(f"{tag}.b", weights[layer + ".bias"], np.float16)
            elif kind == "qlinear":
                q, s = quantise_weight(weights[layer + ".weight"])
                w.put(f"{tag}.w8", q.T, np.int8)
                w.put(f"{tag}.ws", s, np.float32)
                w.put(f"{tag}.b", weights[layer + ".bias"], np.float16)
                w.put(f"{tag}.clip", np.array([clips[layer]], np.float32), np.float32)
            else:
                w.put(f"{tag}.n1w", weights[layer + ".norm1.weight"], np.float16)
                w.put(f"{tag}.n1b", weights[layer + ".norm1.bias"], np.float16)
                for c in ("c1", "c2"):
                    conv = f"{layer}.conv{c[1]}"
                    q, s = quantise_weight(weights[conv + ".weight"])           # [Co, 3, 3, 3, Ci]
                    w.put(f"{tag}.{c}w8", q.reshape(q.shape[0], 27, -1).transpose(1, 2, 0), np.int8)
                    w.put(f"{tag}.{c}ws", s, np.float32)
                    w.put(f"{tag}.{c}b", weights[conv + ".bias"], np.float16)
                    w.put(f"{tag}.{c}clip", np.array([clips[conv]], np.float32), np.float32)
        w.put("uv_bias", uv_bias, np.float32)
    finally:
        w.f.close()
    enc = np.asarray(weights["encoder_fuse.weight"])
    meta = {"H": ROWS * down, "W": COLS * down, "R": ROWS, "C": COLS, "levels": L, "channels": [int(c) for c in channels],
            "enc_channels": int(enc.shape[1]), "enc_out": int(enc.shape[0]),
            "depth_resolution": float(depth_resolution), "weights": w.index}
    with open(out / "refiner.json", "w") as f:
        json.dump(meta, f, indent=1)
    return out


@dataclass
class DeployedRefiner:
    """A refiner.bin directory in the engine's terms."""
    height: int
    width: int
    channels: list
    enc_channels: int
    depth_resolution: float
    weights: dict        # reference module name -> array: ".weight_q8"/".weight_scale" for quantised layers
    clips: dict          # quantised layer -> activation clip of its input
    uv_bias: np.ndarray  # [C_last, R, C] fp32


def read_refiner_dir(path) -> DeployedRefiner:
    """Read refiner.json / refiner.bin.  Raises ValueError on a missing block or a block that runs past the file."""
    d = Path(path)
    meta = json.loads((d / "refiner.json").read_text())
    blob = np.fromfile(d / "refiner.bin", dtype=np.uint8)
    index = meta["weights"]

    def get(name):
        if name not in index:
            raise ValueError(f"refiner.bin: missing block {name}")
        e = index[name]
        dt = np.dtype(e["dtype"])
        end = e["offset"] + e["count"] * dt.itemsize
        if e["offset"] < 0 or end > blob.size:
            raise ValueError(f"refiner.bin: block {name} runs past the end of the file")
        a = blob[e["offset"]:end].view(dt).reshape(e["shape"])
        return a

    L = int(meta["levels"])
    W, clips = {}, {}
    for tag, kind, layer in block_layout(L):
        if kind == "linear":
            W[layer + ".weight"] = np.ascontiguousarray(get(f"{tag}.w").astype(np.float32).T)
            W[layer + ".bias"] = get(f"{tag}.b").astype(np.float32)
        elif kind == "qlinear":
            W[layer + ".weight_q8"] = np.ascontiguousarray(get(f"{tag}.w8").T)
            W[layer + ".weight_scale"] = get(f"{tag}.ws").astype(np.float32).copy()
            W[layer + ".bias"] = get(f"{tag}.b").astype(np.float32)
            clips[layer] = float(get(f"{tag}.clip")[0])
        else:
            W[layer + ".norm1.weight"] = get(f"{tag}.n1w").astype(np.float32)
            W[layer + ".norm1.bias"] = get(f"{tag}.n1b").astype(np.float32)
            for c in ("c1", "c2"):
                conv = f"{layer}.conv{c[1]}"
                q = get(f"{tag}.{c}w8")                                       # [27, Ci, Co]
                W[conv + ".weight_q8"] = np.ascontiguousarray(q.transpose(2, 0, 1)).reshape(
                    q.shape[2], 3, 3, 3, q.shape[1])
                W[conv + ".weight_scale"] = get(f"{tag}.{c}ws").astype(np.float32).copy()
                W[conv + ".bias"] = get(f"{tag}.{c}b").astype(np.float32)
                clips[conv] = float(get(f"{tag}.{c}clip")[0])
    return DeployedRefiner(height=int(meta["H"]), width=int(meta["W"]), channels=[int(c) for c in meta["channels"]],
                           enc_channels=int(meta["enc_channels"]), depth_resolution=float(meta["depth_resolution"]),
                           weights=W, clips=clips, uv_bias=get("uv_bias").astype(np.float32).copy())
