"""User-facing refinement API: host (numpy / CPU tensor) frames in, refined point maps out.

``Refiner`` wraps one RefinerEngine plan (a model geometry and a frame batch), keeps pinned staging buffers, and runs
``refine(...)`` as: host->device copies of the frame's inputs, the per-frame encoder conditioning, the K-step CUDA
graph, device->host copy of the refined point map and the per-frame (s, t) of the last LiDAR fit -- the refine loop
of MoGeModel.forward (moge/model/v3.py:537-576) for ``infer(model, image, lidar, conf, refine_steps=K)``.
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import torch

from . import synth
from .engine import Geometry, RefinerEngine
from . import ops
from .ops import fit_state_view

_CLIPS = Path(__file__).resolve().parent / "synth_clips.json"


def synthetic_model(model: str = "A", seed: int = 0):
    """Random-init weights of a model's refiner and the activation clips the reference's observer pass produced for
    them on the seed-0 synthetic frame (tests/golden/make_golden.py)."""
    weights = synth.make_refiner_weights(model, seed)
    m = synth.MODELS[model]
    clips = json.loads(_CLIPS.read_text())[f"{model}_{m['H']}x{m['W']}_seed{seed}"]
    return weights, clips


class Refiner:
    def __init__(self, weights: dict, clips: dict, model: str = "A", height: int | None = None,
                 width: int | None = None, batch: int = 1, device="cuda", capacity=None, channels=None,
                 enc_channels: int = synth.ENC_CHANNELS, depth_resolution: float = synth.DEPTH_RESOLUTION,
                 uv_bias=None, max_split: int = 4, pdl: bool = True):
        m = synth.MODELS[model] if model is not None else {}
        self.geo = Geometry(channels=list(channels or m["model_channels"]), height=height or m["H"],
                            width=width or m["W"], batch=batch, enc_channels=enc_channels,
                            depth_resolution=depth_resolution)
        self.default_uv = uv_bias      # baked UV conditioning [C_last, h, w] used when refine() gets none
        self.device = torch.device(device)
        self.engine = RefinerEngine(weights, clips, self.geo, device=self.device, capacity=capacity,
                                    max_split=max_split, pdl=pdl)
        B, H, W = batch, self.geo.height, self.geo.width
        ed = 2 ** (self.geo.levels - 1)
        lh, lw = self.geo.lidar_hw
        dev = self.device
        # device-resident inputs the graph reads, and pinned host staging
        self.d_pc = torch.empty((B, H, W, 3), dtype=torch.float32, device=dev)
        self.d_ld = torch.empty((B, 1, lh, lw), dtype=torch.float32, device=dev)
        self.d_lc = torch.empty((B, 1, lh, lw), dtype=torch.float32, device=dev)
        self.d_enc = torch.empty((B, self.geo.enc_channels, H // ed, W // ed), dtype=torch.float16, device=dev)
        self.d_uv = torch.empty((B, self.geo.channels[-1], H // ed, W // ed), dtype=torch.float32, device=dev)
        self.h_out = torch.empty((B, H, W, 3), dtype=torch.float32).pin_memory()
        self.h_fit = torch.empty((B, 18), dtype=torch.int32).pin_memory()
        self.engine.set_inputs(self.d_pc, self.d_ld, self.d_lc)
        self._K = None
        self._raw = None
        self._uv_dev = None
        self._side = None

    def input_bytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in (self.d_pc, self.d_ld, self.d_lc, self.d_enc, self.d_uv))

    def output_bytes(self) -> int:
        return self.h_out.numel() * 4 + self.h_fit.numel() * 4

    def _ensure_graph(self, K: int):
        if self._K != K:
            self.engine.set_inputs(self.d_pc, self.d_ld, self.d_lc)
            self.engine.capture(K)
            self._K = K

    def refine(self, point_coord, lidar_depth, lidar_conf, encoder_feature, uv_bias=None, K: int = 1,
               sync: bool = True, fill: bool = False, out: torch.Tensor | None = None):
        """Refine a batch of frames.  Host arrays/tensors (pinned CPU tensors copy asynchronously):
        point_coord [B,H,W,3] fp32, lidar_depth/lidar_conf [B,1,192,256] fp32, encoder_feature [B,1024,h,w] fp16,
        uv_bias [B,C,h,w] fp32 or None.  fill=True first applies promptmoge.nearest_fill to the sensor frames on the
        device (promptmoge.infer does so by default before the model sees them, promptmoge/model.py:93-94).
        out: a host tensor [B,H,W,3] (pinned for an asynchronous copy) the refined point map is copied into instead of
        the Refiner's own staging buffer.  Returns (refined point map [B,H,W,3] host tensor, fit list)."""
        self._ensure_graph(K)
        s = torch.cuda.current_stream(self.device)
        if fill:
            if self._raw is None:
                self._raw = (torch.empty_like(self.d_ld), torch.empty_like(self.d_lc))
            ld, lc = self._raw
        else:
            ld, lc = self.d_ld, self.d_lc
        # the step's own inputs on the step's stream; the per-frame conditioning (encoder feature, UV planes,
        # encoder_fuse) on a side stream that the step waits for only before its encoder fusion, so its copy and
        # kernels overlap the finer levels.  The side stream waits for the step's input copies (and so for the
        # previous call's step): its host copies then follow them on the bus instead of sharing it with them.
        if self._side is None:
            self._side = torch.cuda.Stream(self.device)
        for dst, src in ((self.d_pc, point_coord), (ld, lidar_depth), (lc, lidar_conf)):
            dst.copy_(torch.as_tensor(src), non_blocking=True)
        self._side.wait_stream(s)
        if fill:
            ops.nearest_fill(ld, lc, out=(self.d_ld, self.d_lc))
        with torch.cuda.stream(self._side):
            for src in (encoder_feature, uv_bias):
                # a device tensor read on the side stream stays allocated until that stream is done with it
                if isinstance(src, torch.Tensor) and src.is_cuda:
                    src.record_stream(self._side)
            self.d_enc.copy_(torch.as_tensor(encoder_feature), non_blocking=True)
            if uv_bias is None and self.default_uv is not None:
                if self._uv_dev is None:
                    self._uv_dev = torch.as_tensor(self.default_uv).to(self.device).expand_as(self.d_uv).contiguous()
                self.d_uv.copy_(self._uv_dev)
                uv_bias = self._uv_dev
            elif uv_bias is not None:
                self.d_uv.copy_(torch.as_tensor(uv_bias), non_blocking=True)
            self.engine.set_frame(self.d_enc, self.d_uv if uv_bias is not None else None)
        res, fit = self.engine.replay()
        dst = self.h_out if out is None else out
        dst.copy_(res, non_blocking=True)
        self.h_fit.copy_(fit, non_blocking=True)
        if sync:
            s.synchronize()
            return dst, fit_state_view(self.h_fit)
        return dst, None

    @classmethod
    def from_refiner_dir(cls, path, batch: int = 1, device="cuda", capacity=None):
        """A Refiner running the deployed int8 weights of a refiner.bin / refiner.json directory (the Metal
        engine's ``Refiner(dir:)``, Refiner.swift:65-116): int8 weights and scales as stored, fp16 parameters
        widened to fp32, the baked UV conditioning used whenever refine() is given no uv_bias."""
        from .refiner_bin import read_refiner_dir
        dep = read_refiner_dir(path)
        return cls(dep.weights, dep.clips, model=None, height=dep.height, width=dep.width, batch=batch,
                   device=device, capacity=capacity, channels=dep.channels, enc_channels=dep.enc_channels,
                   depth_resolution=dep.depth_resolution, uv_bias=dep.uv_bias)

    def close(self):
        self.engine.close()


def pinned(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a)).pin_memory()
