"""The B200 refiner under the reference's own model API: ``install_refiner(model)``.

PromptMoGe's user entry point ``promptmoge.infer(model, image, lidar, conf, refine_steps=K)``
(promptmoge/model.py:75-100) calls ``MoGeModel.infer`` -> ``MoGeModel.forward``, whose refine loop
(moge/model/v3.py:537-576) runs, per step:

    log_d_aff, gate, s, t = self._lidar_in_affine_frame(logz, lidar_depth, lidar_conf, soft_gate=...)   (v3.py:362-383)
    prompt_feats = stack([(log_d_aff - logz) * gate, gate])                                               (v3.py:554-555)
    refined_logz = self._refine_logz(coord, feature, prompt_feats=..., encoder_bias_map=...)              (v3.py:346-360)

``install_refiner`` binds both methods of one model instance to this library: ``_lidar_in_affine_frame`` becomes the
trimmed least-squares fit and affine-frame kernels (pmg_fit_prep_prompt, pmg_fit_solve, pmg_affine_frame), and
``_refine_logz`` becomes one replay of a captured CUDA graph of the refiner plan (voxelisation, the level structure,
the int8 U-Net of the model's own QAT weights, logz += delta) that reads the prompt features the loop passes in.  The
loop itself, ``promptmoge.infer`` and every caller stay unchanged; the optional output gate and elastic anchor of the
loop (v3.py:565-573) keep running as the reference wrote them, on top of the hooked fit.

The weights are the model's own: every quantised layer's fp32 master weight and activation clip
(moge/model/modules/qat.py:101-138), quantised per output channel with the training / export rule.  There is no CPU
path: inputs that are not CUDA tensors raise.
"""
from __future__ import annotations

import torch

from . import ops
from .engine import Geometry, RefinerEngine, quantised_layer_names, state_dict_from_module

PMG_ERR_OVERFLOW = 4


def refiner_geometry(unet) -> dict:
    """Layer geometry of a reference Sparse3DUNet (moge/model/modules/sparse_unet.py:33-120) that the plan supports:
    one residual block per stage, factor-2 pooling, 3x3x3 convs."""
    channels = [int(stage[0].norm1.normalized_shape[0]) for stage in unet.down_stages]
    if any(len(stage) != 1 for stage in unet.down_stages) or any(len(s) != 1 for s in unet.up_stages) or \
            len(unet.bottleneck_stage) != 1:
        raise NotImplementedError("the B200 refiner plan runs one residual block per stage")
    if any(int(f) != 2 for f in unet.downsample_factors):
        raise NotImplementedError(f"the B200 refiner plan pools by 2, got {unet.downsample_factors}")
    return dict(channels=channels, enc_channels=int(unet.encoder_fuse.weight.shape[1]),
                prompt_channels=int(getattr(unet, "prompt_channels", 0) or 0),
                encoder_downsample=int(unet.encoder_downsample))


class _Plan:
    """One refiner plan and its captured one-step graph for a (batch, height, width, prompt) shape."""

    def __init__(self, hook: "RefinerHook", B: int, H: int, W: int, use_prompt: bool, device):
        self.device = device
        geo = Geometry(channels=hook.geo["channels"], height=H, width=W, batch=B, enc_channels=hook.geo["enc_channels"],
                       depth_resolution=hook.depth_resolution)
        self.engine = RefinerEngine(hook.weights, hook.clips, geo, device=device, use_prompt=use_prompt,
                                    max_split=hook.max_split, pdl=hook.pdl)
        self.pc = torch.empty((B, H, W, 3), dtype=torch.float32, device=device)
        self.prompt = torch.empty((B * H * W, 2), dtype=torch.float32, device=device) if use_prompt else None
        self.engine.set_inputs(self.pc, None, None)
        self.engine.set_prompt(self.prompt)
        self._frame = None          # the encoder feature / bias tensors of the last set_frame (held, so not reused)
        self._captured = False

    def _capture(self):
        self.engine.capture(1)
        self._captured = True

    def _set_frame(self, encoder_feature, encoder_bias_map):
        key = (encoder_feature, encoder_feature._version, encoder_bias_map,
               None if encoder_bias_map is None else encoder_bias_map._version)
        last = self._frame
        if last is not None and last[0] is key[0] and last[1] == key[1] and last[2] is key[2] and last[3] == key[3]:
            return
        self.engine.set_frame(encoder_feature, encoder_bias_map)
        self._frame = key

    def _resized(self, encoder_feature, encoder_bias_map):
        """After a capacity change: the plan's buffers (the frame's encoder tokens among them) are new, so the frame
        is conditioned again and the step re-captured."""
        self.engine.set_inputs(self.pc, None, None)
        self._frame = None
        self._set_frame(encoder_feature, encoder_bias_map)
        self._capture()

    def step(self, point_coord, encoder_feature, prompt_feats, encoder_bias_map):
        self.pc.copy_(point_coord)
        if self.prompt is not None:
            self.prompt.copy_(prompt_feats.reshape(self.prompt.shape))
        self._set_frame(encoder_feature, encoder_bias_map)
        if not self._captured:
            # first call: run with every level sized for the whole frame (cannot overflow), then shrink the levels
            # to the measured voxel counts with headroom and capture the step
            self.engine.run(1)
            rc, counts = self.engine.status()
            if rc != 0:
                raise RuntimeError(f"B200 refiner: device status {rc}")
            self.engine.fit_to(counts)
            self._resized(encoder_feature, encoder_bias_map)
        out, _ = self.engine.replay()
        rc, _ = self.engine.status()
        if rc == PMG_ERR_OVERFLOW:
            # a level outgrew its buffers (the Metal engine's overflow flag + regrow, VoxelStructure.swift:200-217):
            # back to whole-frame capacities, re-capture, and run the step again
            self.engine.set_capacity([0] * self.engine.geo.levels)
            self._resized(encoder_feature, encoder_bias_map)
            out, _ = self.engine.replay()
            rc, _ = self.engine.status()
        if rc != 0:
            raise RuntimeError(f"B200 refiner: device status {rc}")
        return out[..., 2].clone()

    def close(self):
        self.engine.close()


class RefinerHook:
    """The replacements of ``_refine_logz`` and ``_lidar_in_affine_frame`` for one MoGeModel instance."""

    def __init__(self, model, max_split: int = 4, pdl: bool = True):
        unet = model.refiner
        self.model = model
        self.geo = refiner_geometry(unet)
        self.weights, self.clips = state_dict_from_module(unet)
        missing = [n for n in quantised_layer_names(len(self.geo["channels"])) if n not in self.clips]
        if missing:
            raise ValueError("the refiner is not int8 QAT (enable_refiner_qat, moge/model/modules/qat.py:118-138): "
                             f"no activation clip for {missing[:3]}")
        self.depth_resolution = float(getattr(model, "refiner_depth_resolution", 256.0))
        self.max_split, self.pdl = max_split, pdl
        self._plans: dict = {}
        self._orig_refine = type(model)._refine_logz
        self._orig_affine = type(model)._lidar_in_affine_frame

    @staticmethod
    def _cuda(t: torch.Tensor, name: str):
        if not isinstance(t, torch.Tensor) or not t.is_cuda:
            raise RuntimeError(f"B200 refiner: {name} must be a CUDA tensor (this library has no CPU path)")

    def lidar_in_affine_frame(self, logz, lidar_depth, lidar_conf, soft_gate: bool = False):
        """MoGeModel._lidar_in_affine_frame (v3.py:362-383): (log_d_aff, gate, s, t) from the device fit."""
        for t, n in ((logz, "logz"), (lidar_depth, "lidar_depth"), (lidar_conf, "lidar_conf")):
            self._cuda(t, n)
        return ops.lidar_in_affine_frame(logz.float(), lidar_depth.float().contiguous(),
                                         lidar_conf.float().contiguous(), soft_gate=bool(soft_gate))

    def refine_logz(self, point_coord, encoder_feature, prompt_feats=None, encoder_bias_map=None, refiner=None):
        """MoGeModel._refine_logz (v3.py:346-360): refined log-depth [B,H,W] of one refine step."""
        if refiner is not None and refiner is not self.model.refiner:
            # another refiner (the distillation teacher of training, v3.py:558-563) is not this plan's
            return self._orig_refine(self.model, point_coord, encoder_feature, prompt_feats=prompt_feats,
                                     encoder_bias_map=encoder_bias_map, refiner=refiner)
        self._cuda(point_coord, "point_coord")
        self._cuda(encoder_feature, "encoder_feature")
        B, H, W, _ = point_coord.shape
        ed = self.geo["encoder_downsample"]
        if encoder_feature.shape[-2:] != (H // ed, W // ed):
            raise ValueError(f"encoder feature {tuple(encoder_feature.shape)} does not match a {H}x{W} point map")
        use_prompt = prompt_feats is not None
        if use_prompt and not self.geo["prompt_channels"]:
            raise ValueError("prompt features given to a refiner built without prompt_channels")
        key = (B, H, W, use_prompt, point_coord.device)
        plan = self._plans.get(key)
        if plan is None:
            plan = self._plans[key] = _Plan(self, B, H, W, use_prompt, point_coord.device)
        return plan.step(point_coord, encoder_feature, prompt_feats, encoder_bias_map)

    def close(self):
        for p in self._plans.values():
            p.close()
        self._plans.clear()


def install_refiner(model, max_split: int = 4, pdl: bool = True) -> RefinerHook:
    """Run ``model``'s refine loop (moge/model/v3.py:537-576) on this library, for every later ``model.forward`` /
    ``model.infer`` / ``promptmoge.infer(model, ...)`` call: the instance's ``_refine_logz`` and
    ``_lidar_in_affine_frame`` are replaced by the hook's; ``uninstall_refiner`` restores them."""
    if getattr(model, "_pmg_refiner_hook", None) is not None:
        return model._pmg_refiner_hook
    hook = RefinerHook(model, max_split=max_split, pdl=pdl)
    model._refine_logz = hook.refine_logz
    model._lidar_in_affine_frame = hook.lidar_in_affine_frame
    model._pmg_refiner_hook = hook
    return hook


def uninstall_refiner(model) -> None:
    hook = getattr(model, "_pmg_refiner_hook", None)
    if hook is None:
        return
    for name in ("_refine_logz", "_lidar_in_affine_frame", "_pmg_refiner_hook"):
        if name in model.__dict__:
            del model.__dict__[name]
    hook.close()
