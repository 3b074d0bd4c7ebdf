"""The fused int8 refiner runtime: a plan per (model geometry, batch), K refine steps captured in one CUDA graph.

Replaces the refine loop of MoGeModel.forward (moge/model/v3.py:537-576): per step the LiDAR fit
(_lidar_in_affine_frame, v3.py:362-383), the prompt features, _voxelize (v3.py:305-344), Sparse3DUNet.forward
(moge/model/modules/sparse_unet.py:176-258) on int8 layers, and logz += delta (v3.py:358-359).

Weights are taken from a reference-format state dict (fp32 master weights under the reference's module names) plus
the QAT activation clips, and quantised with the training / export rule (moge/model/modules/qat.py:40-57,
promptmoge/export/refiner.py:40-46): per output channel s_w = amax / 127, q_w = clamp(round(w / s_w), +-127).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from ._lib import RefinerConfig, call

QMAX = np.float32(127.0)


def quantise_weight(w: np.ndarray):
    """Per-output-channel int8 of a fp32 weight (axis 0 = output channel): (q int8, s fp32 [Co])."""
    w = np.asarray(w, np.float32)
    amax = np.abs(w).reshape(w.shape[0], -1).max(axis=1)
    s = np.maximum((amax / QMAX).astype(np.float32), np.float32(1e-12))
    q = np.clip(np.rint(w / s.reshape((-1,) + (1,) * (w.ndim - 1))), -QMAX, QMAX).astype(np.int8)
    return q, s


def act_scale(clip: float) -> float:
    """s_a = clip / 127 in fp32 (qat.py:97 with _fake_quant's clamp_min(1e-12))."""
    return float(max(np.float32(clip) / QMAX, np.float32(1e-12)))


def quantised_layer_names(levels: int) -> list:
    """The 31 (Model A) / 25 (Model B) layers enable_refiner_qat quantises (qat.py:118-138)."""
    names = ["encoder_fuse", "fuse_proj.0", "fuse_proj.2"]
    for k in range(levels):
        names += [f"down_stages.{k}.0.conv1", f"down_stages.{k}.0.conv2"]
    names += [f"downsample_blocks.{k}.linear" for k in range(levels - 1)]
    names += ["bottleneck_stage.0.conv1", "bottleneck_stage.0.conv2"]
    names += [f"upsample_blocks.{i}.linear" for i in range(levels - 1)]
    for i in range(levels - 1):
        names += [f"up_stages.{i}.0.conv1", f"up_stages.{i}.0.conv2"]
    return names


def state_dict_from_module(unet) -> tuple[dict, dict]:
    """(fp32 master weights by reference name, activation clips) from a reference Sparse3DUNet, QAT or not."""
    sd = {}
    for k, v in unet.state_dict().items():
        k2 = k.replace(".parametrizations.weight.original", ".weight")
        if k2.startswith("aq_") or k2.endswith(".observed") or k2.endswith(".clip"):
            continue
        sd[k2] = v.detach().float().cpu().numpy()
    clips = {}
    for name, mod in unet.named_modules():
        if hasattr(mod, "weight") and hasattr(unet, "aq_" + name.replace(".", "_")):
            clips[name] = float(getattr(unet, "aq_" + name.replace(".", "_")).clip)
    return sd, clips


@dataclass
class Geometry:
    channels: list
    height: int
    width: int
    batch: int = 1
    enc_channels: int = 1024
    lidar_hw: tuple = (192, 256)
    depth_resolution: float = 256.0

    @property
    def levels(self) -> int:
        return len(self.channels)


class RefinerEngine:
    """Device-resident int8 refiner.  All tensors it returns live on `device`."""

    def __init__(self, weights: dict, clips: dict, geometry: Geometry, device="cuda", capacity=None,
                 use_prompt: bool = True, tensor_cores: bool = True, max_split: int = 4,
                 output_gate_floor: float | None = None, anchor_beta: float = 0.0, pdl: bool = True,
                 soft_gate: bool = True, multi_launch_fit: bool = False, multi_launch_transitions: bool = False):
        _lib.load()
        self.geo = geometry
        self.device = torch.device(device)
        self.use_prompt = use_prompt
        self.tensor_cores = tensor_cores
        L = geometry.levels
        cfg = RefinerConfig()
        cfg.batch, cfg.height, cfg.width, cfg.levels = geometry.batch, geometry.height, geometry.width, L
        for k, c in enumerate(geometry.channels):
            cfg.channels[k] = c
        cfg.enc_channels = geometry.enc_channels
        cfg.lidar_h, cfg.lidar_w = geometry.lidar_hw
        cfg.depth_resolution = geometry.depth_resolution
        cfg.soft_gate, cfg.fit_iters, cfg.fit_trim, cfg.fit_min_points = int(soft_gate), 4, 0.2, 32
        cfg.use_prompt = int(use_prompt)
        cfg.use_tensor_cores = int(tensor_cores)
        cfg.max_split = int(max_split)
        # the optional refiner-side gates (off in the released configs): refiner_output_gate / output_gate_floor,
        # anchor_strength (moge/model/v3.py:116-118, 565-573)
        cfg.output_gate = int(output_gate_floor is not None)
        cfg.output_gate_floor = float(output_gate_floor) if output_gate_floor is not None else 0.1
        cfg.anchor_beta = float(anchor_beta)
        cfg.use_pdl = int(pdl)
        cfg.multi_launch_fit = int(multi_launch_fit)
        cfg.multi_launch_transitions = int(multi_launch_transitions)
        for k in range(L):
            cfg.capacity[k] = int(capacity[k]) if capacity is not None else 0
        self._cfg = cfg
        with torch.cuda.device(self.device):
            h = C.c_void_p()
            call("pmg_refiner_create", C.byref(cfg), C.byref(h))
        self._h = h
        self._keep = []       # device tensors the plan points into
        self._load_weights(weights, clips)
        self._graph_key = None

    # -- weights ------------------------------------------------------------------------------------------------- #
    def _t(self, a, dtype):
        t = torch.as_tensor(np.ascontiguousarray(a)).to(device=self.device, dtype=dtype).contiguous()
        self._keep.append(t)
        return C.c_void_p(t.data_ptr())

    def _load_weights(self, w: dict, clips: dict):
        L = self.geo.levels
        for name in quantised_layer_names(L):
            if name + ".weight_q8" in w:      # already quantised (a deployed refiner.bin): used as stored
                q = np.asarray(w[name + ".weight_q8"], np.int8)
                s = np.asarray(w[name + ".weight_scale"], np.float32)
            else:
                q, s = quantise_weight(w[name + ".weight"])
            if q.ndim == 5:      # (Co, 3, 3, 3, Ci) -> tap-major [27][Co][Ci]
                q = q.reshape(q.shape[0], 27, q.shape[-1]).transpose(1, 0, 2)
            call("pmg_refiner_set_qlayer", self._h, name.encode(), self._t(q, torch.int8),
                 self._t(s, torch.float32), self._t(w[name + ".bias"], torch.float32), act_scale(clips[name]))
        blocks = [f"down_stages.{k}.0" for k in range(L)] + ["bottleneck_stage.0"] + \
                 [f"up_stages.{i}.0" for i in range(L - 1)]
        for b in blocks:
            call("pmg_refiner_set_norm", self._h, (b + ".norm1").encode(), self._t(w[b + ".norm1.weight"], torch.float32),
                 self._t(w[b + ".norm1.bias"], torch.float32))
        for p in ("input_proj", "prompt_proj", "out_proj"):
            if p == "prompt_proj" and not self.use_prompt:
                continue
            call("pmg_refiner_set_proj", self._h, p.encode(), self._t(w[p + ".weight"], torch.float32),
                 self._t(w[p + ".bias"], torch.float32))

    # -- per frame / per run ------------------------------------------------------------------------------------- #
    def set_frame(self, encoder_feature: torch.Tensor, uv_bias: torch.Tensor | None = None):
        """encoder_feature [B,1024,h,w] (fp16 on device), uv_bias [B,C_last,h,w] fp32 or None."""
        enc = encoder_feature.to(device=self.device, dtype=torch.float16).contiguous()
        uvb = uv_bias.to(device=self.device, dtype=torch.float32).contiguous() if uv_bias is not None else None
        self._enc, self._uvb = enc, uvb
        call("pmg_refiner_set_frame", self._h, C.c_void_p(enc.data_ptr()),
             C.c_void_p(uvb.data_ptr()) if uvb is not None else None, self._stream())

    def set_inputs(self, point_coord: torch.Tensor, lidar_depth: torch.Tensor | None, lidar_conf: torch.Tensor | None):
        """Device tensors [B,H,W,3] fp32, [B,1,h,w] fp32, [B,1,h,w] fp32; the plan reads them when it runs."""
        self._pc = point_coord.to(device=self.device, dtype=torch.float32).contiguous()
        self._ld = lidar_depth.to(device=self.device, dtype=torch.float32).contiguous() if lidar_depth is not None else None
        self._lc = lidar_conf.to(device=self.device, dtype=torch.float32).contiguous() if lidar_conf is not None else None
        call("pmg_refiner_set_inputs", self._h, C.c_void_p(self._pc.data_ptr()),
             C.c_void_p(self._ld.data_ptr()) if self._ld is not None else None,
             C.c_void_p(self._lc.data_ptr()) if self._lc is not None else None)
        self._graph_key = None

    def set_prompt(self, prompt_feats: torch.Tensor | None):
        """Prompt features [B*H*W, 2] fp32 on the device that every step reads instead of running its own LiDAR fit
        (the prompt_feats argument of MoGeModel._refine_logz); None restores the plan's own fit."""
        self._prompt = None if prompt_feats is None else \
            prompt_feats.to(device=self.device, dtype=torch.float32).contiguous()
        call("pmg_refiner_set_prompt", self._h, C.c_void_p(self._prompt.data_ptr()) if self._prompt is not None else None)
        self._graph_key = None

    def _outputs(self):
        if getattr(self, "_out", None) is None or self._out.shape != self._pc.shape:
            self._out = torch.empty_like(self._pc)
            self._fit = torch.zeros((self.geo.batch, 18), dtype=torch.int32, device=self.device)
        return self._out, self._fit

    @staticmethod
    def _stream():
        return C.c_void_p(torch.cuda.current_stream().cuda_stream)

    def run(self, K: int = 1):
        """Enqueue K steps on the current stream (no graph).  Returns (refined point map, fit state) tensors."""
        out, fit = self._outputs()
        call("pmg_refiner_enqueue", self._h, int(K), C.c_void_p(out.data_ptr()), C.c_void_p(fit.data_ptr()),
             self._stream())
        return out, fit

    def capture(self, K: int = 1):
        """Capture K steps into the plan's CUDA graph (re-capture when K or the input tensors change)."""
        out, fit = self._outputs()
        torch.cuda.synchronize(self.device)
        call("pmg_refiner_capture", self._h, int(K), C.c_void_p(out.data_ptr()), C.c_void_p(fit.data_ptr()), None)
        self._graph_key = (K, self._pc.data_ptr())
        return out, fit

    def replay(self):
        call("pmg_refiner_launch", self._h, self._stream())
        return self._out, self._fit

    def status(self, clear: bool = True):
        """(status code, required voxel count per level of the last step); synchronises the current stream."""
        counts = (C.c_int32 * self.geo.levels)()
        rc = _lib.load().pmg_refiner_status(self._h, counts, int(clear), self._stream())
        return rc, list(counts)

    def set_capacity(self, caps):
        arr = (C.c_int64 * 8)(*([int(c) for c in caps] + [0] * (8 - len(caps))))
        call("pmg_refiner_set_capacity", self._h, arr)
        self._graph_key = None

    def fit_to(self, counts, headroom: float = 1.25, align: int = 1024):
        """Shrink/grow level capacities to the measured counts with headroom (level 0 stays exact)."""
        caps = [int(np.ceil(c * headroom / align) * align) for c in counts]
        caps[0] = 0
        self.set_capacity(caps)

    def launches_per_step(self) -> int:
        return _lib.load().pmg_refiner_launches_per_step(self._h)

    def level_info(self, level: int):
        cap, H, W, Cc = C.c_int64(), C.c_int32(), C.c_int32(), C.c_int32()
        call("pmg_refiner_level_info", self._h, level, C.byref(cap), C.byref(H), C.byref(W), C.byref(Cc))
        return dict(cap=cap.value, H=H.value, W=W.value, C=Cc.value)

    def debug_tensor(self, what: str, level: int, shape, dtype):
        """A torch view of a plan buffer (for parity checks); valid until the plan is resized or freed."""
        ptr = _lib.load().pmg_refiner_debug_ptr(self._h, what.encode(), level)
        if not ptr:
            raise KeyError(what)
        n = int(np.prod(shape))
        esize = torch.empty((), dtype=dtype).element_size()
        buf = _device_view(ptr, n * esize, self.device)
        return buf.view(dtype)[:n].view(*shape)

    def close(self):
        if getattr(self, "_h", None):
            _lib.load().pmg_refiner_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _device_view(ptr: int, nbytes: int, device) -> torch.Tensor:
    """Wrap raw device memory as a uint8 tensor without copying (the owner outlives the view)."""
    class _Holder:
        pass
    h = _Holder()
    h.__cuda_array_interface__ = dict(shape=(nbytes,), typestr="|u1", data=(ptr, False), version=3, strides=None)
    return torch.as_tensor(h, device=device)
