"""A stand-in for the reference's MoGeModel around its refiner, for the install_refiner tests.

The reference model (ViT backbone, heads, trained checkpoints) is not available where the tests run, so this stub
carries exactly what the refine loop of MoGeModel.forward (moge/model/v3.py:537-576) touches: ``refiner`` (a module
tree with the reference Sparse3DUNet's attribute and parameter names, moge/model/modules/sparse_unet.py:33-120, and
one activation-clip holder ``aq_<layer>`` per int8 QAT layer, moge/model/modules/qat.py:101-115),
``refiner_depth_resolution``, ``lidar_prompt_cfg``, and the two methods the loop calls, which here refuse to run so a
test can tell that the hook replaced them.  ``refine_loop`` makes the loop's per-step calls in the loop's order.
"""
from __future__ import annotations

import torch
from torch import nn


class _Conv(nn.Module):
    def __init__(self, ci: int, co: int):
        super().__init__()
        self.weight = nn.Parameter(torch.zeros(co, 3, 3, 3, ci))
        self.bias = nn.Parameter(torch.zeros(co))


class _ResBlock(nn.Module):
    def __init__(self, c: int):
        super().__init__()
        self.norm1 = nn.LayerNorm(c, eps=1e-6)
        self.conv1 = _Conv(c, c)
        self.conv2 = _Conv(c, c)


class _Linear(nn.Module):
    def __init__(self, ci: int, co: int):
        super().__init__()
        self.linear = nn.Linear(ci, co)


class _Clip(nn.Module):
    def __init__(self, clip: float):
        super().__init__()
        self.register_buffer("clip", torch.tensor(float(clip)))


class StubRefiner(nn.Module):
    def __init__(self, channels, encoder_channels=1024, prompt_channels=2, blocks=1):
        super().__init__()
        L = len(channels)
        self.prompt_channels = prompt_channels
        self.downsample_factors = [2] * (L - 1)
        self.encoder_downsample = 2 ** (L - 1)
        self.input_proj = nn.Linear(3, channels[0])
        if prompt_channels:
            self.prompt_proj = nn.Linear(prompt_channels, channels[0])
        self.encoder_fuse = nn.Linear(encoder_channels, channels[-1])
        self.fuse_proj = nn.Sequential(nn.Linear(2 * channels[-1], channels[-1]), nn.SiLU(),
                                       nn.Linear(channels[-1], channels[-1]))
        self.down_stages = nn.ModuleList(nn.ModuleList(_ResBlock(c) for _ in range(blocks)) for c in channels)
        self.downsample_blocks = nn.ModuleList(_Linear(channels[k], channels[k + 1]) for k in range(L - 1))
        self.bottleneck_stage = nn.ModuleList([_ResBlock(channels[-1])])
        self.upsample_blocks = nn.ModuleList(_Linear(channels[L - 1 - i], channels[L - 2 - i]) for i in range(L - 1))
        self.up_stages = nn.ModuleList(nn.ModuleList([_ResBlock(channels[L - 2 - i])]) for i in range(L - 1))
        self.out_proj = nn.Linear(channels[0], 1)

    def attach_clips(self, clips: dict):
        for name, clip in clips.items():
            self.add_module("aq_" + name.replace(".", "_"), _Clip(clip))


class StubMoGe(nn.Module):
    def __init__(self, refiner: nn.Module, soft_residual_gate: bool = True):
        super().__init__()
        self.refiner = refiner
        self.refiner_depth_resolution = 256.0
        self.lidar_prompt_cfg = {"soft_residual_gate": soft_residual_gate}

    def _refine_logz(self, point_coord, encoder_feature, prompt_feats=None, encoder_bias_map=None, refiner=None):
        raise AssertionError("the stub's own _refine_logz ran: the hook is not installed")

    @staticmethod
    def _lidar_in_affine_frame(logz, lidar_depth, lidar_conf, soft_gate=False):
        raise AssertionError("the stub's own _lidar_in_affine_frame ran: the hook is not installed")

    def refine_loop(self, coord, feature, uv_bias, lidar_depth, lidar_conf, steps: int):
        """The refine loop's calls per step (v3.py:547-559, 574): fit in the affine frame, prompt features from the
        gated residual, the refiner step, the new coordinate map."""
        soft = bool(self.lidar_prompt_cfg.get("soft_residual_gate", False))
        for _ in range(steps):
            logz = coord[..., 2]
            log_d_aff, gate, _, _ = self._lidar_in_affine_frame(logz, lidar_depth, lidar_conf, soft_gate=soft)
            prompt = torch.stack([(log_d_aff - logz) * gate, gate], dim=-1).reshape(-1, 2)
            refined = self._refine_logz(coord, feature, prompt_feats=prompt, encoder_bias_map=uv_bias)
            coord = torch.cat([coord[..., :2], refined.unsqueeze(-1)], dim=-1)
        return coord


def stub_model(model: str = "B", seed: int = 0, qat: bool = True, blocks: int = 1) -> StubMoGe:
    """A stub with the synthetic refiner's weights (promptmoge_b200.synth) and the reference observer's clips."""
    from promptmoge_b200 import synth
    from promptmoge_b200.refine import synthetic_model
    weights, clips = synthetic_model(model, seed)
    unet = StubRefiner(synth.MODELS[model]["model_channels"], blocks=blocks)
    if blocks == 1:
        unet.load_state_dict({k: torch.from_numpy(v) for k, v in weights.items()}, strict=True)
    if qat:
        unet.attach_clips(clips)
    return StubMoGe(unet.eval())


# ---- stand-ins for the reference's QAT wrappers (moge/model/modules/qat.py:40-115), for the flex_gemm drop-in's
# int8 routing: a per-output-channel weight parametrisation and a per-tensor input quantiser attached as a forward
# pre-hook, with the attribute names the reference's classes carry (ch_dim / enabled, clip / observed / enabled).
class StubWeightFakeQuant(nn.Module):
    def __init__(self):
        super().__init__()
        self.ch_dim, self.enabled = 0, True

    def forward(self, w):
        dims = [d for d in range(w.ndim) if d != 0]
        s = (w.detach().abs().amax(dim=dims, keepdim=True) / 127.0).float().clamp_min(1e-12)
        return torch.clamp(torch.round(w.float() / s), -127, 127) * s


class StubActFakeQuant(nn.Module):
    def __init__(self, clip: float):
        super().__init__()
        self.enabled = True
        self.register_buffer("clip", torch.tensor(float(clip)))
        self.register_buffer("observed", torch.ones((), dtype=torch.long))

    def forward(self, x):
        s = (self.clip / 127.0).float().clamp_min(1e-12)
        return torch.clamp(torch.round(x.float() / s), -127, 127) * s


def stub_qat(module: nn.Module, clip: float) -> StubActFakeQuant:
    """Wrap one conv / linear the way enable_refiner_qat does (parametrisation + input pre-hook)."""
    import torch.nn.utils.parametrize as P
    P.register_parametrization(module, "weight", StubWeightFakeQuant())
    aq = StubActFakeQuant(clip)

    def make_hook(q):
        def hook(mod, args):
            return (q(args[0]), *args[1:])
        return hook
    module.register_forward_pre_hook(make_hook(aq))
    return aq
