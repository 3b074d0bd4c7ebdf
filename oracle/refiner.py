"""Oracle (test infrastructure): the narrowed int8 QAT refiner's forward, restated in numpy with exact integer
accumulation.

The reference runs the refiner as fp32 PyTorch on its bundled FlexGEMM fallback with fake quantisation
(moge/model/modules/qat.py): every SubmanifoldConv3d / nn.Linear except input/prompt/out proj quantises its input per
tensor, q = clamp(round(x / s_a), -127, 127) with s_a = clip / 127 in fp32 (qat.py:28-37, 60-98, 101-115), and its
weight per output channel, q_w = clamp(round(w / s_w), -127, 127), s_w = amax|w[n]| / 127 (qat.py:40-57; the same
rule the exporter re-derives, promptmoge/export/refiner.py:40-46).  The deployed arithmetic
(SparseConvInt8.metal:1-21; verify_int8.py:86-103) is the integer form of that layer:

    acc[o, n] = sum_v sum_c q[nmap[o, v], c] * q_w[n, v, c]          (exact; float64 here, |acc| < 2^53)
    y[o, n]   = (float(acc) * s_a) * s_w[n] + b[n]                      (fp32, this operation order)

which equals the fake-quant fp32 layer up to fp32 rounding.  Everything between quantised layers (LayerNorm eps 1e-6,
SiLU, mean pool, nearest upsample, residuals, input/prompt/out projections) is fp32 as in the reference
(flex_sparse_blocks.py:50-105, sparse_unet.py:176-258, _core.py:399-505).
"""
from __future__ import annotations

import numpy as np

from . import structure

f32 = np.float32
QMAX = f32(127.0)


def act_scale(clip: float) -> np.float32:
    """s_a = clip / 127 in fp32, clamped at 1e-12 (qat.py:34-35, 97)."""
    return max(f32(clip) / QMAX, f32(1e-12))


def quant_act(x: np.ndarray, clip: float):
    """q = clamp(round(x / s_a), -127, 127) (qat.py:35-36), round half to even in fp32."""
    s = act_scale(clip)
    q = np.clip(np.rint(np.asarray(x, f32) / s), -QMAX, QMAX).astype(np.int8)
    return q, s


def quant_weight(w: np.ndarray):
    """Per-output-channel int8 weights (qat.py:48-57; export/refiner.py:40-46): s_w = amax / 127 (fp32, clamped at
    1e-12), q_w = clamp(round(w / s_w), -127, 127).  Returns (q_w int8 same shape, s_w [Co] fp32)."""
    w = np.asarray(w, f32)
    amax = np.abs(w).reshape(w.shape[0], -1).max(axis=1)
    s = np.maximum((amax / QMAX).astype(f32), f32(1e-12))
    q = np.clip(np.rint(w / s.reshape((-1,) + (1,) * (w.ndim - 1))), -QMAX, QMAX).astype(np.int8)
    return q, s


def dequant(acc: np.ndarray, s_a, s_w: np.ndarray, b: np.ndarray) -> np.ndarray:
    """y = (float(acc) * s_a) * s_w[n] + b[n] in fp32 (int -> fp32 rounds to nearest even)."""
    return ((acc.astype(f32) * f32(s_a)) * s_w[None, :] + b[None, :]).astype(f32)


_NATIVE = None


def _native():
    """oracle/_build/liboracle.so (oracle/conv.c, built by oracle/build.py) when present, else None."""
    global _NATIVE
    if _NATIVE is None:
        import ctypes as C
        from pathlib import Path
        p = Path(__file__).resolve().parent / "_build" / "liboracle.so"
        _NATIVE = False
        if p.exists():
            try:
                lib = C.CDLL(str(p))
                lib.oracle_conv_acc.restype = C.c_int
                lib.oracle_conv_acc.argtypes = [C.c_void_p, C.c_int64, C.c_void_p, C.c_int64, C.c_void_p, C.c_int,
                                                C.c_int, C.c_void_p]
                _NATIVE = lib
            except OSError:
                _NATIVE = False
    return _NATIVE or None


def conv_acc(q_in: np.ndarray, nmap: np.ndarray, q_w: np.ndarray) -> np.ndarray:
    """int32 accumulators of a submanifold conv (_core.py:399-441 in integer form).  q_in [M, Ci] int8,
    nmap [M, 27] int32, q_w [Co, 3, 3, 3, Ci] int8 -> [M, Co] integers (int32 from the C restatement, oracle/conv.c:
    exact int32 sums on all host threads, used when it is built; int64 from the numpy form below): the same values."""
    lib = _native()
    if lib is not None and q_w.shape[0] % 16 == 0 and q_w.shape[-1] % 2 == 0:
        q = np.ascontiguousarray(q_in, dtype=np.int8)
        nm = np.ascontiguousarray(nmap, dtype=np.int32)
        w = np.ascontiguousarray(q_w, dtype=np.int8).reshape(q_w.shape[0], 27, q_w.shape[-1])
        out = np.empty((nm.shape[0], w.shape[0]), np.int32)
        rc = lib.oracle_conv_acc(q.ctypes.data, q.shape[0], nm.ctypes.data, nm.shape[0], w.ctypes.data, w.shape[2],
                                 w.shape[0], out.ctypes.data)
        if rc != 0:
            raise ValueError("oracle_conv_acc: neighbour index out of range")
        return out
    return conv_acc_numpy(q_in, nmap, q_w)


def conv_acc_numpy(q_in: np.ndarray, nmap: np.ndarray, q_w: np.ndarray) -> np.ndarray:
    """int32 accumulators of a submanifold conv (_core.py:399-441 in integer form: per tap, gather the neighbour rows,
    multiply by the tap's weight, add into the output rows).  q_in [M, Ci] int8, nmap [M, 27] int32,
    q_w [Co, 3, 3, 3, Ci] int8 -> [M, Co] int64.

    Each tap's product is an fp32 GEMM, which is exact here: every term is an integer of magnitude <= 127 * 127 and
    every partial sum of one output has magnitude <= Ci * 127^2 <= 2^22 for Ci <= 256, below 2^24, so no rounding
    happens in any summation order; the 27 taps are then summed in int64."""
    M = nmap.shape[0]
    Co, Ci = q_w.shape[0], q_w.shape[-1]
    assert Ci * 127 * 127 < 2 ** 24, "fp32 tap products are exact only for Ci <= 1040"
    w = q_w.reshape(Co, 27, Ci).astype(np.float32)
    acc = np.zeros((M, Co), np.int64)
    for v in range(27):
        idx = nmap[:, v]
        rows = np.nonzero(idx >= 0)[0]
        if rows.size == 0:
            continue
        acc[rows] += (q_in[idx[rows]].astype(np.float32) @ w[:, v, :].T).astype(np.int64)
    return acc


def linear_acc(q_in: np.ndarray, q_w: np.ndarray) -> np.ndarray:
    """int32 accumulators of a dense layer: q_in [M, K] int8, q_w [N, K] int8 -> [M, N] int64."""
    return (q_in.astype(np.float64) @ q_w.astype(np.float64).T).astype(np.int64)


def layer_norm(x: np.ndarray, w: np.ndarray, b: np.ndarray, eps: float = 1e-6) -> np.ndarray:
    """nn.LayerNorm(C, eps=1e-6) (flex_sparse_blocks.py:58): biased variance (statistics taken in float64 here),
    then y = (x * rstd + (-rstd * mean)) * gamma + beta in fp32, the form of aten's CPU layer-norm kernel."""
    xd = x.astype(np.float64)
    mean = xd.mean(axis=1, keepdims=True)
    var = ((xd - mean) ** 2).mean(axis=1, keepdims=True)
    rstd = (1.0 / np.sqrt(var + eps)).astype(f32)
    shift = (-rstd * mean.astype(f32)).astype(f32)
    return ((x * rstd + shift) * w[None, :] + b[None, :]).astype(f32)


def silu(x: np.ndarray) -> np.ndarray:
    """x / (1 + exp(-x)) in fp32."""
    x = np.asarray(x, f32)
    with np.errstate(over="ignore"):
        return (x / (f32(1.0) + np.exp(-x))).astype(f32)


def linear_f32(x: np.ndarray, w: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Unquantised nn.Linear (input/prompt/out proj), products summed in float64 and rounded to fp32."""
    return (x.astype(np.float64) @ w.astype(np.float64).T + b.astype(np.float64)).astype(f32)


class QuantRefiner:
    """The int8 refiner forward.  `weights`: the reference state-dict names -> fp32 arrays; `clips`: quantised layer
    name (e.g. 'down_stages.0.0.conv1') -> activation clip.  `levels`/`pools` come from structure.build_levels."""

    def __init__(self, weights: dict, clips: dict, model_channels, downsample_factors):
        self.w = {k: np.asarray(v, f32) for k, v in weights.items()}
        self.clips = {k: float(v) for k, v in clips.items()}
        self.ch = list(model_channels)
        self.factors = list(downsample_factors)
        self.qw = {}
        for name in self.clips:
            self.qw[name] = quant_weight(self.w[name + ".weight"])

    # -- quantised layers --------------------------------------------------------------------------------------- #
    def qconv(self, name, x, nmap, trace):
        q, sa = quant_act(x, self.clips[name])
        qw, sw = self.qw[name]
        acc = conv_acc(q, nmap, qw)
        y = dequant(acc, sa, sw, self.w[name + ".bias"])
        if trace is not None:
            trace[name] = dict(q=q, acc=acc, y=y)
        return y

    def qlinear(self, name, x, trace):
        q, sa = quant_act(x, self.clips[name])
        qw, sw = self.qw[name]
        acc = linear_acc(q, qw)
        y = dequant(acc, sa, sw, self.w[name + ".bias"])
        if trace is not None:
            trace[name] = dict(q=q, acc=acc, y=y)
        return y

    def resblock(self, prefix, x, nmap, trace):
        """SparseResBlock3d.forward, flex_sparse_blocks.py:70-75."""
        h = silu(layer_norm(x, self.w[prefix + ".norm1.weight"], self.w[prefix + ".norm1.bias"]))
        h = silu(self.qconv(prefix + ".conv1", h, nmap, trace))
        h = self.qconv(prefix + ".conv2", h, nmap, trace)
        return (h + x).astype(f32)

    # -- forward ------------------------------------------------------------------------------------------------ #
    def forward(self, feats, prompt_feats, levels, pools, encoder_feature, uv_bias=None, trace=None):
        """Sparse3DUNet.forward, sparse_unet.py:176-258, with the int8 layers above.  Returns out [M0, 1] fp32."""
        L = len(self.ch)
        w = self.w
        x = linear_f32(feats, w["input_proj.weight"], w["input_proj.bias"])
        if prompt_feats is not None:
            x = (x + linear_f32(prompt_feats, w["prompt_proj.weight"], w["prompt_proj.bias"])).astype(f32)
        skips = []
        for k in range(L):
            x = self.resblock(f"down_stages.{k}.0", x, levels[k]["nmap"], trace)
            if k < L - 1:
                skips.append(x)
                p = pools[k]
                x = pool_mean(x, p["seg_indices"], p["seg_offsets"])
                x = self.qlinear(f"downsample_blocks.{k}.linear", x, trace)
        c = levels[L - 1]["coords"].astype(np.int64)
        enc = np.asarray(encoder_feature, f32)[c[:, 0], :, c[:, 1], c[:, 2]]
        enc = self.qlinear("encoder_fuse", enc, trace)
        if uv_bias is not None:
            enc = (enc + np.asarray(uv_bias, f32)[c[:, 0], :, c[:, 1], c[:, 2]]).astype(f32)
        h = self.qlinear("fuse_proj.0", np.concatenate([x, enc], axis=1), trace)
        x = self.qlinear("fuse_proj.2", silu(h), trace)
        x = self.resblock("bottleneck_stage.0", x, levels[L - 1]["nmap"], trace)
        for i in range(L - 1):
            t = L - 2 - i
            xc = self.qlinear(f"upsample_blocks.{i}.linear", x, trace)
            x = (xc[pools[t]["parent"]] + skips[t]).astype(f32)
            x = self.resblock(f"up_stages.{i}.0", x, levels[t]["nmap"], trace)
        return linear_f32(x, w["out_proj.weight"], w["out_proj.bias"])


def pool_mean(x: np.ndarray, seg_indices: np.ndarray, seg_offsets: np.ndarray) -> np.ndarray:
    """sparse_pool reduce='mean', _core.py:444-481: children summed in fp32 in ascending input order (index_add_),
    divided by the child count."""
    Mo = seg_offsets.shape[0] - 1
    out = np.zeros((Mo, x.shape[1]), f32)
    cnt = np.diff(seg_offsets)
    # Child j of every parent, in ascending input order, added in rounds (each round is one fp32 add per parent).
    for j in range(int(cnt.max()) if Mo else 0):
        has = cnt > j
        par = np.nonzero(has)[0]
        out[par] = (out[par] + x[seg_indices[seg_offsets[par] + j]]).astype(f32)
    return (out / np.maximum(cnt, 1).astype(f32)[:, None]).astype(f32)


def lidar_uncertainty(H, W, lidar_depth, lidar_conf):
    """MoGeModel._lidar_uncertainty (v3.py:385-393): u = 1 - c (1 - clamp((d - 3) / 2, 0, 1)) on the nearest-resized
    sensor, 1 where it has no value.  [B, H, W] fp32."""
    from .fit import nearest_resize
    d = nearest_resize(np.asarray(lidar_depth, f32), H, W)[:, 0]
    c = np.clip((nearest_resize(np.asarray(lidar_conf, f32), H, W)[:, 0] / f32(2.0)).astype(f32), f32(0), f32(1))
    with np.errstate(invalid="ignore"):
        valid = np.isfinite(d) & (d > 0)
        rng = np.clip(((d - f32(3.0)) / f32(2.0)).astype(f32), f32(0), f32(1))
    u = (f32(1.0) - (c * (f32(1.0) - rng).astype(f32)).astype(f32)).astype(f32)
    return np.where(valid, u, f32(1.0)).astype(f32)


def refiner_gates(cur_logz, new_logz, lidar_depth, lidar_conf, output_gate_floor=None, anchor_beta=0.0):
    """The optional refiner-side gates of the refine loop (v3.py:565-573): the output gate scales the update by
    floor + (1 - floor) u; the elastic anchor relaxes toward the re-aligned LiDAR, logz += beta gate (log_d_aff -
    logz) with a hard gate (a fresh fit on the gated logz).  fp32 in the reference's order."""
    from .fit import lidar_in_affine_frame
    cur = np.asarray(cur_logz, f32)
    new = np.asarray(new_logz, f32)
    B, H, W = new.shape
    if output_gate_floor is not None:
        u = lidar_uncertainty(H, W, lidar_depth, lidar_conf)
        fl = float(output_gate_floor)
        g = (f32(fl) + (f32(1.0 - fl) * u).astype(f32)).astype(f32)
        new = (cur + (g * (new - cur).astype(f32)).astype(f32)).astype(f32)
    if anchor_beta > 0:
        log_d_aff, gate, _, _ = lidar_in_affine_frame(new, lidar_depth, lidar_conf, soft_gate=False)
        bg = (f32(anchor_beta) * gate).astype(f32)
        new = (new + (bg * (log_d_aff - new).astype(f32)).astype(f32)).astype(f32)
    return new


def refine_step(model, point_coord, lidar_depth, lidar_conf, encoder_feature, uv_bias, trace=None, res=256.0,
                output_gate_floor=None, anchor_beta=0.0):
    """One step of the refine loop (v3.py:547-576 with the soft-gated LiDAR residual): fit -> prompt feats ->
    voxelise -> U-Net -> logz += delta (-> the optional output gate and elastic anchor).  Returns (new point_coord,
    info)."""
    from . import fit as fitmod
    pc = np.asarray(point_coord, f32)
    B, H, W, _ = pc.shape
    logz = pc[..., 2]
    pf, s, t = fitmod.prompt_feats(logz, lidar_depth, lidar_conf)
    feats, coords, shape, _ = structure.voxelize(pc, res)
    levels, pools = structure.build_levels(coords, shape, model.factors)
    out = model.forward(feats, pf, levels, pools, encoder_feature, uv_bias, trace)
    new_logz = (logz + out[:, 0].reshape(B, H, W)).astype(f32)
    if output_gate_floor is not None or anchor_beta > 0:
        new_logz = refiner_gates(logz, new_logz, lidar_depth, lidar_conf, output_gate_floor, anchor_beta)
    new_pc = pc.copy()
    new_pc[..., 2] = new_logz
    return new_pc, dict(s=s, t=t, prompt_feats=pf, levels=levels, pools=pools, delta=out[:, 0], shape=shape)
