"""Generate the golden fixtures under tests/golden/ by running the REFERENCE's own pure-PyTorch path.

Usage (in a container where the PromptMoGe sources are present; they are read, never modified):

    python tests/golden/make_golden.py --reference /path/to/PromptMoGe [--only NAME ...]

For each configuration it builds the seeded synthetic scene and random-init weights of promptmoge_b200.synth, loads
the weights into the reference's ``Sparse3DUNet`` (moge/model/modules/sparse_unet.py), turns on the reference QAT
(moge/model/modules/qat.py enable_refiner_qat; one eval forward = the observer pass that sets the activation clips),
and runs the reference refine loop (moge/model/v3.py:547-576: ``_lidar_in_affine_frame`` with the soft gate ->
``_refine_logz`` -> ``_voxelize`` -> U-Net on the bundled FlexGEMM fallback).  Recorded:

* structure per level: coords, nmap (the NeighborCache the convs built), pool parent / seg_indices / seg_offsets;
* per quantised layer: its int8 input q (the reference rule round(x / (clip/127)) applied to the layer's real
  input), the exact int32 accumulators computed by the reference's own operators on the integers in float64
  (submanifold_conv for convs, the verify_int8.py:86-103 float64 GEMM for linears) as a SHA-256 plus sampled rows,
  and the reference layer's float output on the sampled rows; for every conv, also the SHA-256 of the exact int32
  accumulators of the same layer on a seeded int8 input (synth.seeded_conv_input) and the reference's neighbour cache;
* per step: the fit (s, t), prompt features, the refined logz;
* the final 'lidar_ls' fit (v3.py:768-777) on the refined depth and the gauge polynomial (v3.py:151-183).

Full-size configurations store SHA-256 digests of the structure arrays and accumulators, sampled outputs and the
frame's refinement (delta log-depth) in float16, so the committed files stay small.  The synthetic model's activation clips for the benchmark configurations are also written to
promptmoge_b200/synth_clips.json.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import sys
import types
from pathlib import Path
from types import SimpleNamespace

import numpy as np

REPO = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(REPO))

from promptmoge_b200 import synth  # noqa: E402

GOLDEN = Path(__file__).resolve().parent

CONFIGS = {
    # name: (model, H, W, encoder_downsample, K, seed, full_dump)
    "B_small": ("B", 32, 48, 8, 2, 11, True),
    "A_small": ("A", 48, 64, 16, 1, 12, True),
    "B_full": ("B", 240, 320, 8, 1, 0, False),
    "A_full": ("A", 480, 640, 16, 1, 0, False),
}
CONV_CONFIGS = {
    # name: (N, C, seed) -- isolated submanifold conv on surface shells in a 2^21 grid
    "conv_100k_c16": (100_000, 16, 3),
    "conv_20k_c32": (20_000, 32, 4),
}
SAMPLE_ROWS = 48


def sha(a: np.ndarray) -> str:
    a = np.ascontiguousarray(a)
    return hashlib.sha256(a.dtype.str.encode() + str(a.shape).encode() + a.tobytes()).hexdigest()


def import_reference(ref: Path):
    sys.modules.setdefault("utils3d", types.ModuleType("utils3d"))   # only used after refinement (v3.py:758-799)
    sys.path.insert(0, str(ref / "promptmoge" / "_fallback"))
    sys.path.insert(0, str(ref))
    import torch  # noqa: F401
    from moge.model.modules.sparse_unet import Sparse3DUNet
    from moge.model.modules.qat import enable_refiner_qat, ActFakeQuant
    from moge.model.modules.prompt_stem import fit_scale_shift
    from moge.model.v3 import MoGeModel
    import flex_gemm
    assert "torch-reference" in flex_gemm.__version__, "expected the bundled FlexGEMM fallback"
    return SimpleNamespace(Sparse3DUNet=Sparse3DUNet, enable_refiner_qat=enable_refiner_qat,
                           ActFakeQuant=ActFakeQuant, fit_scale_shift=fit_scale_shift, MoGeModel=MoGeModel,
                           flex_gemm=flex_gemm)


def build_reference_refiner(R, model: str, seed: int):
    import torch
    m = synth.MODELS[model]
    unet = R.Sparse3DUNet(in_channels=3, out_channels=1, encoder_channels=synth.ENC_CHANNELS,
                          model_channels=m["model_channels"], encoder_blocks_per_level=1, decoder_blocks_per_level=1,
                          bottleneck_blocks=1, downsample_factors=m["downsample_factors"],
                          encoder_downsample=m["encoder_downsample"], prompt_channels=2)
    w = synth.make_refiner_weights(model, seed)
    missing, unexpected = unet.load_state_dict({k: torch.from_numpy(v) for k, v in w.items()}, strict=True), None
    return unet.eval(), w


def run_config(R, name, model, H, W, ed, K, seed, full_dump):
    import torch
    import torch.nn.functional as F
    torch.manual_seed(1234)
    scene = synth.make_scene(seed, H, W, ed, synth.MODELS[model]["model_channels"][-1])
    unet, weights = build_reference_refiner(R, model, seed)
    # Capture each quantised layer's raw input: register BEFORE the QAT pre-hooks so ours runs first.
    qnames = []
    for n, mod in unet.named_modules():
        if isinstance(mod, (R.flex_gemm.nn.SubmanifoldConv3d, torch.nn.Linear)) and \
                n.split(".")[-1] not in ("input_proj", "prompt_proj", "out_proj"):
            qnames.append(n)
    raw_in, outs, caches = {}, {}, {}
    mods = dict(unet.named_modules())
    hooks = []
    for n in qnames:
        def pre(module, args, n=n):
            raw_in[n] = args[0].detach().clone()
        def post(module, args, out, n=n):
            if isinstance(out, tuple):
                outs[n] = out[0].detach().clone()
                caches[n] = out[1]
            else:
                outs[n] = out.detach().clone()
        hooks.append(mods[n].register_forward_pre_hook(pre))
        hooks.append(mods[n].register_forward_hook(post))
    pool_caches = {}
    for k, blk in enumerate(unet.downsample_blocks):
        def ppost(module, args, out, k=k):
            pool_caches[k] = out[3]
        hooks.append(blk.register_forward_hook(ppost))
    done = R.enable_refiner_qat(unet)
    assert sorted(done) == sorted(qnames), (done, qnames)

    ns = SimpleNamespace(refiner_depth_resolution=256.0, refiner=unet)
    ns._voxelize = lambda pc: R.MoGeModel._voxelize(ns, pc)
    pc = torch.from_numpy(scene.point_coord.copy())
    lidar = torch.from_numpy(scene.lidar_depth)
    conf = torch.from_numpy(scene.lidar_conf)
    enc = torch.from_numpy(scene.encoder_feature.astype(np.float32))
    uvb = torch.from_numpy(scene.uv_bias)

    out = dict(config=np.array(json.dumps(dict(name=name, model=model, H=H, W=W, encoder_downsample=ed, K=K,
                                                   seed=seed, full=full_dump))))
    digests = {}
    clips = None
    rng = np.random.default_rng(99)
    with torch.inference_mode():
        for step in range(K):
            raw_in.clear(); outs.clear(); caches.clear(); pool_caches.clear()
            logz = pc[..., 2]
            log_d_aff, gate, s, t = R.MoGeModel._lidar_in_affine_frame(logz, lidar, conf, soft_gate=True)
            residual = (log_d_aff - logz) * gate
            prompt_feats = torch.stack([residual, gate], dim=-1).reshape(-1, 2)
            refined = R.MoGeModel._refine_logz(ns, pc, enc, prompt_feats=prompt_feats, encoder_bias_map=uvb)
            if clips is None:
                clips = {n: float(getattr(unet, "aq_" + n.replace(".", "_")).clip) for n in qnames}
            P = f"s{step}_"
            out[P + "fit_st"] = np.stack([s.numpy(), t.numpy()], -1).astype(np.float32)
            # structure
            feats, coords, shape, _ = R.MoGeModel._voxelize(ns, pc)
            lv_coords = [coords]
            for k in range(len(pool_caches)):
                lv_coords.append(pool_caches[k].output_coords)
            lv_nmap = {}
            for n, cache in caches.items():
                M = cache.nmap.shape[0]
                lv = [i for i, c in enumerate(lv_coords) if c.shape[0] == M and torch.equal(c, cache.input_coords)]
                lv_nmap[lv[0]] = cache.nmap
            for k, c in enumerate(lv_coords):
                arrs = {f"L{k}_coords": c.numpy().astype(np.int32), f"L{k}_nmap": lv_nmap[k].numpy().astype(np.int32)}
                if k < len(pool_caches):
                    pcache = pool_caches[k]
                    arrs[f"P{k}_parent"] = pcache.parent.numpy().astype(np.int32)
                    arrs[f"P{k}_seg_indices"] = pcache.seg_indices.numpy().astype(np.int32)
                    arrs[f"P{k}_seg_offsets"] = pcache.seg_offsets.numpy().astype(np.int64)
                for kk, a in arrs.items():
                    digests[P + kk] = sha(a)
                    if full_dump:
                        out[P + kk] = a
            out[P + "shape"] = np.array([int(v) for v in shape[:4]], np.int64)
            # per quantised layer (first step only; later steps record structure and outputs)
            for n in (qnames if step == 0 else []):
                aq = getattr(unet, "aq_" + n.replace(".", "_"))
                x = raw_in[n].float()
                sa = (aq.clip / 127.0).float().clamp_min(1e-12)
                q = torch.clamp(torch.round(x / sa), -127, 127)
                wq = mods[n].weight.detach().float()              # the fake-quantised weight (q_w * s_w)
                wmaster = mods[n].parametrizations.weight.original.detach().float()
                dims = tuple(range(1, wmaster.ndim))
                sw = (wmaster.abs().amax(dim=dims, keepdim=True) / 127.0).float().clamp_min(1e-12)
                qw = torch.clamp(torch.round(wmaster / sw), -127, 127)
                assert torch.equal((qw * sw).to(wmaster.dtype), wq), n     # export/refiner.py:45
                if n in caches:
                    cache = caches[n]
                    acc, _ = R.flex_gemm.ops.submanifold_conv(q.double(), cache.input_coords, shape, qw.double(),
                                                              None, neighbor_cache=cache)
                else:
                    acc = q.double() @ qw.double().T
                assert float((acc - acc.round()).abs().max()) == 0.0
                acc = acc.long()
                assert int(acc.abs().max()) < 2 ** 31
                acc32 = acc.numpy().astype(np.int32)
                q8 = q.numpy().astype(np.int8)
                M = q8.shape[0]
                rows = np.sort(rng.choice(M, min(M, SAMPLE_ROWS), replace=False)).astype(np.int64)
                key = P + "Q_" + n
                digests[key + "_q"] = sha(q8)
                digests[key + "_acc"] = sha(acc32)
                out[key + "_rows"] = rows
                out[key + "_acc_rows"] = acc32[rows]
                out[key + "_y_rows"] = outs[n].float().numpy()[rows]
                if full_dump:
                    out[key + "_q"] = q8
                if n in caches:
                    # the same layer on a seeded int8 input (synth.seeded_conv_input, regenerated by the GPU tests):
                    # pins the int32 accumulators at every size, independently of upstream float rounding
                    qs = synth.seeded_conv_input(n, M, q8.shape[1])
                    acc_s, _ = R.flex_gemm.ops.submanifold_conv(torch.from_numpy(qs).double(), cache.input_coords,
                                                                shape, qw.double(), None, neighbor_cache=cache)
                    assert float((acc_s - acc_s.round()).abs().max()) == 0.0
                    acc_s = acc_s.long()
                    assert int(acc_s.abs().max()) < 2 ** 31
                    digests[P + "S_" + n + "_acc"] = sha(acc_s.numpy().astype(np.int32))
            out[P + "prompt_feats_digest_rows"] = prompt_feats.numpy()[:: max(1, prompt_feats.shape[0] // 2048)]
            delta = (refined - logz).numpy()
            if full_dump:
                out[P + "logz_in"] = logz.numpy().astype(np.float32)
                out[P + "prompt_feats"] = prompt_feats.numpy().astype(np.float32)
                out[P + "delta"] = delta.astype(np.float32)
            else:
                out[P + "delta_f16"] = delta.astype(np.float16)       # the whole frame's refinement, half precision
                pix = np.sort(rng.choice(delta.size, 8192, replace=False))
                out[P + "pix"] = pix
                out[P + "delta_pix"] = delta.reshape(-1)[pix].astype(np.float32)
                out[P + "logz_in_pix"] = logz.numpy().reshape(-1)[pix].astype(np.float32)
            out[P + "delta_stats"] = np.array([delta.mean(), np.abs(delta).mean(), delta.std()], np.float64)
            pc = torch.cat([pc[..., :2], refined.unsqueeze(-1)], dim=-1)

        # final metric fit on the refined depth (v3.py:768-777) and the gauge polynomial (v3.py:151-183)
        depth = torch.exp(pc[..., 2])
        d_lr = F.interpolate(depth.unsqueeze(1), lidar.shape[-2:], mode="area").squeeze(1)
        m_lr = (conf.squeeze(1) >= 2) & (lidar.squeeze(1) > 0) & (d_lr > 0)
        s_f, t_f = R.fit_scale_shift(d_lr.flatten(1), lidar.squeeze(1).flatten(1), m_lr.flatten(1))
        depth_m = s_f[:, None, None] * depth + t_f[:, None, None]
        corr = R.MoGeModel.prompt_gauge_poly(depth_m, lidar, conf, degree=2)
        out["final_fit_st"] = np.stack([s_f.numpy(), t_f.numpy()], -1).astype(np.float32)
        out["final_d_lr"] = d_lr.numpy().astype(np.float32) if full_dump else d_lr.numpy()[:, ::8, ::8]
        out["final_logz"] = pc[..., 2].numpy().astype(np.float32) if full_dump else \
            pc[..., 2].numpy().reshape(-1)[out["s0_pix"]]
        out["gauge_corr_rows"] = corr.numpy()[:, ::4, ::4].astype(np.float32)
    for h in hooks:
        h.remove()
    out["digests"] = np.array(json.dumps(digests, sort_keys=True))
    out["clips"] = np.array(json.dumps(clips, sort_keys=True))
    np.savez_compressed(GOLDEN / f"{name}.npz", **out)
    print(f"{name}: {len(digests)} digests, wrote {GOLDEN / (name + '.npz')}")
    return clips


def run_conv_config(R, name, N, C, seed):
    import torch
    coords = synth.make_surface_voxels(N, seed)
    shape = [1, 1 << 21, 1 << 21, 1 << 21]
    ct = torch.from_numpy(coords)
    cache = R.flex_gemm.ops.build_submanifold_cache(ct, shape, (3, 3, 3))
    rng = np.random.default_rng(seed + 100)
    q = rng.integers(-127, 128, (coords.shape[0], C)).astype(np.int8)
    qw = rng.integers(-127, 128, (C, 3, 3, 3, C)).astype(np.int8)
    acc, _ = R.flex_gemm.ops.submanifold_conv(torch.from_numpy(q).double(), ct, torch.Size(shape + [C]),
                                              torch.from_numpy(qw).double(), None, neighbor_cache=cache)
    acc = acc.long().numpy().astype(np.int32)
    nmap = cache.nmap.numpy().astype(np.int32)
    occ = (nmap >= 0).sum(1)
    out = dict(config=np.array(json.dumps(dict(name=name, N=N, C=C, seed=seed))),
               nmap_sha=np.array(sha(nmap)), acc_sha=np.array(sha(acc)),
               nmap_rows=nmap[:2048], acc_rows=acc[:2048], occupancy=np.array([occ.mean(), occ.max()]),
               backend=np.array(cache.build_backend))
    np.savez_compressed(GOLDEN / f"{name}.npz", **out)
    print(f"{name}: M={coords.shape[0]} mean taps {occ.mean():.2f} backend {cache.build_backend}")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--only", nargs="*")
    a = ap.parse_args()
    R = import_reference(Path(a.reference))
    import torch
    torch.set_num_threads(8)
    clip_table = {}
    clips_path = REPO / "promptmoge_b200" / "synth_clips.json"
    if clips_path.exists():
        clip_table = json.loads(clips_path.read_text())
    for name, cfg in CONFIGS.items():
        if a.only and name not in a.only:
            continue
        clips = run_config(R, name, *cfg)
        model, H, W, ed, K, seed, _ = cfg
        clip_table[f"{model}_{H}x{W}_seed{seed}"] = clips
    for name, cfg in CONV_CONFIGS.items():
        if a.only and name not in a.only:
            continue
        run_conv_config(R, name, *cfg)
    clips_path.write_text(json.dumps(clip_table, indent=1, sort_keys=True))


if __name__ == "__main__":
    main()
