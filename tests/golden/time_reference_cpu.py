"""Time the reference's own CPU path of one refine step beside this repository's CPU port, on one host.

    python tests/golden/time_reference_cpu.py /path/to/PromptMoGe [--steps 5]

The reference is Python and is not importable where the GPU benchmark runs, so its CPU time cannot be taken in the
same run as the GPU number; this script measures, on the host it runs on, the reference's refine step of Model A at
480 x 640 (moge/model/v3.py:547-559: ``_lidar_in_affine_frame`` with the soft gate, the prompt features,
``_refine_logz`` = ``_voxelize`` + ``Sparse3DUNet.forward`` (moge/model/modules/sparse_unet.py:176-258) under
``enable_refiner_qat`` on the bundled FlexGEMM fallback) plus the final metric fit (v3.py:768-777), fp32,
``torch.inference_mode()``, all host threads, warm, median of ``--steps``; and the numpy port (oracle.refiner.refine_step
+ oracle.fit.final_fit) on the same synthetic frame.  The result goes to tests/golden/reference_cpu_timing.json,
which bench.py reports beside its own CPU baseline (the port) as the measured port / reference time ratio.
"""
from __future__ import annotations

import argparse
import json
import os
import platform
import sys
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(HERE))

from promptmoge_b200 import synth  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("reference")
    ap.add_argument("--steps", type=int, default=5)
    a = ap.parse_args()
    import make_golden
    R = make_golden.import_reference(Path(a.reference))
    import torch
    import torch.nn.functional as F
    threads = os.cpu_count()
    torch.set_num_threads(threads)
    model, seed = "A", 0
    m = synth.MODELS[model]
    H, W = m["H"], m["W"]
    scene = synth.make_scene(seed, H, W, m["encoder_downsample"], m["model_channels"][-1])
    unet, weights = make_golden.build_reference_refiner(R, model, seed)
    R.enable_refiner_qat(unet)
    from types import SimpleNamespace
    ns = SimpleNamespace(refiner_depth_resolution=256.0, refiner=unet)
    ns._voxelize = lambda pc: R.MoGeModel._voxelize(ns, pc)
    pc = torch.from_numpy(scene.point_coord.copy())
    lidar = torch.from_numpy(scene.lidar_depth)
    conf = torch.from_numpy(scene.lidar_conf)
    enc = torch.from_numpy(scene.encoder_feature.astype(np.float32))
    uvb = torch.from_numpy(scene.uv_bias)

    def ref_step():
        logz = pc[..., 2]
        log_d_aff, gate, s, t = R.MoGeModel._lidar_in_affine_frame(logz, lidar, conf, soft_gate=True)
        residual = (log_d_aff - logz) * gate
        prompt_feats = torch.stack([residual, gate], dim=-1).reshape(-1, 2)
        refined = R.MoGeModel._refine_logz(ns, pc, enc, prompt_feats=prompt_feats, encoder_bias_map=uvb)
        depth = torch.exp(refined)
        d_lr = F.interpolate(depth.unsqueeze(1), lidar.shape[-2:], mode="area").squeeze(1)
        m_lr = (conf.squeeze(1) >= 2) & (lidar.squeeze(1) > 0) & (d_lr > 0)
        return R.fit_scale_shift(d_lr.flatten(1), lidar.squeeze(1).flatten(1), m_lr.flatten(1))

    with torch.inference_mode():
        ref_step()                      # the QAT observer pass (first eval forward), then warm steps
        ref_step()
        ref_t = []
        for _ in range(a.steps):
            t0 = time.perf_counter()
            ref_step()
            ref_t.append(time.perf_counter() - t0)

    from oracle import fit as ofit
    from oracle import refiner as oref
    from promptmoge_b200.refine import synthetic_model
    w2, clips = synthetic_model(model, seed)
    qr = oref.QuantRefiner(w2, clips, m["model_channels"], [2] * (len(m["model_channels"]) - 1))
    encf = scene.encoder_feature.astype(np.float32)

    def port_step():
        new_pc, _ = oref.refine_step(qr, scene.point_coord, scene.lidar_depth, scene.lidar_conf, encf, scene.uv_bias)
        ofit.final_fit(np.exp(new_pc[..., 2]).astype(np.float32), scene.lidar_depth, scene.lidar_conf)

    port_step()
    port_t = []
    for _ in range(max(2, a.steps // 2)):
        t0 = time.perf_counter()
        port_step()
        port_t.append(time.perf_counter() - t0)
    res = {
        "host": {"threads": threads, "machine": platform.machine(), "processor": platform.processor() or None,
                 "torch": torch.__version__, "numpy": np.__version__},
        "workload": "one refine step of Model A at 480x640 (seed 0 synthetic frame) + the final metric fit",
        "reference_s_per_step": round(float(np.median(ref_t)), 4),
        "reference_steps": [round(x, 4) for x in ref_t],
        "reference_path": "moge v3 refine-loop body on the bundled FlexGEMM fallback, enable_refiner_qat, fp32, "
                          "torch.inference_mode, torch.set_num_threads(os.cpu_count())",
        "port_s_per_step": round(float(np.median(port_t)), 4),
        "port_steps": [round(x, 4) for x in port_t],
        "port_path": "oracle.refiner.refine_step + oracle.fit.final_fit (this repository's CPU restatement: int8 convs in C with OpenMP, oracle/conv.c; the rest numpy)",
    }
    res["port_over_reference"] = round(res["port_s_per_step"] / res["reference_s_per_step"], 3)
    (HERE / "reference_cpu_timing.json").write_text(json.dumps(res, indent=1) + "\n")
    print(json.dumps(res, indent=1))


if __name__ == "__main__":
    main()
