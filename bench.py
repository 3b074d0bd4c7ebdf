"""Benchmark of the sparse 3-D refinement step on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: Model A refiner, one refine step (K=1), batch 1, 480x640 synthetic room frame per
GPU (seed = rank), random-init int8 weights with the reference observer's clips.  A "step" = fit -> prompt features
-> voxelise -> 5-level structure (dedup + neighbour maps) -> int8 U-Net -> logz update, replayed as one CUDA graph.
With N > 1 every rank refines its own independent frames (frame-batch sharding, weak scaling) and the per-frame fits
are all-gathered once at the end of the timed region.

One JSON line on rank 0: value = refine steps/s over all ranks (device time, inputs resident), e2e = the same through
the public host API (pinned host -> device copies, encoder conditioning, graph, device -> host of the refined point
map), roofline of the dominant kernel, the CPU oracle baseline, clocks sampled during the timed region.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "refine steps/s (Model A, 480x640, K=1)"
UNIT = "steps/s"


def _dist():
    import torch
    import torch.distributed as dist
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1 and not dist.is_initialized():
        import datetime
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return ws, rank, local


class Clocks:
    """nvidia-smi sampling during the timed region (SM clock, throttle reasons)."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.p = None

    def __enter__(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "100"],
                                      stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.p = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.p is not None:
            self.p.terminate()
            try:
                out, _ = self.p.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.p.kill()
                out, _ = self.p.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in self.lines:
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def int8_peak_tops(torch):
    """Measured int8 tensor throughput of cuBLASLt (torch._int_mm, 8192^3, best of 10) in TOP/s."""
    n = 8192
    a = torch.randint(-127, 127, (n, n), dtype=torch.int8, device="cuda")
    b = torch.randint(-127, 127, (n, n), dtype=torch.int8, device="cuda")
    for _ in range(3):
        torch._int_mm(a, b)
    best = 1e9
    for _ in range(10):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        torch._int_mm(a, b)
        e.record()
        e.synchronize()
        best = min(best, s.elapsed_time(e))
    return 2.0 * n ** 3 / (best * 1e-3) / 1e12


def dominant_conv(torch, eng, reps: int = 20):
    """Time each level's conv1 (the fused SiLU + requantise epilogue) standalone with CUDA events on the current
    stream, inputs = the plan's own level structure and activations; return the level whose convs dominate."""
    from promptmoge_b200 import ops
    L = eng.geo.levels
    _, counts = eng.status(clear=False)
    flush = torch.empty(64 << 20, dtype=torch.float32, device="cuda")
    res = []
    for k in range(L):
        info = eng.level_info(k)
        cap, C_ = info["cap"], info["C"]
        M = counts[k]
        nmap = eng.debug_tensor("nmap", k, (27, cap), torch.int32)
        mask = eng.debug_tensor("tile_mask", k, (cap // 32 + 2,), torch.int32)
        q1 = eng.debug_tensor("q1", k, (cap, C_), torch.int8)
        cnt = torch.tensor([M], dtype=torch.int32, device="cuda")
        w = torch.randint(-127, 127, (27, C_, C_), dtype=torch.int8, device="cuda")
        ws = torch.full((C_,), 1e-3, device="cuda")
        b = torch.zeros(C_, device="cuda")
        nnz = int((nmap[:, :M] >= 0).sum().item())
        tc = bool(eng.tensor_cores) and ops.tc_supported(C_, C_)
        run = lambda: ops.spconv_i8(q1, nmap, mask, w, ws, b, 0.01, ops.EPI_SILU_Q8, 0.02, count=cnt,
                                    tensor_cores=tc)

        def timed(fn):
            fn()
            torch.cuda.synchronize()
            tms = []
            for _ in range(reps):
                flush.zero_()
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s.record()
                fn()
                e.record()
                torch.cuda.synchronize()
                tms.append(s.elapsed_time(e))
            return float(np.median(tms))
        t = timed(run)
        ops_ = 2.0 * nnz * C_ * C_
        byts = M * C_ + M * C_ + 27 * 4 * M + 27 * C_ * C_
        # this level's convs per step: 2 down + 2 up (4 at L<L-1), 2 down + 2 bottleneck at the last level
        res.append(dict(level=k, M=M, C=C_, ms=t, ops=ops_, bytes=byts, per_step=4 * t))
    return res


def run_ours(args, ws, rank, local):
    import torch
    import torch.distributed as dist
    from promptmoge_b200 import synth
    from promptmoge_b200.refine import Refiner, pinned, synthetic_model

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    weights, clips = synthetic_model("A", 0)
    batch = args.batch
    ref = Refiner(weights, clips, "A", batch=batch, device=dev)
    sc = synth.make_scene(1000 * rank, 480, 640, 16, 256, batch=batch)
    h_pc, h_ld, h_lc = pinned(sc.point_coord), pinned(sc.lidar_depth), pinned(sc.lidar_conf)
    h_enc, h_uv = pinned(sc.encoder_feature), pinned(sc.uv_bias)
    # first call sizes the plan: run once, shrink level capacities to the measured counts (+25 %), recapture
    ref.refine(h_pc, h_ld, h_lc, h_enc, h_uv, K=args.K)
    rc, counts = ref.engine.status()
    if rc != 0:
        raise RuntimeError(f"device status {rc}")
    ref.engine.fit_to(counts)
    ref._K = None
    ref.refine(h_pc, h_ld, h_lc, h_enc, h_uv, K=args.K)
    rc, counts = ref.engine.status()
    if rc != 0:
        raise RuntimeError(f"device status {rc} after resize")
    eng = ref.engine
    flush = torch.empty(256 << 18, dtype=torch.float32, device=dev)   # 256 MiB > L2 (126 MB)

    def step():
        eng.replay()

    # ---------------- device-resident throughput ---------------- #
    for _ in range(args.warmup):
        flush.zero_()
        step()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    gather_out = torch.empty((ws, batch, 18), dtype=torch.int32, device=dev) if ws > 1 else None
    if ws > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with Clocks(local) as clk:
        for i in range(args.steps):
            flush.zero_()
            ev[i][0].record()
            out, fit = eng.replay()
            if ws > 1 and i == args.steps - 1:
                dist.all_gather_into_tensor(gather_out, fit.contiguous())
            ev[i][1].record()
        torch.cuda.synchronize()
    if ws > 1:
        dist.barrier()
    step_ms = [s.elapsed_time(e) for s, e in ev]
    total_ms = float(sum(step_ms))
    if ws > 1:
        t = torch.tensor([total_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
    value = ws * batch * args.steps / (total_ms * 1e-3)
    rc, _ = eng.status()
    if rc != 0:
        raise RuntimeError(f"device status {rc} in the timed region")
    if args.ncu:
        # profiling mode (run under ncu): the replays above are what is profiled; numbers are not bench values
        ref.close()
        return {"ncu_mode": True, "ms_per_step_unprofiled_invalid": total_ms / args.steps} if rank == 0 else None

    # ---------------- end to end through the public host API ---------------- #
    for _ in range(2):
        ref.refine(h_pc, h_ld, h_lc, h_enc, h_uv, K=args.K)
    e2e_ms = []
    for _ in range(args.steps):
        flush.zero_()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        ref.refine(h_pc, h_ld, h_lc, h_enc, h_uv, K=args.K, sync=False)
        e.record()
        e.synchronize()
        e2e_ms.append(s.elapsed_time(e))
    e2e_total = float(sum(e2e_ms))
    if ws > 1:
        t = torch.tensor([e2e_total], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_total = float(t.item())
    e2e_value = ws * batch * args.steps / (e2e_total * 1e-3)

    line = None
    if rank == 0:
        launches = eng.launches_per_step() * args.K
        # roofline of the dominant kernel
        convs = dominant_conv(torch, eng)
        dom = max(convs, key=lambda r: r["per_step"])
        peak = int8_peak_tops(torch)
        achieved = dom["ops"] / (dom["ms"] * 1e-3) / 1e12
        traffic = None
        tfile = ROOT / "profiles" / "traffic.json"
        if tfile.exists():
            tj = json.loads(tfile.read_text())
            traffic = tj.get(f"conv_L{dom['level']}")
        roof = {"bound": "tensor", "achieved": round(achieved, 3), "peak": round(peak, 1), "unit": "TOP/s",
                "frac": round(achieved / peak, 5), "traffic": traffic,
                "kernel": f"int8 submanifold conv level {dom['level']} (M={dom['M']}, C={dom['C']})",
                "peak_source": "measured in this run: cuBLASLt int8 GEMM (torch._int_mm 8192^3, best of 10); "
                               "MEASURED_PEAKS.json has no int8 figure",
                "per_level_ms": {f"L{r['level']}": round(r["ms"], 4) for r in convs}}
        cpu = None
        if ws == 1 and not args.no_cpu_baseline:
            cpu = cpu_baseline(batch=1, steps=1)
        line = {
            "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(total_ms / args.steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": "C2: Model A refiner (widths 32-64-128-256-256), 1 refine step, 480x640, "
                                   f"batch {batch} per GPU, synthetic room (seed = 1000*rank)",
                       "model": "PromptMoGe Model A sparse refiner (random-init int8 QAT weights)",
                       "K": args.K, "global_batch": ws * batch, "parallelism": f"frame-batch x{ws}",
                       "levels_voxels": counts, "l2": "flushed by a 256 MiB write before every timed step",
                       "timing": "CUDA events around each graph replay, max over ranks"},
            "e2e": {"value": round(e2e_value, 3), "unit": UNIT,
                    "h2d_bytes_per_step": ref.input_bytes(), "d2h_bytes_per_step": ref.output_bytes()},
            "gpu_launches": launches * args.steps,
            "roofline": roof,
            "cpu_baseline": cpu,
            "clocks": clk.summary(),
        }
    ref.close()
    return line


def cpu_baseline(batch=1, steps=1):
    """The numpy oracle (a restatement of the reference's CPU path) on the host cores: one full 480x640 step."""
    import json as _j
    from oracle import refiner as oref
    from promptmoge_b200 import synth
    from promptmoge_b200.refine import synthetic_model
    weights, clips = synthetic_model("A", 0)
    ch = synth.MODELS["A"]["model_channels"]
    qr = oref.QuantRefiner(weights, clips, ch, [2] * (len(ch) - 1))
    sc = synth.make_scene(0, 480, 640, 16, 256, batch=batch)
    enc = sc.encoder_feature.astype(np.float32)
    t0 = time.perf_counter()
    for _ in range(steps):
        oref.refine_step(qr, sc.point_coord, sc.lidar_depth, sc.lidar_conf, enc, sc.uv_bias)
    dt = (time.perf_counter() - t0) / steps
    del _j
    return {"value": round(batch / dt, 5), "unit": UNIT, "cores": os.cpu_count(), "kind": "port",
            "sample": f"{steps} full refine step(s) of one 480x640 Model A frame with the numpy oracle "
                      f"(float64-exact int8 GEMMs via BLAS on all host threads): {dt:.2f} s/step"}


def profile_conv(args):
    """Profiling driver (run under ncu): the real 480x640 level structure of the benchmark frame, random int8
    activations and weights, `--steps` launches of that level's conv (fused SiLU + requantise epilogue).  Only the
    profiled kernels are int8 GEMM launches, so `ncu -k regex:k_gemm -s 1 -c 2` captures two warm launches."""
    import torch
    from promptmoge_b200 import ops, synth
    from promptmoge_b200.levels import build_levels
    torch.cuda.set_device(0)
    sc = synth.make_scene(0, 480, 640, 16, 256)
    lv, _ = build_levels(torch.from_numpy(sc.point_coord).cuda(), 5, with_coords=False)
    k = args.profile_conv
    C_ = synth.MODELS["A"]["model_channels"][k]
    l = lv[k]
    M = l["count"]
    g = torch.Generator(device="cuda").manual_seed(0)
    q = torch.randint(-127, 127, (M, C_), dtype=torch.int8, device="cuda", generator=g)
    w = torch.randint(-127, 127, (27, C_, C_), dtype=torch.int8, device="cuda", generator=g)
    tc_path = ops.tc_supported(C_, C_) and not args.simt
    ws_ = torch.full((C_,), 1e-3, device="cuda")
    b = torch.zeros(C_, device="cuda")
    for _ in range(max(1, args.steps)):
        ops.spconv_i8(q, l["nmap_tm"], l["mask"], w, ws_, b, 0.01, ops.EPI_SILU_Q8, 0.02, rows=M,
                      tensor_cores=tc_path)
    torch.cuda.synchronize()
    nnz = int((l["nmap_tm"][:, :M] >= 0).sum().item())
    return {"profile_conv": k, "M": M, "C": C_, "occupied_taps": nnz, "path": "tcgen05" if tc_path else "simt"}


def run_reference(args, ws, rank):
    """Reference arm: the reference's CPU algorithm (the oracle port) on the host cores, rank 0 only."""
    if rank != 0:
        return None
    steps = max(1, min(args.steps, 2))
    warm = min(args.warmup, 1)
    from oracle import refiner as oref
    from promptmoge_b200 import synth
    from promptmoge_b200.refine import synthetic_model
    weights, clips = synthetic_model("A", 0)
    ch = synth.MODELS["A"]["model_channels"]
    qr = oref.QuantRefiner(weights, clips, ch, [2] * (len(ch) - 1))
    sc = synth.make_scene(0, 480, 640, 16, 256, batch=1)
    enc = sc.encoder_feature.astype(np.float32)
    for _ in range(warm):
        oref.refine_step(qr, sc.point_coord, sc.lidar_depth, sc.lidar_conf, enc, sc.uv_bias)
    t0 = time.perf_counter()
    for _ in range(steps):
        oref.refine_step(qr, sc.point_coord, sc.lidar_depth, sc.lidar_conf, enc, sc.uv_bias)
    dt = (time.perf_counter() - t0) / steps
    v = round(1.0 / dt, 5)
    sample = f"{steps} timed + {warm} warm-up full 480x640 refine steps (numpy oracle port, all host threads)"
    return {"impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": ws, "steps": steps,
            "warmup": warm, "ms_per_step": round(dt * 1e3, 1), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": "C2: Model A refiner, 1 refine step, 480x640, batch 1 (synthetic room, seed 0)",
                       "K": 1},
            "cpu_baseline": {"value": v, "unit": UNIT, "cores": os.cpu_count(), "kind": "port", "sample": sample},
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--K", type=int, default=1, help="refine steps per graph (the workload's K)")
    ap.add_argument("--batch", type=int, default=1, help="frames per GPU per step")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--ncu", action="store_true", help="profiling mode: warm-up + timed replays only, no extras")
    ap.add_argument("--profile-conv", type=int, default=None, metavar="LEVEL",
                    help="profiling driver: launch one level's conv --steps times on the benchmark frame's structure")
    ap.add_argument("--simt", action="store_true", help="with --profile-conv: the SIMT kernel instead of tcgen05")
    args = ap.parse_args()
    if args.profile_conv is not None:
        print(json.dumps(profile_conv(args)), flush=True)
        return
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    if args.impl == "reference":
        ws = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        line = run_reference(args, ws, rank)
    else:
        ws, rank, local = _dist()
        line = run_ours(args, ws, rank, local)
        if ws > 1:
            import torch.distributed as dist
            dist.barrier()
            dist.destroy_process_group()
    if line is not None:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
