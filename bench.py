"""Benchmark of the sparse 3-D refinement step on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (benchmark configuration 2): Model A refiner, one refine step (K=1), batch 1, 480x640 synthetic room frame per
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
METRIC_B = "refine steps/s (Model B, 240x320, K=1)"
# The only published numbers for this path (int8 Metal, iPad Pro 11" M5, warm, K = 1)
PUBLISHED_MS = {"A": 27.3, "B": 10.4}
PUBLISHED_STEPS_S = {k: 1000.0 / v for k, v in PUBLISHED_MS.items()}
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
        if k == 0 and bool(eng.tensor_cores) and ops.grid0_supported(C_, C_):
            # level 0 runs the neighbour-map-free frame-grid kernel in the plan
            g = eng.geo
            lanes = eng.debug_tensor("lanes0", 0, ((g.batch * g.height * g.width + 127) // 128, 27, 4), torch.int32)
            run = lambda: ops.spconv_i8_grid0(q1, lanes, g.batch, g.height, g.width, w, ws, b, 0.01,
                                              ops.EPI_SILU_Q8, 0.02)
        else:
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
        if k == 0 and bool(eng.tensor_cores) and ops.grid0_supported(C_, C_):
            byts = M * C_ + M * C_ + 27 * M // 8 + 27 * C_ * C_      # tap masks (3.4 B/row) instead of the map
        else:
            byts = M * C_ + M * C_ + 27 * 4 * M + 27 * C_ * C_
        # this level's convs per step: 2 down + 2 up (4 at L<L-1), 2 down + 2 bottleneck at the last level
        res.append(dict(level=k, M=M, C=C_, ms=t, ops=ops_, bytes=byts, per_step=4 * t))
    return res


def run_ours(args, ws, rank, local):
    import torch
    import torch.distributed as dist
    if ws > 1:
        # one process per GPU: each takes its share of the host cores for its host-side work (copies, Python)
        torch.set_num_threads(max(1, (os.cpu_count() or 1) // ws))
    from promptmoge_b200 import synth
    from promptmoge_b200.refine import Refiner, pinned, synthetic_model

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    mdl = synth.MODELS[args.model]
    weights, clips = synthetic_model(args.model, 0)
    batch = args.batch
    ref = Refiner(weights, clips, args.model, batch=batch, device=dev, max_split=args.max_split, pdl=not args.no_pdl)
    sc = synth.make_scene(1000 * rank, mdl["H"], mdl["W"], mdl["encoder_downsample"], mdl["model_channels"][-1],
                          batch=batch)
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
        # roofline of the dominant kernel: the conv level with the largest per-step time.  Convs with C <= 64 are
        # bandwidth-bound (minimum traffic M*Ci + M*Co + 27*4*M + 27*Ci*Co bytes), wider ones tensor-bound (2 * occupied
        # taps * Ci * Co ops); the int8 peak is measured in this run (MEASURED_PEAKS.json holds bf16 only).
        convs = dominant_conv(torch, eng)
        dom = max(convs, key=lambda r: r["per_step"])
        tops = dom["ops"] / (dom["ms"] * 1e-3) / 1e12
        peak_i8 = int8_peak_tops(torch)
        traffic = None
        prof = ROOT / "profiles" / f"conv_i8_L{dom['level']}_A480x640_ncu.md"
        if prof.exists():
            for ln in prof.read_text().splitlines():
                if ln.startswith("dram_bytes_per_launch:"):
                    traffic = int(ln.split(":")[1])
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
        hbm = float(peaks.get("hbm_gbs", 6650.0))
        if dom["C"] <= 64:
            gbs = dom["bytes"] / (dom["ms"] * 1e-3) / 1e9
            roof = {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm, "unit": "GB/s", "frac": round(gbs / hbm, 5),
                    "peak_source": "MEASURED_PEAKS.json hbm_gbs (measured)" if peaks else "fallback 6650 GB/s"}
        else:
            roof = {"bound": "tensor", "achieved": round(tops, 3), "peak": round(peak_i8, 1), "unit": "TOP/s",
                    "frac": round(tops / peak_i8, 5),
                    "peak_source": "measured in this run: cuBLASLt int8 GEMM (torch._int_mm 8192^3, best of 10)"}
        roof.update({"traffic": traffic, "algorithmic_bytes": dom["bytes"],
                     "kernel": f"int8 submanifold conv level {dom['level']} (M={dom['M']}, C={dom['C']}), "
                               + ("k_conv_grid0" if dom["level"] == 0 and eng.tensor_cores else "k_gemm_tc"),
                     "int8_tops": round(tops, 3), "int8_peak_tops": round(peak_i8, 1),
                     "traffic_source": f"profiles/{prof.name} (ncu dram bytes read + written, one launch)",
                     "per_level_ms": {f"L{r['level']}": round(r["ms"], 4) for r in convs}})
        cpu = None
        if ws == 1 and not args.no_cpu_baseline and args.model == "A":
            cpu = cpu_baseline(batch=1, steps=1)
        prep = prompt_prep(torch, sc, dev, cpu=ws == 1 and not args.no_cpu_baseline)
        post_t = post_output(torch, out, sc, dev, cpu=ws == 1 and not args.no_cpu_baseline)
        line = {
            "metric": METRIC if args.model == "A" else METRIC_B, "value": round(value, 3), "unit": UNIT, "n_gpus": ws,
            "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(total_ms / args.steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": round(value / PUBLISHED_STEPS_S[args.model], 3),
            "vs_baseline_basis": f"the reference's published int8 Metal time for one refine step of Model "
                                 f"{args.model} on an iPad Pro M5 ({PUBLISHED_MS[args.model]} ms, docs/index.html:453)",
            "dtype": "int8", "data": "synthetic",
            "reference_arm": "bench.py --impl reference times one frame's step on the host cores of one machine "
                             "(rank 0 only at any N), so against this line's N-GPU aggregate its ratio grows with N",
            "config": {"workload": (f"C2: Model A refiner (widths 32-64-128-256-256), 1 refine step, 480x640, "
                                    if args.model == "A" else
                                    "C1: Model B refiner (widths 32-64-128-256), 1 refine step, 240x320, ")
                                   + f"batch {batch} per GPU, synthetic room (seed = 1000*rank)",
                       "model": f"PromptMoGe Model {args.model} sparse refiner (random-init int8 QAT weights)",
                       "K": args.K, "global_batch": ws * batch, "parallelism": f"frame-batch x{ws}",
                       "levels_voxels": counts, "l2": "flushed by a 256 MiB write before every timed step",
                       "timing": "CUDA events around each graph replay, max over ranks"},
            "e2e": {"value": round(e2e_value, 3), "unit": UNIT,
                    "h2d_bytes_per_step": ref.input_bytes(), "d2h_bytes_per_step": ref.output_bytes()},
            "gpu_launches": launches * args.steps,
            "roofline": roof,
            "cpu_baseline": cpu,
            "clocks": clk.summary(),
            "prompt_prep": prep,
            "post_output": post_t,
        }
    ref.close()
    if args.c4_frames > 0 and args.model == "A":
        c4 = c4_batched(torch, args, ws, rank, dev, weights, clips)
        if line is not None:
            line["c4"] = c4
    if args.c5_poses > 0 and args.model == "A":
        # config 5 sub-record: the fused scene over the same ranks (strong scaling), its own steps and warm-up
        import copy
        a5 = copy.copy(args)
        a5.fused_poses, a5.steps, a5.warmup = args.c5_poses, args.c5_steps, 3
        c5 = fused_scene(a5, ws, rank, local)
        if line is not None:
            line["c5"] = c5
    return line


def c4_batched(torch, args, ws, rank, dev, weights, clips):
    """Benchmark configuration 4: args.c4_frames independent 480x640 Model A frames at K = args.c4_K, frame-batch
    sharded over the ranks (promptmoge_b200.dist.ShardedRefiner: contiguous frame ranges, args.c4_batch frames per
    graph replay, host inputs copied in and refined point maps copied out per batch, one all-gather of every frame's
    fit state at the end).  Frame f uses synthetic room f mod 8 (eight distinct seeded scenes, pinned once).  Timed
    on the device with CUDA events around the whole sharded run, max over ranks; frames/s of the whole job."""
    import torch.distributed as dist
    from promptmoge_b200 import synth
    from promptmoge_b200.dist import ShardedRefiner, frame_range
    from promptmoge_b200.refine import Refiner, pinned
    B, K, n = args.c4_batch, args.c4_K, args.c4_frames
    mdl = synth.MODELS["A"]
    scenes = [synth.make_scene(500 + i, mdl["H"], mdl["W"], mdl["encoder_downsample"], mdl["model_channels"][-1])
              for i in range(8)]
    # the batches the run can meet: B consecutive frames starting anywhere modulo 8
    batch_cache = {}

    def batch_frames(ids):
        key = tuple(i % 8 for i in ids)
        if key not in batch_cache:
            batch_cache[key] = tuple(
                pinned(np.concatenate([getattr(scenes[i], f) for i in key]))
                for f in ("point_coord", "lidar_depth", "lidar_conf", "encoder_feature", "uv_bias"))
        return batch_cache[key]

    ref = Refiner(weights, clips, "A", batch=B, device=dev, max_split=args.max_split, pdl=not args.no_pdl)
    b0, e0 = frame_range(n, rank, ws)
    for f0 in range(b0, e0, B):
        batch_frames([min(f, e0 - 1) for f in range(f0, f0 + B)])
    # size the plan once: whole-frame capacities, every distinct batch of this rank once, then the largest measured
    # level counts + 25 %; warm up
    need = None
    for bt in list(batch_cache.values()):
        ref.refine(*bt[:4], uv_bias=bt[4], K=K)
        rc, counts = ref.engine.status()
        if rc != 0:
            raise RuntimeError(f"c4: device status {rc}")
        need = counts if need is None else [max(a, c) for a, c in zip(need, counts)]
    ref.engine.fit_to(need)
    ref._K = None
    warm = next(iter(batch_cache.values()))
    for _ in range(2):
        ref.refine(*warm[:4], uv_bias=warm[4], K=K)
    sharded = ShardedRefiner(ref, n)
    out_host = torch.empty((e0 - b0, mdl["H"], mdl["W"], 3), dtype=torch.float32).pin_memory()
    if ws > 1:
        dist.barrier()
    torch.cuda.synchronize()
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record()
    _, fits = sharded.run(None, K=K, batch_frames=batch_frames, out=out_host)
    s1.record()
    torch.cuda.synchronize()
    rc, _ = ref.engine.status()
    if rc != 0:
        raise RuntimeError(f"c4: device status {rc} in the timed run")
    ms = s0.elapsed_time(s1)
    t = torch.tensor([ms], device=dev)
    if ws > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    ref.close()
    return {"metric": "refined frames/s (C4: Model A 480x640, K=3, frame-batch sharded)",
            "value": round(n / (ms * 1e-3), 2), "unit": "frames/s", "frames": n, "K": K, "batch_per_replay": B,
            "n_gpus": ws, "frames_per_rank": [e - b for b, e in (frame_range(n, r, ws) for r in range(ws))],
            "ms": round(ms, 2), "frames_per_s_per_gpu": round(n / (ms * 1e-3) / ws, 2),
            "fit_states_gathered": int(fits.shape[0]), "scaling": "strong (the frame set is fixed)",
            "timing": "CUDA events around the whole sharded run (per batch: pinned H2D of its inputs, the K-step "
                      "graph, D2H of the refined point maps into a pinned per-rank buffer, batches queued without a "
                      "host wait; the final all-gather of the fit states), max over ranks",
            "data": "synthetic: frame f is seeded room 500 + f mod 8"}


def post_output(torch, out, sc, dev, cpu: bool, reps: int = 20):
    """The output path of infer after the refine loop on the refined frame (promptmoge_b200.post.postprocess:
    resize + remap to the 480x640 image, focal / shift, shifted depth, final LiDAR fit, point map, gauge): device
    time (CUDA events, mean of `reps`), and the CPU time of the same steps through torch's CPU resize, the numpy
    focal / shift, fit, point-map and gauge oracle (the reference solves focal / shift with scipy on the host)."""
    from promptmoge_b200 import post
    coords = out.detach().clone()
    ld = torch.from_numpy(sc.lidar_depth).to(dev)
    lc = torch.from_numpy(sc.lidar_conf).to(dev)
    H, W = coords.shape[1], coords.shape[2]
    pg = post.PostGraph(coords.shape[0], (H, W), (H, W), tuple(ld.shape[-2:]), device=dev)
    for _ in range(3):
        pg.run(coords, ld, lc)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        pg.run(coords, ld, lc)
    e1.record()
    e1.synchronize()
    res = {"frames": int(coords.shape[0]), "image_hw": [H, W], "gpu_us": round(e0.elapsed_time(e1) * 1e3 / reps, 1),
           "timing": "the captured post graph (post.PostGraph), CUDA events, mean of replays"}
    if cpu:
        import numpy as np
        import torch.nn.functional as F
        from oracle import fit as ofit
        from oracle import gauge as ogauge
        from oracle import post as opost
        c = coords.cpu()
        t0 = time.perf_counter()
        r = F.interpolate(c.movedim(-1, -3), (H, W), mode="bilinear", align_corners=False).movedim(-3, -1).numpy()
        pts = opost.remap_exp(r)
        f, s = opost.recover_focal_shift(pts)
        depth = (pts[..., 2] + s[:, None, None]).astype(np.float32)
        depth, _, _ = ofit.final_fit(depth, sc.lidar_depth, sc.lidar_conf)
        fx, fy = zip(*[opost.focal_to_fxfy(np.float32(x), W, H) for x in f])
        points = opost.depth_to_points(depth, fx, fy)
        corr = ogauge.prompt_gauge_poly(depth, sc.lidar_depth[:, 0], sc.lidar_conf[:, 0], degree=2)
        _ = (points * corr[..., None], depth * corr)
        res["cpu_us"] = round((time.perf_counter() - t0) * 1e6, 1)
        res["cpu_kind"] = "torch CPU resize + numpy oracle of focal/shift, fit, point map, gauge; 1 thread"
    return res


def prompt_prep(torch, sc, dev, cpu: bool, reps: int = 50):
    """The per-frame LiDAR prompt preparation in front of the refiner (promptmoge.infer: nearest_fill of the
    192x256 sensor frame, then build_prompt onto the 420x560 token grid of 1200 tokens): device time of the two
    kernels pairs (CUDA events, mean of `reps`), and the CPU time of the same work through scipy's exact distance
    transform (the reference's call) plus the numpy prompt oracle."""
    from promptmoge_b200 import ops
    ld = torch.from_numpy(sc.lidar_depth).to(dev)
    lc = torch.from_numpy(sc.lidar_conf).to(dev)
    fd, fc = torch.empty_like(ld), torch.empty_like(lc)
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        for _ in range(3):
            ops.nearest_fill(ld, lc, out=(fd, fc))
            ops.build_prompt(fd, fc, (420, 560))
    torch.cuda.current_stream(dev).wait_stream(side)
    # each step captured once, so the figures are device time (CUDA graph replays), not Python launch overhead
    g_fill, g_prompt = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_fill):
        ops.nearest_fill(ld, lc, out=(fd, fc))
    with torch.cuda.graph(g_prompt):
        ops.build_prompt(fd, fc, (420, 560))
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    ev[0].record()
    for _ in range(reps):
        g_fill.replay()
    ev[1].record()
    for _ in range(reps):
        g_prompt.replay()
    ev[2].record()
    ev[2].synchronize()
    out = {"frames": int(ld.shape[0]), "sensor_hw": list(ld.shape[-2:]), "token_grid_hw": [420, 560],
           "nearest_fill_us": round(ev[0].elapsed_time(ev[1]) * 1e3 / reps, 2),
           "build_prompt_us": round(ev[1].elapsed_time(ev[2]) * 1e3 / reps, 2),
           "timing": "CUDA graph replays of each step, CUDA events, mean"}
    if cpu:
        import numpy as np
        from scipy import ndimage
        from oracle import prompt as oprompt
        d = sc.lidar_depth.reshape(-1, *sc.lidar_depth.shape[-2:])
        c = sc.lidar_conf.reshape(-1, *sc.lidar_conf.shape[-2:])
        t0 = time.perf_counter()
        filled = []
        for b in range(d.shape[0]):
            valid = d[b] > 0
            idx = ndimage.distance_transform_edt(~valid, return_distances=False, return_indices=True)
            filled.append((d[b][tuple(idx)], np.where(valid, c[b], 1).astype(np.float32)))
        t1 = time.perf_counter()
        oprompt.build_prompt(np.stack([f[0] for f in filled])[:, None], np.stack([f[1] for f in filled])[:, None],
                             (420, 560))
        t2 = time.perf_counter()
        out["cpu"] = {"nearest_fill_us": round((t1 - t0) * 1e6, 1), "build_prompt_us": round((t2 - t1) * 1e6, 1),
                      "kind": "scipy distance_transform_edt (the reference's call) + numpy prompt oracle, 1 thread"}
    return out


def cpu_baseline(batch=1, steps=1):
    """The CPU port (a restatement of the reference's CPU path) on the host cores: one full 480x640 step."""
    dt, sample = _port_step(steps, 1)
    return {"value": round(batch / dt, 5), "unit": UNIT, "cores": os.cpu_count(), "kind": "port", "sample": sample,
            "reference_measured": reference_cpu_record()}


def profile_step(args):
    """Profiling driver (run under ncu, one kernel family per capture with -k): the 480x640 Model A refine step of
    the benchmark frame replayed --steps times after one sizing run (every structure, fit, row and conv kernel of the
    step), then one hash neighbour map over a 2M-voxel surface-shell set (the generic-voxel-set builder of
    configuration 3) and one output path of the refined frame (the gauge fit).  Not a bench value."""
    import torch
    from promptmoge_b200 import ops, post, synth
    from promptmoge_b200.refine import Refiner, pinned, synthetic_model
    torch.cuda.set_device(0)
    weights, clips = synthetic_model("A", 0)
    sc = synth.make_scene(0, 480, 640, 16, 256)
    ref = Refiner(weights, clips, "A")
    h = [pinned(x) for x in (sc.point_coord, sc.lidar_depth, sc.lidar_conf, sc.encoder_feature, sc.uv_bias)]
    ref.refine(*h[:4], uv_bias=h[4])
    rc, counts = ref.engine.status()
    ref.engine.fit_to(counts)
    ref._K = None
    flush = torch.empty(256 << 18, dtype=torch.float32, device="cuda")
    for _ in range(max(1, args.steps)):
        flush.zero_()
        out, _ = ref.refine(*h[:4], uv_bias=h[4])
    coords = torch.from_numpy(synth.make_surface_voxels(2_000_000, seed=5)).cuda()
    nmap, mask, st = ops.nmap_hash(coords, [1, 1 << 21, 1 << 21, 1 << 21])
    torch.cuda.synchronize()
    coords_out = out.cuda()
    ld, lc = torch.from_numpy(sc.lidar_depth).cuda(), torch.from_numpy(sc.lidar_conf).cuda()
    pg = post.PostGraph(1, (480, 640), (480, 640), (192, 256), device="cuda")
    pg.run(coords_out, ld, lc)
    torch.cuda.synchronize()
    ref.close()
    return {"profile_step": True, "steps": args.steps, "levels_voxels": counts, "hash_voxels": int(coords.shape[0]),
            "hash_status": int(st.item())}


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
    grid0 = k == 0 and not args.simt and ops.grid0_supported(C_, C_)
    ws_ = torch.full((C_,), 1e-3, device="cuda")
    b = torch.zeros(C_, device="cuda")
    lanes = ops.l0_tap_lanes(l["z"], 1, 480, 640) if grid0 else None
    for _ in range(max(1, args.steps)):
        if grid0:   # level 0 runs the neighbour-map-free frame-grid kernel in the plan
            ops.spconv_i8_grid0(q, lanes, 1, 480, 640, w, ws_, b, 0.01, ops.EPI_SILU_Q8, 0.02)
        else:
            ops.spconv_i8(q, l["nmap_tm"], l["mask"], w, ws_, b, 0.01, ops.EPI_SILU_Q8, 0.02, rows=M,
                          tensor_cores=tc_path)
    torch.cuda.synchronize()
    nnz = int((l["nmap_tm"][:, :M] >= 0).sum().item())
    return {"profile_conv": k, "M": M, "C": C_, "occupied_taps": nnz,
            "path": "tcgen05 frame grid" if grid0 else ("tcgen05" if tc_path else "simt")}


def conv_sweep(args):
    """Benchmark configuration 3: the isolated int8 submanifold conv on surface-shell voxel sets (about 9 occupied taps per
    voxel) of N in {1e5, 5e5, 2e6, 8e6} voxels, C in {16, 32, 64, 128}: neighbour map by the hash builder, then the
    conv (tcgen05 where the width allows, SIMT dp4a at C = 16) with the SiLU + requantise epilogue, timed alone with
    CUDA events (median of --steps, inputs 2-128 MB, L2 flushed before each launch).  One JSON line per (N, C) with
    voxel*GOPS = 2 * occupied taps * C * C / t."""
    import torch
    from promptmoge_b200 import ops, synth
    torch.cuda.set_device(0)
    flush = torch.empty(256 << 18, dtype=torch.float32, device="cuda")
    sizes = [int(x) for x in args.sweep_n.split(",")]
    for N in sizes:
        coords = torch.from_numpy(synth.make_surface_voxels(N, seed=N % 97)).cuda()
        M = coords.shape[0]
        nmap, mask, st = ops.nmap_hash(coords, [1, 1 << 21, 1 << 21, 1 << 21])
        if int(st.item()) != 0:
            raise RuntimeError("hash neighbour map failed")
        nnz = int((nmap >= 0).sum().item())
        for C in (16, 32, 64, 128):
            g = torch.Generator(device="cuda").manual_seed(C)
            q = torch.randint(-127, 127, (M, C), dtype=torch.int8, device="cuda", generator=g)
            w = torch.randint(-127, 127, (27, C, C), dtype=torch.int8, device="cuda", generator=g)
            ws_ = torch.full((C,), 1e-3, device="cuda")
            b = torch.zeros(C, device="cuda")
            run = lambda: ops.spconv_i8(q, nmap, mask, w, ws_, b, 0.01, ops.EPI_SILU_Q8, 0.02)
            for _ in range(3):
                run()
            torch.cuda.synchronize()
            ts = []
            for _ in range(max(3, args.steps)):
                flush.zero_()
                s0, e0 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s0.record()
                run()
                e0.record()
                torch.cuda.synchronize()
                ts.append(s0.elapsed_time(e0))
            t = float(np.median(ts))
            print(json.dumps({"metric": "int8 sparse-conv voxel*GOPS (C3)", "value": round(2.0 * nnz * C * C / (t * 1e-3) / 1e9, 1),
                              "unit": "GOPS", "N": M, "C": C, "ms": round(t, 4), "occupied_taps_per_voxel":
                              round(nnz / M, 2), "path": "tcgen05" if ops.tc_supported(C, C) else "simt",
                              "data": "synthetic surface shells", "l2": "flushed before each launch"}), flush=True)
        del nmap, mask


def _rows_of_index(idx, C: int):
    """Seeded int8 rows [n, C] as a function of the voxels' global indices (the same rows whichever rank holds them)."""
    import torch
    ch = torch.arange(C, device=idx.device, dtype=torch.int64)
    h = (idx.to(torch.int64)[:, None] * 2654435761 + ch[None, :] * 40503 + 12345) & 0xFFFFFFFF
    h = (h ^ (h >> 15)) * 2246822519 & 0xFFFFFFFF
    return ((h >> 13) % 255 - 127).to(torch.int8)


def fused_scene(args, ws, rank, local):
    """Benchmark configuration 5: one synthetic 12 x 12 x 3 m room seen from --fused-poses poses (480 x 640, random walk),
    fused into a 1 cm voxel grid and sharded by Morton ranges WITHOUT a global view: each rank back-projects its own
    contiguous share of the poses, voxels go to the owners of their code ranges (count-balanced splitters from one
    all-gather of code samples), neighbours across a range boundary are looked up at their owner, and every coarser
    level is the parents (code >> 3) of the level below, each level with its own count-balanced ranges
    (promptmoge_b200.fused.build_levels).
    The timed step is a sharded U-Net encoder with Model A's widths (32, 64, 128, 256, 256), two int8 submanifold
    convs per level (tcgen05, SiLU + requantise epilogue), each after a one-voxel halo exchange (NCCL all-to-all of
    int8 rows), and between levels the mean pool into parents (children moved to their parent's owner, summed in code
    order) plus the transition's int8 linear.  value = voxel-layers/s of the whole job (strong scaling: the scene is fixed).  Rank
    0 also runs the same pipeline as the only rank over the whole scene and every level's output is compared."""
    import hashlib
    import torch
    import torch.distributed as dist
    from promptmoge_b200 import fused, ops
    from promptmoge_b200.dist import frame_range
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    widths = [32, 64, 128, 256, 256]
    convs, links = fused.encoder_layers(widths, 2, seed=7, device=dev)

    def nmap_fn(coords, ext):
        nm, _, st = ops.nmap_hash(coords, ext)
        if int(st.item()) != 0:
            raise RuntimeError("hash neighbour map failed")
        return nm

    group = None if ws > 1 else fused.LOCAL
    layout = fused.scene_layout(0, args.fused_poses)
    b, e = frame_range(args.fused_poses, rank, ws)
    if ws > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    local_codes = fused.scene_codes(0, layout, range(b, e), device=dev)
    torch.cuda.synchronize()
    t1 = time.perf_counter()
    levels = fused.build_levels(local_codes, len(widths), nmap_fn, group, aligned=args.fused_ranges == "aligned")
    pools = [fused.PoolPlan(levels[k], levels[k + 1], group) for k in range(len(widths) - 1)]
    torch.cuda.synchronize()
    t2 = time.perf_counter()
    q0 = _rows_of_index(torch.arange(levels[0].offset, levels[0].offset + levels[0].plan.n_own, device=dev),
                        widths[0])

    def step(overlap=True):
        return fused.encoder_forward(levels, q0, convs, links, fused.gpu_conv, fused.gpu_link, group, pools=pools,
                                     overlap=overlap)

    graph_error = []

    def timed(overlap, graph=False):
        for _ in range(args.warmup):
            step(overlap)
        torch.cuda.synchronize()
        g = None
        if graph:
            # the whole step (convs, exchanges, pools, links) as one CUDA graph: no host work per launch.  Every rank
            # captures; the ranks agree (one all-reduce outside the capture) before any replay.
            ok = torch.ones(1, device=dev)
            try:
                side = torch.cuda.Stream(dev)
                side.wait_stream(torch.cuda.current_stream(dev))
                with torch.cuda.stream(side):
                    step(overlap)
                torch.cuda.current_stream(dev).wait_stream(side)
                torch.cuda.synchronize()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    o_graph = step(overlap)
            except RuntimeError as exc:
                g = None
                ok.zero_()
                graph_error.append(str(exc).splitlines()[0][:300] if str(exc) else type(exc).__name__)
            torch.cuda.synchronize()
            if ws > 1:
                dist.all_reduce(ok, op=dist.ReduceOp.MIN)
            if float(ok.item()) < 1.0:
                g = None
                return None, None, None
        if ws > 1:
            dist.barrier()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with Clocks(local) as clk:
            s0.record()
            for _ in range(args.steps):
                if g is not None:
                    g.replay()
                    o = o_graph
                else:
                    o = step(overlap)
            s1.record()
            torch.cuda.synchronize()
        if ws > 1:
            dist.barrier()
        outs_ = [x.clone() for x in o]
        del g                                      # released before the process group is destroyed
        torch.cuda.synchronize()
        return s0.elapsed_time(s1), outs_, clk

    # three ways to run the same step, all bit-identical: eager (exchange then conv), eager with every exchange
    # beside the interior rows' conv (several ranks only), and the plain step replayed as one CUDA graph (when its
    # capture succeeds on every rank).  The fastest is the line's value; every one is reported.
    ms_eager, outs, clk = timed(False)
    modes = {"eager": (ms_eager, clk)}
    if ws > 1:
        ms_o, outs_o, clk_o = timed(True)
        if not all(torch.equal(a, b) for a, b in zip(outs, outs_o)):
            raise RuntimeError("the overlapped fused-scene step differs from the eager step")
        modes["eager_overlapped"] = (ms_o, clk_o)
    ms_g, outs_g, clk_g = timed(False, graph=True)
    if ms_g is not None:
        if not all(torch.equal(a, b) for a, b in zip(outs, outs_g)):
            raise RuntimeError("graph replay of the fused-scene step differs from the eager step")
        modes["graph"] = (ms_g, clk_g)
    # the same mode on every rank: the slowest rank's time per mode decides
    names = ["eager", "eager_overlapped", "graph"]
    tm = torch.tensor([modes[n][0] if n in modes else float("inf") for n in names], device=dev, dtype=torch.float64)
    if ws > 1:
        dist.all_reduce(tm, op=dist.ReduceOp.MAX)
    mode_ms = {n: float(t) for n, t in zip(names, tm.tolist()) if n in modes}
    best = min(mode_ms, key=mode_ms.get)
    ms, clk = mode_ms[best], modes[best][1]
    build = [t1 - t0, t2 - t1]
    counts = [[l.plan.n_own for l in levels]]
    halos = [[l.plan.n_halo for l in levels]]
    digests = [hashlib.sha256(o.cpu().numpy().tobytes()).hexdigest() for o in outs]
    all_digests = [digests]
    if ws > 1:
        t = torch.tensor(build, device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        build = [float(x) for x in t]
        gathered = [None] * ws
        dist.all_gather_object(gathered, (counts[0], halos[0], digests))
        counts = [g[0] for g in gathered]
        halos = [g[1] for g in gathered]
        all_digests = [g[2] for g in gathered]
    verified = None
    if rank == 0:
        # the same pipeline as the only rank over the whole scene
        whole = fused.scene_codes(0, layout, range(args.fused_poses), device=dev)
        ref_levels = fused.build_levels(whole, len(widths), nmap_fn, fused.LOCAL)
        ref_q0 = _rows_of_index(torch.arange(ref_levels[0].plan.n_own, device=dev), widths[0])
        ref = fused.encoder_forward(ref_levels, ref_q0, convs, links, fused.gpu_conv, fused.gpu_link, fused.LOCAL)
        # each rank's rows of a level are one contiguous Morton range of the whole level: compare their digests
        verified = True
        for k in range(len(widths)):
            off = 0
            for r in range(ws):
                n = counts[r][k]
                d = hashlib.sha256(ref[k][off:off + n].cpu().numpy().tobytes()).hexdigest()
                verified = verified and d == all_digests[r][k]
                off += n
            verified = verified and off == ref[k].shape[0]
        M = [sum(c[k] for c in counts) for k in range(len(widths))]
    if rank != 0:
        return None
    vl = sum(M[k] * len(convs[k]) for k in range(len(widths)))
    value = vl * args.steps / (ms * 1e-3)
    return {"metric": "fused-scene voxel-layers/s (C5)", "value": round(value, 1), "unit": "voxel-layers/s",
            "n_gpus": ws, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4),
            "step_mode": best, "ms_per_step_by_mode": {n: round(v / args.steps, 4) for n, v in mode_ms.items()},
            "graph_error": graph_error[0] if graph_error else None,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": f"C5: fused scene, {args.fused_poses} poses 480x640 into a 1 cm grid ({M[0]} voxels), "
                                   "sharded U-Net encoder with Model A widths: 2 int8 submanifold convs per level, "
                                   "halo exchange before each, mean pool + int8 linear between levels",
                       "voxels_per_level": M, "voxels_per_rank_per_level": counts, "halo_rows_per_rank_per_level": halos,
                       "convs_per_level": 2, "widths": widths,
                       "build_s": {"backproject_own_poses": round(build[0], 3),
                                   "levels_sharded_structure": round(build[1], 3)},
                       "sharding": ("Morton ranges: level 0 cut to balance the whole encoder's work, every coarser "
                                    "level's ranges the parent codes of the level-0 boundaries (a parent's children "
                                    "stay on its rank)") if args.fused_ranges == "aligned" else
                                   ("Morton ranges balanced on every level's own count; parents whose children all "
                                    "sit on one rank are pooled there and only the pooled row moves"),
                       "exchange": "NCCL all-to-all (halo rows; children to their parent's owner) before each "
                                   "conv; eager_overlapped: each halo exchange beside the conv of the rows with no "
                                   "halo neighbour, the boundary rows' conv after it lands",
                       "modes": "eager = host-issued launches; graph = the step (convs, exchanges, pools, links) "
                                "as one CUDA graph replay; all modes give identical outputs"},
            "verified_vs_single_device": verified, "level_output_sha256_rank0": digests, "clocks": clk.summary()}


def _port_step(steps: int, warm: int):
    """Time the CPU port of one refine step (the oracle: exact int8 convs in C on all host threads, oracle/conv.c, the
    rest in numpy), Model A at 480x640 plus the final metric fit; returns (seconds per step, description)."""
    from oracle import build as obuild
    from oracle import fit as ofit
    from oracle import refiner as oref
    from promptmoge_b200 import synth
    from promptmoge_b200.refine import synthetic_model
    obuild.build()           # the C restatement, if this host did not receive it prebuilt (gcc, seconds)
    weights, clips = synthetic_model("A", 0)
    ch = synth.MODELS["A"]["model_channels"]
    qr = oref.QuantRefiner(weights, clips, ch, [2] * (len(ch) - 1))
    sc = synth.make_scene(0, 480, 640, 16, 256, batch=1)
    enc = sc.encoder_feature.astype(np.float32)

    def one():
        new_pc, _ = oref.refine_step(qr, sc.point_coord, sc.lidar_depth, sc.lidar_conf, enc, sc.uv_bias)
        ofit.final_fit(np.exp(new_pc[..., 2]).astype(np.float32), sc.lidar_depth, sc.lidar_conf)

    for _ in range(warm):
        one()
    t0 = time.perf_counter()
    for _ in range(steps):
        one()
    dt = (time.perf_counter() - t0) / steps
    conv = "C (OpenMP, all host threads)" if oref._native() is not None else "numpy"
    desc = (f"{steps} timed + {warm} warm-up full 480x640 Model A refine steps + final metric fit, CPU port "
            f"(convs in {conv}, the rest numpy): {dt:.2f} s/step")
    return dt, desc


def reference_cpu_record():
    """The reference's own CPU path timed beside the port on one host (tests/golden/reference_cpu_timing.json,
    written by tests/golden/time_reference_cpu.py where the reference is importable; it is not on the GPU hosts)."""
    p = ROOT / "tests" / "golden" / "reference_cpu_timing.json"
    if not p.exists():
        return None
    r = json.loads(p.read_text())
    return {"reference_s_per_step": r["reference_s_per_step"], "port_s_per_step": r["port_s_per_step"],
            "port_over_reference": r["port_over_reference"], "threads": r["host"]["threads"],
            "source": "tests/golden/reference_cpu_timing.json (the reference's moge v3 refine-loop body on its bundled "
                      "FlexGEMM fallback, fp32, vs this port, same host, same frame)"}


def run_reference(args, ws, rank):
    """Reference arm: the reference's CPU algorithm (the oracle port) on the host cores, rank 0 only.  The reference
    itself is Python and is not importable on the GPU hosts; its own CPU time, measured beside this port on one host,
    is attached as `reference_measured`."""
    if rank != 0:
        return None
    steps = max(1, min(args.steps, 3))
    warm = min(args.warmup, 1)
    dt, sample = _port_step(steps, warm)
    v = round(1.0 / dt, 5)
    return {"impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": ws, "steps": steps,
            "warmup": warm, "ms_per_step": round(dt * 1e3, 1), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "steps_note": "CPU steps take seconds: at most 3 timed steps (the GPU arm times --steps)",
            "scope": "one frame at a time on the host cores of one machine, whatever --gpus says",
            "config": {"workload": "C2: Model A refiner, 1 refine step, 480x640, batch 1 (synthetic room, seed 0)",
                       "K": 1},
            "cpu_baseline": {"value": v, "unit": UNIT, "cores": os.cpu_count(), "kind": "port", "sample": sample,
                             "reference_measured": reference_cpu_record()},
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--K", type=int, default=1, help="refine steps per graph (the workload's K)")
    ap.add_argument("--batch", type=int, default=1, help="frames per GPU per step")
    ap.add_argument("--no-pdl", action="store_true",
                    help="ordinary instead of programmatic kernel-to-kernel edges in the step graph")
    ap.add_argument("--max-split", type=int, default=4,
                    help="split-K limit of the plan's wide convs of levels with fewer tiles than SMs (1 = off)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--ncu", action="store_true", help="profiling mode: warm-up + timed replays only, no extras")
    ap.add_argument("--profile-conv", type=int, default=None, metavar="LEVEL",
                    help="profiling driver: launch one level's conv --steps times on the benchmark frame's structure")
    ap.add_argument("--profile-step", action="store_true",
                    help="profiling driver: --steps refine steps, a 2M-voxel hash neighbour map and one output path")
    ap.add_argument("--simt", action="store_true", help="with --profile-conv: the SIMT kernel instead of tcgen05")
    ap.add_argument("--model", choices=["A", "B"], default="A",
                    help="A: the headline config (480x640); B: config 1 (Model B, 240x320)")
    ap.add_argument("--conv-sweep", action="store_true", help="config 3: isolated int8 conv sweep (one line per N, C)")
    ap.add_argument("--sweep-n", default="100000,500000,2000000,8000000")
    ap.add_argument("--fused-scene", action="store_true", help="config 5: fused multi-pose scene over Morton shards")
    ap.add_argument("--fused-poses", type=int, default=200)
    ap.add_argument("--fused-ranges", choices=["aligned", "balanced"], default="balanced",
                    help="config 5: coarser levels' ranges the parents of level 0's (aligned) or balanced per level")
    ap.add_argument("--c4-frames", type=int, default=256,
                    help="config 4 sub-record: frames of the batched sharded run (0 = skip)")
    ap.add_argument("--c4-K", type=int, default=3)
    ap.add_argument("--c4-batch", type=int, default=4, help="config 4: frames per graph replay")
    ap.add_argument("--c5-poses", type=int, default=200,
                    help="config 5 sub-record: poses of the fused scene run after the main line (0 = skip)")
    ap.add_argument("--c5-steps", type=int, default=10, help="config 5 sub-record: timed encoder steps")
    args = ap.parse_args()
    if args.profile_conv is not None:
        print(json.dumps(profile_conv(args)), flush=True)
        return
    if args.profile_step:
        print(json.dumps(profile_step(args)), flush=True)
        return
    if args.conv_sweep:
        conv_sweep(args)
        return
    if args.fused_scene:
        ws, rank, local = _dist()
        line = fused_scene(args, ws, rank, local)
        if ws > 1:
            import torch.distributed as dist
            dist.barrier()
            dist.destroy_process_group()
        if line is not None:
            print(json.dumps(line), flush=True)
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
