"""The fused refiner plan (one refine step as device work / one CUDA graph) against the oracle and the reference."""
import numpy as np
import pytest
import torch

from conftest import sha

pytestmark = pytest.mark.gpu


def _engine(g, batch=1):
    from promptmoge_b200 import synth
    from promptmoge_b200.engine import Geometry, RefinerEngine
    c = g.config
    geo = Geometry(channels=synth.MODELS[c["model"]]["model_channels"], height=c["H"], width=c["W"], batch=batch)
    return RefinerEngine(g.weights(), g.clips, geo)


def _inputs(eng, sc):
    eng.set_frame(torch.from_numpy(sc.encoder_feature).cuda(), torch.from_numpy(sc.uv_bias).cuda())
    eng.set_inputs(torch.from_numpy(sc.point_coord).cuda(), torch.from_numpy(sc.lidar_depth).cuda(),
                   torch.from_numpy(sc.lidar_conf).cuda())


@pytest.mark.parametrize("name", ["B_small", "A_small"])
def test_step_matches_oracle_and_reference(golden, name):
    from oracle import refiner as oref
    from promptmoge_b200 import synth
    g = golden(name)
    sc = g.scene()
    eng = _engine(g)
    _inputs(eng, sc)
    out, fit = eng.run(1)
    rc, counts = eng.status()
    assert rc == 0
    torch.cuda.synchronize()
    # structure of the step, read back from the plan, bit-exact against the reference
    widths = synth.MODELS[g.config["model"]]["model_channels"]
    for k in range(1, len(widths)):
        info = eng.level_info(k)
        M = counts[k]
        assert M == g[f"s0_L{k}_coords"].shape[0]
        nm = eng.debug_tensor("nmap", k, (27, info["cap"]), torch.int32)[:, :M].t().cpu().numpy()
        np.testing.assert_array_equal(nm, g[f"s0_L{k}_nmap"])
    # refined log-depth vs the oracle's step on the same inputs, and vs the reference
    qr = oref.QuantRefiner(g.weights(), g.clips, widths, [2] * (len(widths) - 1))
    new_pc, info = oref.refine_step(qr, sc.point_coord, sc.lidar_depth, sc.lidar_conf,
                                    sc.encoder_feature.astype(np.float32), sc.uv_bias)
    got = out.cpu().numpy()
    np.testing.assert_array_equal(got[..., :2], sc.point_coord[..., :2])
    for ref_logz in (new_pc[..., 2], (g["s0_logz_in"] + g["s0_delta"]).astype(np.float32)):
        d_g, d_r = np.exp(got[..., 2].astype(np.float64)), np.exp(ref_logz.astype(np.float64))
        assert np.mean(np.abs(d_g - d_r) / d_r) < 2e-3          # AbsRel-delta of the refined depth
        assert np.abs(got[..., 2] - ref_logz).max() < 2e-3


def test_graph_replay_is_bitwise_deterministic(golden):
    g = golden("A_small")
    sc = g.scene()
    eng = _engine(g)
    _inputs(eng, sc)
    ref, _ = eng.run(2)
    ref = ref.clone()
    out, _ = eng.capture(2)
    for _ in range(3):
        eng.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, ref)
    assert eng.status()[0] == 0


@pytest.mark.parametrize("name", ["B_full", "A_full"])
def test_full_size_step_against_reference(golden, name):
    """480x640 / 240x320: the plan's level structure hashes to the reference's, and the refined log-depth agrees with
    the reference's on its sampled pixels and over the whole frame (depth AbsRel-delta < 0.2 %)."""
    from promptmoge_b200 import synth
    g = golden(name)
    sc = g.scene()
    eng = _engine(g)
    _inputs(eng, sc)
    eng.capture(1)
    out, fit = eng.replay()
    rc, counts = eng.status()
    assert rc == 0
    widths = synth.MODELS[g.config["model"]]["model_channels"]
    for k in range(1, len(widths)):
        info = eng.level_info(k)
        nm = eng.debug_tensor("nmap", k, (27, info["cap"]), torch.int32)[:, :counts[k]].t().contiguous().cpu().numpy()
        assert sha(nm) == g.digests[f"s0_L{k}_nmap"], k
    got = out.cpu().numpy()[..., 2].reshape(-1)
    pix = g["s0_pix"]
    ref_logz = (g["s0_logz_in_pix"] + g["s0_delta_pix"]).astype(np.float32)
    d_g, d_r = np.exp(got[pix].astype(np.float64)), np.exp(ref_logz.astype(np.float64))
    assert np.mean(np.abs(d_g - d_r) / d_r) < 2e-3
    np.testing.assert_allclose(got[pix], ref_logz, atol=5e-3)
    # the whole frame: the reference's refinement of every pixel (stored in float16, ~1e-4 of a delta of ~0.1) added
    # to the input log-depth, depth AbsRel-delta < 0.2 %
    logz_in = sc.point_coord[..., 2].reshape(-1).astype(np.float64)
    ref_full = logz_in + g["s0_delta_f16"].reshape(-1).astype(np.float64)
    d_g, d_r = np.exp(got.astype(np.float64)), np.exp(ref_full)
    absrel = float(np.mean(np.abs(d_g - d_r) / d_r))
    assert absrel < 2e-3, absrel


def test_batched_frames_equal_single_frames(golden):
    """Frames are independent: a batch of two gives each frame's single-frame result bit for bit."""
    from promptmoge_b200 import synth
    g = golden("B_small")
    c = g.config
    sc2 = synth.make_scene(c["seed"], c["H"], c["W"], c["encoder_downsample"], 256, batch=2)
    eng2 = _engine(g, batch=2)
    _inputs(eng2, sc2)
    out2, _ = eng2.run(1)
    out2 = out2.cpu().numpy()
    for b in range(2):
        sc1 = synth.make_scene(c["seed"] + b, c["H"], c["W"], c["encoder_downsample"], 256, batch=1)
        eng1 = _engine(g)
        _inputs(eng1, sc1)
        out1, _ = eng1.run(1)
        np.testing.assert_array_equal(out2[b], out1.cpu().numpy()[0])


def test_tensor_core_plan_equals_simt_plan(golden):
    """The plan with tcgen05 int8 layers and the plan with SIMT int8 layers refine to the same bits."""
    from promptmoge_b200 import synth
    from promptmoge_b200.engine import Geometry, RefinerEngine
    g = golden("A_small")
    sc = g.scene()
    c = g.config
    geo = Geometry(channels=synth.MODELS[c["model"]]["model_channels"], height=c["H"], width=c["W"])
    outs = []
    for tc in (False, True):
        eng = RefinerEngine(g.weights(), g.clips, geo, tensor_cores=tc)
        _inputs(eng, sc)
        out, _ = eng.run(2)
        assert eng.status()[0] == 0
        outs.append(out.clone())
        eng.close()
    assert torch.equal(outs[0], outs[1])


@pytest.mark.parametrize("name", ["A_full", "A_small"])
def test_split_k_plan_equals_unsplit_plan(golden, name):
    """The plan's wide convs of the small levels split across CTAs (max_split=4) or not (max_split=1): identical
    bits, over captured-graph replays, with capacities fitted to the counts (the split count is chosen on the
    device)."""
    from promptmoge_b200 import synth
    from promptmoge_b200.engine import Geometry, RefinerEngine
    g = golden(name)
    sc = g.scene()
    c = g.config
    geo = Geometry(channels=synth.MODELS[c["model"]]["model_channels"], height=c["H"], width=c["W"])
    outs = []
    for ms in (1, 4):
        eng = RefinerEngine(g.weights(), g.clips, geo, max_split=ms)
        _inputs(eng, sc)
        eng.run(1)
        rc, counts = eng.status()
        assert rc == 0
        eng.fit_to(counts)
        _inputs(eng, sc)
        eng.capture(1)
        for _ in range(3):
            out, _ = eng.replay()
        assert eng.status()[0] == 0
        outs.append(out.clone())
        eng.close()
    assert torch.equal(outs[0], outs[1])


@pytest.mark.parametrize("name", ["A_full", "B_small"])
def test_programmatic_edges_equal_ordinary_edges(golden, name):
    """The step graph with programmatic kernel-to-kernel edges (each kernel scheduled during its predecessor's tail,
    waiting on the device) refines to the same bits as the graph with ordinary edges, replay after replay."""
    from promptmoge_b200 import synth
    from promptmoge_b200.engine import Geometry, RefinerEngine
    g = golden(name)
    sc = g.scene()
    c = g.config
    geo = Geometry(channels=synth.MODELS[c["model"]]["model_channels"], height=c["H"], width=c["W"])
    outs = []
    for pdl in (False, True):
        eng = RefinerEngine(g.weights(), g.clips, geo, pdl=pdl)
        _inputs(eng, sc)
        eng.capture(1)
        for _ in range(5):
            out, fit = eng.replay()
            outs.append((pdl, out.clone(), fit.clone()))
        assert eng.status()[0] == 0
        eng.close()
    ref = outs[0]
    for pdl, o, f in outs[1:]:
        assert torch.equal(o, ref[1]) and torch.equal(f, ref[2]), pdl


def test_refiner_frame_conditioning_follows_each_call():
    """Refiner.refine runs the per-frame conditioning (encoder tokens) on a side stream that the step waits for
    only before its encoder fusion: alternating two frames, every call refines with its own frame's tokens (same
    bits as the first call of that frame, and as the engine with set_frame on the step's stream)."""
    from promptmoge_b200 import synth
    from promptmoge_b200.engine import Geometry, RefinerEngine
    from promptmoge_b200.refine import Refiner, pinned, synthetic_model
    m = synth.MODELS["B"]
    weights, clips = synthetic_model("B", 0)
    scenes = [synth.make_scene(s, m["H"], m["W"], m["encoder_downsample"], m["model_channels"][-1], batch=1)
              for s in (21, 22)]
    args = [tuple(pinned(x) for x in (sc.point_coord, sc.lidar_depth, sc.lidar_conf, sc.encoder_feature, sc.uv_bias))
            for sc in scenes]
    ref = Refiner(weights, clips, "B", batch=1)
    try:
        first = [ref.refine(*a)[0].clone() for a in args]
        assert not torch.equal(first[0], first[1])
        for _ in range(3):
            for i, a in enumerate(args):
                assert torch.equal(ref.refine(*a)[0], first[i])
    finally:
        ref.close()
    geo = Geometry(channels=m["model_channels"], height=m["H"], width=m["W"])
    eng = RefinerEngine(weights, clips, geo)
    try:
        for i, sc in enumerate(scenes):
            _inputs(eng, sc)
            out, _ = eng.run(1)
            assert torch.equal(out.cpu(), first[i])
    finally:
        eng.close()


def test_set_frame_captured_with_the_steps():
    """set_frame recorded into the same stream capture as the steps: the step's encoder fusion depends on that
    capture's encoder GEMM (an ordinary graph edge), so each replay refines with the tokens copied in right before
    it.  Two frames alternate through one graph; every replay matches the uncaptured run of its frame."""
    from promptmoge_b200 import synth
    from promptmoge_b200.engine import Geometry, RefinerEngine
    from promptmoge_b200.refine import synthetic_model
    m = synth.MODELS["B"]
    weights, clips = synthetic_model("B", 0)
    scenes = [synth.make_scene(s, m["H"], m["W"], m["encoder_downsample"], m["model_channels"][-1], batch=1)
              for s in (31, 32)]
    geo = Geometry(channels=m["model_channels"], height=m["H"], width=m["W"])
    eng = RefinerEngine(weights, clips, geo)
    try:
        want = []
        for sc in scenes:
            _inputs(eng, sc)
            out, _ = eng.run(1)
            want.append(out.clone())
        torch.cuda.synchronize()
        assert not torch.equal(want[0], want[1])
        pc = torch.empty_like(want[0])
        ld = torch.empty(scenes[0].lidar_depth.shape, dtype=torch.float32, device="cuda")
        lc = torch.empty_like(ld)
        enc = torch.empty(scenes[0].encoder_feature.shape, dtype=torch.float16, device="cuda")
        uv = torch.empty(scenes[0].uv_bias.shape, dtype=torch.float32, device="cuda")
        eng.set_inputs(pc, ld, lc)
        eng._outputs()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            eng.set_frame(enc, uv)
            out, _ = eng.run(1)
        for _ in range(2):
            for i, sc in enumerate(scenes):
                for dst, src in ((pc, sc.point_coord), (ld, sc.lidar_depth), (lc, sc.lidar_conf),
                                 (enc, sc.encoder_feature), (uv, sc.uv_bias)):
                    dst.copy_(torch.from_numpy(src))
                g.replay()
                torch.cuda.synchronize()
                assert torch.equal(out, want[i]), i
        assert eng.status()[0] == 0
        del g
    finally:
        eng.close()


@pytest.mark.parametrize("name", ["A_full", "B_small"])
def test_one_launch_fit_plan_equals_multi_launch_fit_plan(golden, name):
    """The step with its LiDAR fit as one cluster launch refines to the same bits as the step with the
    multi-launch fit."""
    from promptmoge_b200 import synth
    from promptmoge_b200.engine import Geometry, RefinerEngine
    g = golden(name)
    sc = g.scene()
    c = g.config
    geo = Geometry(channels=synth.MODELS[c["model"]]["model_channels"], height=c["H"], width=c["W"])
    outs = []
    for multi in (True, False):
        eng = RefinerEngine(g.weights(), g.clips, geo, multi_launch_fit=multi)
        _inputs(eng, sc)
        eng.capture(1)
        out, fit = eng.replay()
        outs.append((out.clone(), fit.clone(), eng.launches_per_step()))
        assert eng.status()[0] == 0
        eng.close()
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])
    assert outs[1][2] < outs[0][2]          # the one-launch fit is in use where supported


@pytest.mark.parametrize("name", ["A_full", "B_full", "A_small"])
def test_fused_transitions_plan_equals_multi_launch_plan(golden, name):
    """Pool + linear + the next block's LayerNorm / SiLU / requantise in one row pass (the pooling transitions into
    widths up to 128) and the level-0 LayerNorm inside the input projection refine to the same bits
    as the plan that runs each of those steps as its own launch (the int8 linear by dp4a sums the same integers the
    tensor-core GEMM does)."""
    from promptmoge_b200 import synth
    from promptmoge_b200.engine import Geometry, RefinerEngine
    g = golden(name)
    sc = g.scene()
    c = g.config
    geo = Geometry(channels=synth.MODELS[c["model"]]["model_channels"], height=c["H"], width=c["W"])
    outs = []
    for multi in (True, False):
        eng = RefinerEngine(g.weights(), g.clips, geo, multi_launch_transitions=multi)
        _inputs(eng, sc)
        eng.capture(1)
        out, fit = eng.replay()
        L = geo.levels
        qs = [eng.debug_tensor("q1", k, (eng.level_info(k)["cap"], geo.channels[k]), torch.int8)[:eng.status(False)[1][k]].clone()
              for k in range(L)]
        outs.append((out.clone(), qs, eng.launches_per_step()))
        assert eng.status()[0] == 0
        eng.close()
    assert torch.equal(outs[0][0], outs[1][0])
    for a, b in zip(outs[0][1], outs[1][1]):
        assert torch.equal(a, b)
    assert outs[1][2] < outs[0][2]


def test_sharded_refiner_pipelined_batches_equal_single_frames():
    """ShardedRefiner on one process: 6 frames, 4 per graph replay (the last batch partial), copied straight into a
    pinned output without a host wait per batch, and through the Refiner's own staging buffer: every frame equals its
    single-frame refinement, and every frame's fit state is returned."""
    from promptmoge_b200 import synth
    from promptmoge_b200.dist import ShardedRefiner
    from promptmoge_b200.refine import Refiner, pinned, synthetic_model
    m = synth.MODELS["B"]
    weights, clips = synthetic_model("B", 0)
    scenes = [synth.make_scene(60 + i, m["H"], m["W"], m["encoder_downsample"], m["model_channels"][-1])
              for i in range(6)]
    keys = ("point_coord", "lidar_depth", "lidar_conf", "encoder_feature", "uv_bias")
    single = Refiner(weights, clips, "B", batch=1)
    try:
        want = [single.refine(*[pinned(getattr(sc, k)) for k in keys[:4]], uv_bias=pinned(sc.uv_bias), K=2)[0].clone()
                for sc in scenes]
    finally:
        single.close()
    ref = Refiner(weights, clips, "B", batch=4)
    try:
        def batch_frames(ids):
            return tuple(pinned(np.concatenate([getattr(scenes[i], k) for i in ids])) for k in keys)
        sharded = ShardedRefiner(ref, 6)
        out = torch.empty((6, m["H"], m["W"], 3), dtype=torch.float32).pin_memory()
        for o in (out, None):
            got, fits = sharded.run(None, K=2, batch_frames=batch_frames, out=o)
            assert fits.shape == (6, 18)
            for i in range(6):
                assert torch.equal(got[i:i + 1], want[i]), i
    finally:
        ref.close()
