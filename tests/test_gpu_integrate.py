"""install_refiner on the GPU: a stand-in MoGeModel's refine loop (the reference loop's per-step calls, in its order)
runs on the library's fit kernels and the captured refiner plan, and refines to the same bits as the plan's own
fused K-step run, and within the depth tolerance of the oracle."""
import numpy as np
import pytest
import torch

from stub_moge import stub_model

pytestmark = pytest.mark.gpu


def _scene(model, seed, H=None, W=None):
    from promptmoge_b200 import synth
    m = synth.MODELS[model]
    H, W = H or m["H"], W or m["W"]
    return synth.make_scene(seed, H, W, m["encoder_downsample"], m["model_channels"][-1]), H, W


def _dev(sc):
    return (torch.from_numpy(sc.point_coord).cuda(), torch.from_numpy(sc.encoder_feature).cuda(),
            torch.from_numpy(sc.uv_bias).cuda(), torch.from_numpy(sc.lidar_depth).cuda(),
            torch.from_numpy(sc.lidar_conf).cuda())


@pytest.mark.parametrize("model,hw,K", [("B", None, 1), ("B", None, 2), ("A", (48, 64), 1), ("A", None, 1)])
def test_hooked_loop_equals_fused_plan(model, hw, K):
    from promptmoge_b200 import synth
    from promptmoge_b200.engine import Geometry, RefinerEngine
    from promptmoge_b200.integrate import install_refiner, uninstall_refiner
    from promptmoge_b200.refine import synthetic_model
    sc, H, W = _scene(model, 41, *(hw or (None, None)))
    pc, enc, uv, ld, lc = _dev(sc)
    m = stub_model(model)
    install_refiner(m)
    try:
        got = m.refine_loop(pc, enc, uv, ld, lc, K)
        again = m.refine_loop(pc, enc, uv, ld, lc, K)          # the captured graph, replayed
    finally:
        uninstall_refiner(m)
    torch.cuda.synchronize()
    assert torch.equal(got, again)
    weights, clips = synthetic_model(model, 0)
    eng = RefinerEngine(weights, clips, Geometry(channels=synth.MODELS[model]["model_channels"], height=H, width=W))
    try:
        eng.set_frame(enc, uv)
        eng.set_inputs(pc, ld, lc)
        want, _ = eng.run(K)
        torch.cuda.synchronize()
        assert torch.equal(got, want)
    finally:
        eng.close()


def test_hooked_loop_matches_oracle_and_reference(golden):
    """A_small: the hooked loop's refined depth vs the oracle's refine step and the reference's own (fixture)."""
    from oracle import refiner as oref
    from promptmoge_b200 import synth
    from promptmoge_b200.integrate import install_refiner
    g = golden("A_small")
    sc = g.scene()
    from promptmoge_b200.integrate import uninstall_refiner
    from stub_moge import StubMoGe, StubRefiner
    # the fixture's own weights and clips
    unet = StubRefiner(synth.MODELS["A"]["model_channels"])
    unet.load_state_dict({k: torch.from_numpy(v) for k, v in g.weights().items()}, strict=True)
    unet.attach_clips(g.clips)
    m = StubMoGe(unet.eval())
    install_refiner(m)
    pc, enc, uv, ld, lc = _dev(sc)
    try:
        got = m.refine_loop(pc, enc, uv, ld, lc, 1).cpu().numpy()[..., 2]
    finally:
        uninstall_refiner(m)
    widths = synth.MODELS["A"]["model_channels"]
    qr = oref.QuantRefiner(g.weights(), g.clips, widths, [2] * (len(widths) - 1))
    new_pc, _ = oref.refine_step(qr, sc.point_coord, sc.lidar_depth, sc.lidar_conf,
                                 sc.encoder_feature.astype(np.float32), sc.uv_bias)
    for ref_logz in (new_pc[..., 2], (g["s0_logz_in"] + g["s0_delta"]).astype(np.float32)):
        d_g, d_r = np.exp(got.astype(np.float64)), np.exp(ref_logz.astype(np.float64))
        assert np.mean(np.abs(d_g - d_r) / d_r) < 2e-3


def test_hooked_affine_frame_matches_oracle_fit(golden):
    from promptmoge_b200 import ops
    g = golden("A_small")
    sc = g.scene()
    pc, enc, uv, ld, lc = _dev(sc)
    log_d_aff, gate, s, t = ops.lidar_in_affine_frame(pc[..., 2], ld, lc, soft_gate=True)
    st = g["s0_fit_st"]
    np.testing.assert_allclose(s.cpu().numpy(), st[:, 0], rtol=1e-4)
    np.testing.assert_allclose(t.cpu().numpy(), st[:, 1], rtol=1e-4, atol=1e-4)
    pf = g["s0_prompt_feats"].reshape(log_d_aff.shape + (2,))
    np.testing.assert_array_equal(gate.cpu().numpy(), pf[..., 1])
    res = ((log_d_aff - pc[..., 2]) * gate).cpu().numpy()
    np.testing.assert_allclose(res, pf[..., 0], atol=1e-5)
