"""The optional refiner-side gates on the GPU (output gate, elastic anchor; moge/model/v3.py:565-573): the kernels
against the reference's outputs (tests/golden/gates.npz) -- the output gate bit for bit, the anchor within 5e-6 --
and the plan with both gates on against the oracle's step."""
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import refiner as oref

sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
import make_gates as mg  # noqa: E402

pytestmark = pytest.mark.gpu
G = np.load(Path(__file__).resolve().parent / "golden" / "gates.npz")


@pytest.mark.parametrize("name", list(mg.CASES))
def test_gate_kernels_against_reference(name):
    from promptmoge_b200 import ops
    cur, refined, ld, lc, floor, beta = mg.case(name)
    tl, tc = torch.from_numpy(ld).cuda(), torch.from_numpy(lc).cuda()
    x = torch.from_numpy(refined).cuda()
    if floor is not None:
        x = ops.output_gate(torch.from_numpy(cur).cuda(), x, tl, tc, floor)
    if beta > 0:
        x = ops.anchor(x, tl, tc, beta)
    got = x.cpu().numpy()
    if beta > 0:
        np.testing.assert_allclose(got, G[f"{name}_out"], rtol=0, atol=5e-6)
    else:
        np.testing.assert_array_equal(got, G[f"{name}_out"])


def test_plan_with_gates_matches_oracle(golden):
    from promptmoge_b200 import synth
    from promptmoge_b200.engine import Geometry, RefinerEngine
    g = golden("B_small")
    sc = g.scene()
    c = g.config
    widths = synth.MODELS[c["model"]]["model_channels"]
    geo = Geometry(channels=widths, height=c["H"], width=c["W"])
    eng = RefinerEngine(g.weights(), g.clips, geo, output_gate_floor=0.1, anchor_beta=0.3)
    eng.set_frame(torch.from_numpy(sc.encoder_feature).cuda(), torch.from_numpy(sc.uv_bias).cuda())
    eng.set_inputs(torch.from_numpy(sc.point_coord).cuda(), torch.from_numpy(sc.lidar_depth).cuda(),
                   torch.from_numpy(sc.lidar_conf).cuda())
    out, _ = eng.run(1)
    assert eng.status()[0] == 0
    got = out.cpu().numpy()
    eng.close()
    qr = oref.QuantRefiner(g.weights(), g.clips, widths, [2] * (len(widths) - 1))
    want, _ = oref.refine_step(qr, sc.point_coord, sc.lidar_depth, sc.lidar_conf, sc.encoder_feature.astype(np.float32),
                               sc.uv_bias, output_gate_floor=0.1, anchor_beta=0.3)
    plain, _ = oref.refine_step(qr, sc.point_coord, sc.lidar_depth, sc.lidar_conf,
                                sc.encoder_feature.astype(np.float32), sc.uv_bias)
    d_g, d_o = np.exp(got[..., 2].astype(np.float64)), np.exp(want[..., 2].astype(np.float64))
    assert np.mean(np.abs(d_g - d_o) / d_o) < 2e-3
    assert np.abs(got[..., 2] - want[..., 2]).max() < 2e-3
    assert np.abs(want[..., 2] - plain[..., 2]).max() > 1e-3        # the gates changed the step
