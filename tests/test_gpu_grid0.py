"""Level-0 frame-grid conv (shifted TMA slabs + masked MMA lanes, no neighbour map): int32 accumulators hash to the
reference's exact accumulators for every level-0 conv of the fixtures, and every epilogue equals the gather kernel
(which is itself pinned to the reference) bit for bit on ragged, multi-frame and benchmark-size frames."""
import numpy as np
import pytest
import torch

from conftest import sha
from oracle import refiner as oref

pytestmark = pytest.mark.gpu


def _level0_convs(g):
    return [n for n in g.layer_names(0) if ".conv" in n and
            (n.startswith("down_stages.0.") or n.startswith(f"up_stages.{len(_widths(g)) - 2}."))]


def _widths(g):
    from promptmoge_b200 import synth
    return synth.MODELS[g.config["model"]]["model_channels"]


def _tap_major_weight(qw):
    return torch.from_numpy(np.ascontiguousarray(qw.reshape(qw.shape[0], 27, -1).transpose(1, 0, 2))).cuda()


@pytest.mark.parametrize("name", ["B_small", "A_small"])
def test_grid0_reference_accumulators(golden, name):
    """Every level-0 conv layer, given the reference's int8 input: accumulators equal the reference's (SHA-256 of
    the exact int32 sums), the dequantised output equals the oracle's fp32 arithmetic."""
    from promptmoge_b200 import ops
    from promptmoge_b200.engine import act_scale, quantise_weight
    g = golden(name)
    H, W = g.config["H"], g.config["W"]
    coords = g["s0_L0_coords"]
    assert coords.shape[0] == H * W
    zq = torch.from_numpy(np.ascontiguousarray(coords[:, 3]).astype(np.int32)).cuda()
    lanes = ops.l0_tap_lanes(zq, 1, H, W)
    w = g.weights()
    names = _level0_convs(g)
    assert len(names) == 4, names
    status = torch.zeros(1, dtype=torch.int32).cuda()
    for n in names:
        key = f"s0_Q_{n}"
        q = torch.from_numpy(g[key + "_q"]).cuda()
        qw, sw = quantise_weight(w[n + ".weight"])
        wt = _tap_major_weight(qw)
        acc = ops.spconv_i8_grid0(q, lanes, 1, H, W, wt, status=status)
        sa = act_scale(g.clips[n])
        f32 = ops.spconv_i8_grid0(q, lanes, 1, H, W, wt, torch.from_numpy(sw).cuda(),
                                  torch.from_numpy(w[n + ".bias"]).cuda(), sa, ops.EPI_F32, status=status)
        torch.cuda.synchronize()
        acc_np = acc.cpu().numpy()
        assert sha(acc_np) == g.digests[key + "_acc"], n
        np.testing.assert_array_equal(f32.cpu().numpy(), oref.dequant(acc_np.astype(np.int64), sa, sw,
                                                                      w[n + ".bias"]), err_msg=n)
    assert int(status.item()) == 0


def _rough_point_map(B, H, W, seed):
    """Point map whose quantised log-depth wanders by -2..2 steps between neighbours, so every tap (and absent
    neighbours) occurs, with unrelated frames."""
    rng = np.random.default_rng(seed)
    steps = rng.integers(-2, 3, (B, H, W)).astype(np.float64)
    zq = np.cumsum(np.cumsum(steps, axis=2) * 0.3, axis=1).round() + 400 + 37 * np.arange(B)[:, None, None]
    pc = np.zeros((B, H, W, 3), np.float32)
    pc[..., 0] = rng.standard_normal((B, H, W))
    pc[..., 1] = rng.standard_normal((B, H, W))
    pc[..., 2] = (zq / 256.0).astype(np.float32)
    return pc


CASES = [
    pytest.param(1, 480, 640, 32, "scene", id="A480x640-c32"),
    pytest.param(2, 37, 53, 32, "rough", id="2x37x53-c32-ragged"),
    pytest.param(3, 16, 24, 64, "rough", id="3x16x24-c64"),
    pytest.param(1, 48, 64, 64, "scene", id="48x64-c64"),
    pytest.param(1, 1, 200, 32, "rough", id="1x200-single-row"),
]


@pytest.mark.parametrize("B,H,W,C,kind", CASES)
def test_grid0_equals_gather_every_epilogue(B, H, W, C, kind):
    from promptmoge_b200 import ops, synth
    if kind == "scene":
        pc = synth.make_scene(3, H, W, 16, 256, batch=B).point_coord
    else:
        pc = _rough_point_map(B, H, W, seed=H * W + C)
    zq, _, _, nmap, mask = ops.voxelize_l0(torch.from_numpy(np.ascontiguousarray(pc)).cuda())
    lanes = ops.l0_tap_lanes(zq, B, H, W)
    N = B * H * W
    # the masks are the level-0 neighbour map in bit form
    nm = nmap.cpu().numpy()[:, :N]
    ln = lanes.cpu().numpy().view(np.uint32)
    rows = np.arange(N)
    bits = (ln[rows // 128, :, (rows // 32) % 4] >> (rows % 32)[:, None].astype(np.uint32)) & 1
    np.testing.assert_array_equal(bits.astype(bool), (nm >= 0).T)
    rng = np.random.default_rng(C + N)
    q = torch.from_numpy(rng.integers(-127, 128, (N, C)).astype(np.int8)).cuda()
    wt = torch.from_numpy(rng.integers(-127, 128, (27, C, C)).astype(np.int8)).cuda()
    ws = torch.from_numpy(rng.uniform(1e-4, 1e-3, C).astype(np.float32)).cuda()
    b = torch.from_numpy(rng.standard_normal(C).astype(np.float32)).cuda()
    resid = torch.from_numpy(rng.standard_normal((N, C)).astype(np.float32)).cuda()
    status = torch.zeros(1, dtype=torch.int32).cuda()
    for mode in (ops.EPI_ACC32, ops.EPI_F32, ops.EPI_F32_RESID, ops.EPI_SILU_Q8):
        want = ops.spconv_i8(q, nmap, mask, wt, ws, b, 0.03, mode, 0.05, resid, status=status)
        got = ops.spconv_i8_grid0(q, lanes, B, H, W, wt, ws, b, 0.03, mode, 0.05, resid, status=status)
        again = ops.spconv_i8_grid0(q, lanes, B, H, W, wt, ws, b, 0.03, mode, 0.05, resid, status=status)
        assert torch.equal(got, want), mode
        assert torch.equal(again, got), mode
    if kind == "rough":
        # the oracle's exact int64 accumulators over the level-0 neighbour map
        nm = nmap.cpu().numpy()[:, :N].T
        wnp = wt.cpu().numpy().transpose(1, 0, 2).reshape(C, 3, 3, 3, C)
        acc = ops.spconv_i8_grid0(q, lanes, B, H, W, wt).cpu().numpy()
        np.testing.assert_array_equal(acc.astype(np.int64), oref.conv_acc(q.cpu().numpy(), nm, wnp))
    assert int(status.item()) == 0


def test_grid0_rejects_unsupported_widths():
    from promptmoge_b200 import ops
    q = torch.zeros((64, 128), dtype=torch.int8).cuda()
    lanes = ops.l0_tap_lanes(torch.zeros(64, dtype=torch.int32).cuda(), 1, 8, 8)
    wt = torch.zeros((27, 128, 128), dtype=torch.int8).cuda()
    with pytest.raises(Exception):
        ops.spconv_i8_grid0(q, lanes, 1, 8, 8, wt)
