"""int8 submanifold conv and dense int8 layers on the GPU: int32 accumulators bit-exact against the reference's own
exact accumulators (fixture digests) and the oracle, epilogues bit-exact against the oracle's fp32 formulas."""
import numpy as np
import pytest
import torch

from conftest import sha
from oracle import refiner as oref

pytestmark = pytest.mark.gpu

SMALL = ["B_small", "A_small"]


def _widths(g):
    from promptmoge_b200 import synth
    return synth.MODELS[g.config["model"]]["model_channels"]


def _level_for_conv(name, L):
    if name.startswith("down_stages."):
        return int(name.split(".")[1])
    if name.startswith("bottleneck_stage"):
        return L - 1
    return L - 2 - int(name.split(".")[1])


def _tap_major(nmap_rm: np.ndarray):
    return torch.from_numpy(np.ascontiguousarray(nmap_rm.T)).cuda()


def _mask(nmap_rm: np.ndarray):
    occ = (nmap_rm >= 0).astype(np.int64) << np.arange(27)
    M = nmap_rm.shape[0]
    out = np.zeros((M + 31) // 32 + 1, np.int64)
    for t in range((M + 31) // 32):
        out[t] = np.bitwise_or.reduce(occ[t * 32:(t + 1) * 32].ravel())
    return torch.from_numpy(out.astype(np.uint32).view(np.int32)).cuda()


TC = [pytest.param(False, id="simt"), pytest.param(True, id="tcgen05")]


@pytest.mark.parametrize("tc", TC)
@pytest.mark.parametrize("name", SMALL)
def test_every_layer_accumulator_bit_exact(golden, name, tc):
    """Given the reference's int8 input of each of the 25/31 quantised layers, the GPU's int32 accumulators hash to
    the reference's exact accumulators, and each epilogue equals the oracle's fp32 arithmetic bit for bit."""
    from promptmoge_b200 import ops
    from promptmoge_b200.engine import act_scale, quantise_weight
    g = golden(name)
    widths = _widths(g)
    L = len(widths)
    w = g.weights()
    status = torch.zeros(1, dtype=torch.int32).cuda()
    for n in g.layer_names(0):
        key = f"s0_Q_{n}"
        q = torch.from_numpy(g[key + "_q"]).cuda()
        qw, sw = quantise_weight(w[n + ".weight"])
        bias = w[n + ".bias"]
        sa = act_scale(g.clips[n])
        ep = (torch.from_numpy(sw).cuda(), torch.from_numpy(bias).cuda(), sa, ops.EPI_F32)
        if ".conv" in n:
            nm = g[f"s0_L{_level_for_conv(n, L)}_nmap"]
            tm, mask = _tap_major(nm), _mask(nm)
            wt = torch.from_numpy(np.ascontiguousarray(qw.reshape(qw.shape[0], 27, -1).transpose(1, 0, 2))).cuda()
            acc = ops.spconv_i8(q, tm, mask, wt, tensor_cores=tc, status=status)
            f32 = ops.spconv_i8(q, tm, mask, wt, *ep, tensor_cores=tc, status=status)
        else:
            wt = torch.from_numpy(qw).cuda()
            acc = ops.dense_i8(q, wt, tensor_cores=tc, status=status)
            f32 = ops.dense_i8(q, wt, *ep, tensor_cores=tc, status=status)
        torch.cuda.synchronize()
        acc_np = acc.cpu().numpy()
        assert sha(acc_np) == g.digests[key + "_acc"], n
        y = oref.dequant(acc_np.astype(np.int64), sa, sw, bias)
        np.testing.assert_array_equal(f32.cpu().numpy(), y, err_msg=n)
        rows = g[key + "_rows"]
        yr = g[key + "_y_rows"]
        assert np.abs(f32.cpu().numpy()[rows] - yr).max() <= 1e-3 * np.abs(yr).max(), n
    assert int(status.item()) == 0


@pytest.mark.parametrize("tc", TC)
def test_fused_epilogues_match_oracle(golden, tc):
    from promptmoge_b200 import ops
    from promptmoge_b200.engine import act_scale, quantise_weight
    g = golden("A_small")
    w = g.weights()
    n1, n2 = "down_stages.1.0.conv1", "down_stages.1.0.conv2"
    q = torch.from_numpy(g[f"s0_Q_{n1}_q"]).cuda()
    nm = g["s0_L1_nmap"]
    tm, mask = _tap_major(nm), _mask(nm)
    qw, sw = quantise_weight(w[n1 + ".weight"])
    wt = torch.from_numpy(np.ascontiguousarray(qw.reshape(qw.shape[0], 27, -1).transpose(1, 0, 2))).cuda()
    sa, s_next = act_scale(g.clips[n1]), act_scale(g.clips[n2])
    args = (torch.from_numpy(sw).cuda(), torch.from_numpy(w[n1 + ".bias"]).cuda(), sa)
    acc = ops.spconv_i8(q, tm, mask, wt, tensor_cores=tc).cpu().numpy().astype(np.int64)
    y = oref.dequant(acc, sa, sw, w[n1 + ".bias"])
    q8 = ops.spconv_i8(q, tm, mask, wt, *args, ops.EPI_SILU_Q8, s_next, tensor_cores=tc).cpu().numpy()
    want = np.clip(np.rint(oref.silu(y) / np.float32(s_next)), -127, 127).astype(np.int8)
    # SiLU's exp may differ by an ulp between CUDA and numpy: allow rare one-step flips, nothing larger.
    d = np.abs(q8.astype(np.int32) - want.astype(np.int32))
    assert d.max() <= 1 and (d > 0).mean() < 1e-3
    resid = torch.randn(acc.shape, generator=torch.Generator().manual_seed(0)).cuda()
    r = ops.spconv_i8(q, tm, mask, wt, *args, ops.EPI_F32_RESID, 1.0, resid, tensor_cores=tc).cpu().numpy()
    np.testing.assert_array_equal(r, (y + resid.cpu().numpy()).astype(np.float32))


def test_tensor_core_path_equals_simt_path(golden):
    """The two int8 paths agree bit for bit on every epilogue (same accumulators, same epilogue arithmetic)."""
    from promptmoge_b200 import ops
    g = golden("A_small")
    nm = g["s0_L2_nmap"]
    tm, mask = _tap_major(nm), _mask(nm)
    rng = np.random.default_rng(7)
    C = 128
    q = torch.from_numpy(rng.integers(-127, 128, (nm.shape[0], C)).astype(np.int8)).cuda()
    wt = torch.from_numpy(rng.integers(-127, 128, (27, C, C)).astype(np.int8)).cuda()
    ws = torch.from_numpy(rng.uniform(1e-4, 1e-3, C).astype(np.float32)).cuda()
    b = torch.from_numpy(rng.standard_normal(C).astype(np.float32)).cuda()
    resid = torch.from_numpy(rng.standard_normal((nm.shape[0], C)).astype(np.float32)).cuda()
    for mode in (ops.EPI_ACC32, ops.EPI_F32, ops.EPI_F32_RESID, ops.EPI_SILU_Q8):
        a = ops.spconv_i8(q, tm, mask, wt, ws, b, 0.03, mode, 0.05, resid, tensor_cores=False)
        t = ops.spconv_i8(q, tm, mask, wt, ws, b, 0.03, mode, 0.05, resid, tensor_cores=True)
        assert torch.equal(a, t), mode


@pytest.mark.parametrize("tc", TC)
@pytest.mark.parametrize("name", ["conv_20k_c32", "conv_100k_c16"])
def test_conv_sweep_accumulators(golden, name, tc):
    from promptmoge_b200 import ops, synth
    g = golden(name)
    c = g.config
    coords = torch.from_numpy(synth.make_surface_voxels(c["N"], c["seed"])).cuda()
    nm_tm, mask, _ = ops.nmap_hash(coords, [1, 1 << 21, 1 << 21, 1 << 21])
    rng = np.random.default_rng(c["seed"] + 100)
    q = rng.integers(-127, 128, (coords.shape[0], c["C"])).astype(np.int8)
    qw = rng.integers(-127, 128, (c["C"], 3, 3, 3, c["C"])).astype(np.int8)
    wt = torch.from_numpy(np.ascontiguousarray(qw.reshape(c["C"], 27, c["C"]).transpose(1, 0, 2))).cuda()
    acc = ops.spconv_i8(torch.from_numpy(q).cuda(), nm_tm, mask, wt, tensor_cores=tc)
    torch.cuda.synchronize()
    assert sha(acc.cpu().numpy()) == str(g["acc_sha"])


@pytest.mark.parametrize("tc", TC)
@pytest.mark.parametrize("C", [16, 32, 64, 128, 256])
def test_conv_all_widths_against_oracle(C, tc):
    """Every channel width, random int8 data, with and without tile masks (all-taps path)."""
    from promptmoge_b200 import ops, synth
    from oracle import structure as ost
    coords_np = synth.make_surface_voxels(3000, seed=C)
    coords = torch.from_numpy(coords_np).cuda()
    ext = [1, 1 << 21, 1 << 21, 1 << 21]
    tm, mask, _ = ops.nmap_hash(coords, ext)
    rng = np.random.default_rng(C)
    q = rng.integers(-127, 128, (coords_np.shape[0], C)).astype(np.int8)
    qw = rng.integers(-127, 128, (C, 3, 3, 3, C)).astype(np.int8)
    wt = torch.from_numpy(np.ascontiguousarray(qw.reshape(C, 27, C).transpose(1, 0, 2))).cuda()
    want = oref.conv_acc(q, ost.nmap_sorted(coords_np, ext), qw)
    for m in (mask, None):
        got = ops.spconv_i8(torch.from_numpy(q).cuda(), tm, m, wt, tensor_cores=tc).cpu().numpy()
        np.testing.assert_array_equal(got.astype(np.int64), want)


@pytest.mark.parametrize("tc", TC)
@pytest.mark.parametrize("K,N", [(32, 64), (64, 128), (128, 256), (256, 256), (256, 128), (128, 64), (64, 32),
                                 (1024, 256), (512, 256), (96, 32)])
def test_dense_shapes_against_oracle(K, N, tc):
    from promptmoge_b200 import ops
    rng = np.random.default_rng(K * 1000 + N)
    M = 777
    a = rng.integers(-127, 128, (M, K)).astype(np.int8)
    w = rng.integers(-127, 128, (N, K)).astype(np.int8)
    got = ops.dense_i8(torch.from_numpy(a).cuda(), torch.from_numpy(w).cuda(), tensor_cores=tc).cpu().numpy()
    np.testing.assert_array_equal(got.astype(np.int64), oref.linear_acc(a, w))


@pytest.mark.parametrize("tc", TC)
def test_count_limits_rows(golden, tc):
    """Rows past the device-side count are not written (graph-safe sizing by capacity)."""
    from promptmoge_b200 import ops
    rng = np.random.default_rng(5)
    a = torch.from_numpy(rng.integers(-127, 128, (300, 64)).astype(np.int8)).cuda()
    w = torch.from_numpy(rng.integers(-127, 128, (32, 64)).astype(np.int8)).cuda()
    cnt = torch.tensor([100], dtype=torch.int32).cuda()
    out = ops.dense_i8(a, w, count=cnt, tensor_cores=tc)
    out_full = ops.dense_i8(a, w, tensor_cores=tc)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out[:100].cpu().numpy(), out_full[:100].cpu().numpy())


def test_float_conv_matches_reference_semantics(golden):
    """The fp32 operator behind the flex_gemm-compatible module: bias + sum_v W_v x[nmap_v] (within fp32 rounding)."""
    from promptmoge_b200 import ops
    g = golden("A_small")
    nm = g["s0_L1_nmap"]
    M = nm.shape[0]
    rng = np.random.default_rng(1)
    x = rng.standard_normal((M, 64)).astype(np.float32)
    w = rng.standard_normal((48, 3, 3, 3, 64)).astype(np.float32) * 0.05
    b = rng.standard_normal(48).astype(np.float32)
    want = np.tile(b.astype(np.float64), (M, 1))
    wv = w.reshape(48, 27, 64).astype(np.float64)
    for v in range(27):
        rows = np.nonzero(nm[:, v] >= 0)[0]
        want[rows] += x[nm[rows, v]].astype(np.float64) @ wv[:, v, :].T
    wt = torch.from_numpy(np.ascontiguousarray(w.reshape(48, 27, 64).transpose(1, 0, 2))).cuda()
    got = ops.spconv_f32(torch.from_numpy(x).cuda(), _tap_major(nm), _mask(nm), wt, torch.from_numpy(b).cuda())
    np.testing.assert_allclose(got.cpu().numpy(), want, rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("C,N,split", [(128, 3000, 4), (256, 3000, 3), (256, 12000, 2), (128, 60000, 4),
                                       (256, 200, 4), (128, 129, 2)])
def test_split_k_equals_single_pass(C, N, split):
    """Split-K (several CTAs per output tile, partial int32 tiles summed by the last arrival): accumulators equal the
    oracle's and every epilogue equals the single-pass kernel bit for bit, repeated launches included (the arrival
    counters return to zero)."""
    from promptmoge_b200 import ops, synth
    from oracle import structure as ost
    coords_np = synth.make_surface_voxels(N, seed=C + N)
    coords = torch.from_numpy(coords_np).cuda()
    ext = [1, 1 << 21, 1 << 21, 1 << 21]
    tm, mask, _ = ops.nmap_hash(coords, ext)
    rng = np.random.default_rng(C * 7 + N)
    M = coords_np.shape[0]
    q = torch.from_numpy(rng.integers(-127, 128, (M, C)).astype(np.int8)).cuda()
    qw = rng.integers(-127, 128, (C, 3, 3, 3, C)).astype(np.int8)
    wt = torch.from_numpy(np.ascontiguousarray(qw.reshape(C, 27, C).transpose(1, 0, 2))).cuda()
    ws = torch.from_numpy(rng.uniform(1e-4, 1e-3, C).astype(np.float32)).cuda()
    b = torch.from_numpy(rng.standard_normal(C).astype(np.float32)).cuda()
    resid = torch.from_numpy(rng.standard_normal((M, C)).astype(np.float32)).cuda()
    status = torch.zeros(1, dtype=torch.int32).cuda()
    if N <= 3000:
        want = oref.conv_acc(q.cpu().numpy(), ost.nmap_sorted(coords_np, ext), qw)
        got = ops.spconv_i8(q, tm, mask, wt, split=split, status=status).cpu().numpy()
        np.testing.assert_array_equal(got.astype(np.int64), want)
    for mode in (ops.EPI_ACC32, ops.EPI_F32, ops.EPI_F32_RESID, ops.EPI_SILU_Q8):
        one = ops.spconv_i8(q, tm, mask, wt, ws, b, 0.03, mode, 0.05, resid, status=status)
        for _ in range(2):
            sp = ops.spconv_i8(q, tm, mask, wt, ws, b, 0.03, mode, 0.05, resid, status=status, split=split)
            assert torch.equal(sp, one), mode
    assert int(status.item()) == 0


def _plan_structure(g):
    """Run one step of the refiner plan on the fixture's scene; return the engine (its level structures are
    SHA-equal to the reference's, tests/test_gpu_structure.py) and the per-level voxel counts."""
    from promptmoge_b200 import synth
    from promptmoge_b200.engine import Geometry, RefinerEngine
    c = g.config
    sc = g.scene()
    geo = Geometry(channels=synth.MODELS[c["model"]]["model_channels"], height=c["H"], width=c["W"])
    eng = RefinerEngine(g.weights(), g.clips, geo)
    eng.set_frame(torch.from_numpy(sc.encoder_feature).cuda(), torch.from_numpy(sc.uv_bias).cuda())
    eng.set_inputs(torch.from_numpy(sc.point_coord).cuda(), torch.from_numpy(sc.lidar_depth).cuda(),
                   torch.from_numpy(sc.lidar_conf).cuda())
    eng.run(1)
    rc, counts = eng.status()
    assert rc == 0
    return eng, counts


@pytest.mark.parametrize("name", ["A_full", "B_full", "A_small", "B_small"])
def test_seeded_accumulators_of_every_conv_bit_exact(golden, name):
    """Every submanifold conv layer of the refiner at the benchmark size, on a seeded int8 input
    (synth.seeded_conv_input) and the plan's own level structure, through the kernel the plan runs for that level:
    the frame-grid kernel at level 0, the tcgen05 gather kernel above it, and the split-K variant wherever the plan
    may split (levels with fewer output tiles than SMs; both split counts are run there).  The int32 accumulators
    hash to the reference's exact accumulators of the same layer on the same input (the bundled FlexGEMM fallback's
    submanifold_conv in float64 on its own neighbour cache)."""
    from promptmoge_b200 import ops, synth
    from promptmoge_b200.engine import quantise_weight
    g = golden(name)
    keys = sorted(k for k in g.digests if k.startswith("s0_S_"))
    assert keys, "fixture without seeded accumulator digests"
    widths = _widths(g)
    L = len(widths)
    B, H, W = 1, g.config["H"], g.config["W"]
    w = g.weights()
    eng, counts = _plan_structure(g)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    checked = 0
    try:
        for key in keys:
            n = key[len("s0_S_"):-len("_acc")]
            k = _level_for_conv(n, L)
            M, Cc = counts[k], widths[k]
            qs = torch.from_numpy(synth.seeded_conv_input(n, M, Cc)).cuda()
            qw, _ = quantise_weight(w[n + ".weight"])
            wt = torch.from_numpy(np.ascontiguousarray(qw.reshape(qw.shape[0], 27, -1).transpose(1, 0, 2))).cuda()
            info = eng.level_info(k)
            runs = []
            if k == 0 and ops.grid0_supported(Cc, Cc):
                lanes = eng.debug_tensor("lanes0", 0, ((B * H * W + 127) // 128, 27, 4), torch.int32)
                runs.append(("grid0", ops.spconv_i8_grid0(qs, lanes, B, H, W, wt, status=status)))
            else:
                cap = info["cap"]
                nmap = eng.debug_tensor("nmap", k, (27, cap), torch.int32)
                mask = eng.debug_tensor("tile_mask", k, (cap // 32 + 2,), torch.int32)
                cnt = torch.tensor([M], dtype=torch.int32, device="cuda")
                runs.append(("gather", ops.spconv_i8(qs, nmap, mask, wt, count=cnt, rows=M, status=status)))
                if Cc >= 128 and (M + 127) // 128 * (Cc // 128) < 148:
                    for sp in (2, 4):
                        runs.append((f"split{sp}", ops.spconv_i8(qs, nmap, mask, wt, count=cnt, rows=M,
                                                                 status=status, split=sp)))
            torch.cuda.synchronize()
            for kind, acc in runs:
                assert sha(acc[:M].cpu().numpy()) == g.digests[key], (n, kind)
                checked += 1
        assert int(status.item()) == 0
        assert checked >= len(keys)
    finally:
        eng.close()
