"""LiDAR prompt preparation on the GPU (csrc/prompt.cu through the C ABI) against the reference's outputs
(tests/golden/prompt.npz) and the oracle: nearest_fill bit for bit (ties, single pixels, all / none present, NaN,
+inf, ragged and batched frames), build_prompt's exact channels bit for bit, channel 0 and mu within 1e-6 (one ulp
of log; CUDA's logf and the CPU's log may round differently)."""
import hashlib
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import prompt as op

sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
import make_prompt as mp  # noqa: E402

pytestmark = pytest.mark.gpu
G = np.load(Path(__file__).resolve().parent / "golden" / "prompt.npz")
TOL = 1e-6


def _sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def _fill(d, c):
    from promptmoge_b200 import ops
    fd, fc = ops.nearest_fill(torch.from_numpy(d).cuda(), torch.from_numpy(c).cuda())
    return fd.cpu().numpy(), fc.cpu().numpy()


@pytest.mark.parametrize("name", list(mp.small_cases()))
def test_fill_small_cases(name):
    d, c = mp.small_cases()[name]
    fd, fc = _fill(d, c)
    np.testing.assert_array_equal(fd, G[f"fill_{name}_depth"])
    np.testing.assert_array_equal(fc, G[f"fill_{name}_conf"])


@pytest.mark.parametrize("name", list(mp.LARGE))
def test_fill_sensor_frames(name):
    d, c = mp.frame(name)
    fd, fc = _fill(d, c)
    assert _sha(fd) == str(G[f"fill_{name}_depth_sha"])
    assert _sha(fc) == str(G[f"fill_{name}_conf_sha"])


def test_fill_batched_equals_per_frame():
    """A batch of frames (one of them fully present, one with no present pixel) equals each frame filled alone."""
    frames = [mp.frame(n) for n in ("L192x256_h5", "L192x256_h50", "L192x256_h98")]
    full = (np.random.default_rng(1).uniform(0.5, 3, (192, 256)).astype(np.float32), frames[0][1])
    empty = (np.zeros((192, 256), np.float32), frames[1][1])
    frames += [full, empty]
    d = np.stack([f[0] for f in frames])[:, None]
    c = np.stack([f[1] for f in frames])[:, None]
    fd, fc = _fill(d, c)
    wd, wc = op.nearest_fill_batch(d, c)
    np.testing.assert_array_equal(fd, wd)
    np.testing.assert_array_equal(fc, wc)
    np.testing.assert_array_equal(fd[3, 0], full[0])
    np.testing.assert_array_equal(fd[4, 0], empty[0])


@pytest.mark.parametrize("h,w,p", [(1, 1, 0.5), (2, 3000, 0.001), (3000, 2, 0.001), (33, 65, 0.01), (64, 31, 0.9),
                                   (97, 130, 0.0005), (384, 512, 0.03), (200, 1030, 0.2)])
def test_fill_random_shapes(h, w, p):
    rng = np.random.default_rng(h * 7 + w)
    d = np.where(rng.random((2, h, w)) < p, rng.uniform(0.2, 9, (2, h, w)), 0.0).astype(np.float32)
    d[0].flat[rng.integers(0, h * w)] = 4.0                      # frame 0 has at least one present pixel
    c = rng.choice(np.array([0, 1, 2], np.float32), (2, h, w))
    fd, fc = _fill(d, c)
    wd, wc = op.nearest_fill_batch(d, c)
    np.testing.assert_array_equal(fd, wd)
    np.testing.assert_array_equal(fc, wc)


def test_fill_rejects_aliasing_and_cpu():
    from promptmoge_b200 import _lib, ops
    d = torch.zeros((4, 4), device="cuda")
    with pytest.raises(ValueError):
        ops.nearest_fill(d.cpu())
    ws = torch.empty(_lib.load().pmg_prompt_workspace_bytes(1, 4, 4), dtype=torch.uint8, device="cuda")
    with pytest.raises(RuntimeError):
        _lib.call("pmg_nearest_fill", d.data_ptr(), d.data_ptr(), 1, 4, 4, d.data_ptr(), d.data_ptr(),
                  ws.data_ptr(), ws.numel(), None)


@pytest.mark.parametrize("name", list(mp.PROMPTS))
def test_build_prompt_golden(name):
    from promptmoge_b200 import ops
    d, c, hw = mp.prompt_inputs(name)
    p, st = ops.build_prompt(torch.from_numpy(d).cuda(), torch.from_numpy(c).cuda(), hw)
    p = p.cpu().numpy()
    mu = st["mu"].cpu().numpy()
    assert _sha(p[:, 1:]) == str(G[f"{name}_exact_sha"])
    ch0 = p[:, 0][:, ::3, ::3] if p.shape[-1] > 100 else p[:, 0]
    np.testing.assert_allclose(ch0, G[f"{name}_ch0"], rtol=0, atol=TOL)
    np.testing.assert_allclose(mu, G[f"{name}_mu"], rtol=0, atol=TOL)
    wp, wmu = op.build_prompt(d, c, hw)
    np.testing.assert_allclose(p[:, 0], wp[:, 0], rtol=0, atol=TOL)


def test_fill_then_prompt_pipeline():
    """promptmoge.infer's order: fill the sensor frame, then build the prompt on the token grid (420 x 560)."""
    from promptmoge_b200 import ops
    d, c = mp.frame("L192x256_h50")
    fd, fc = ops.nearest_fill(torch.from_numpy(d).cuda(), torch.from_numpy(c).cuda())
    p, st = ops.build_prompt(fd[None, None], fc[None, None], (420, 560))
    wd, wc = op.nearest_fill(d, c)
    wp, wmu = op.build_prompt(wd[None, None], wc[None, None], (420, 560))
    p = p.cpu().numpy()
    np.testing.assert_array_equal(p[:, 1:], wp[:, 1:])
    np.testing.assert_allclose(p[:, 0], wp[:, 0], rtol=0, atol=TOL)
    np.testing.assert_allclose(st["mu"].cpu().numpy(), wmu, rtol=0, atol=TOL)


def test_refiner_fill_option_equals_prefilled_inputs():
    """Refiner.refine(fill=True) fills the sensor frames on the device before the step graph: same refined points
    and fit as passing the oracle-filled frames with fill=False."""
    from promptmoge_b200 import synth
    from promptmoge_b200.refine import Refiner, pinned, synthetic_model
    m = synth.MODELS["B"]
    weights, clips = synthetic_model("B", 0)
    sc = synth.make_scene(4, m["H"], m["W"], m["encoder_downsample"], m["model_channels"][-1], batch=1)
    ld = sc.lidar_depth.copy()
    ld[..., 40:90, 60:140] = 0.0                                 # a large hole on top of the scene's own holes
    ref = Refiner(weights, clips, "B", batch=1)
    try:
        a, fa = ref.refine(pinned(sc.point_coord), pinned(ld), pinned(sc.lidar_conf), pinned(sc.encoder_feature),
                           pinned(sc.uv_bias), fill=True)
        a = a.clone()
        fd, fc = op.nearest_fill_batch(ld, sc.lidar_conf)
        b, fb = ref.refine(pinned(sc.point_coord), pinned(fd), pinned(fc), pinned(sc.encoder_feature),
                           pinned(sc.uv_bias), fill=False)
        assert torch.equal(a, b)
        assert fa == fb
    finally:
        ref.close()
