"""The engine run from a deployed refiner.bin directory (int8 weights and scales as stored, fp16 parameters widened)
equals the engine run from the fp32 master weights with those parameters rounded to fp16 the same way, bit for
bit, including the baked UV conditioning used when refine() is given none."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _fp16_params(weights, levels):
    """Every parameter the format stores as fp16 (biases, LayerNorm affine, the three projections) rounded to fp16;
    the quantised layers' master weights untouched (the format stores their int8 quantisation)."""
    from promptmoge_b200.engine import quantised_layer_names
    q = {n + ".weight" for n in quantised_layer_names(levels)}
    return {k: v if k in q else v.astype(np.float16).astype(np.float32) for k, v in weights.items()}


def test_refiner_dir_equals_fp16_rounded_weights(tmp_path):
    from promptmoge_b200 import synth
    from promptmoge_b200.refine import Refiner, pinned, synthetic_model
    from promptmoge_b200.refiner_bin import write_refiner_dir
    m = synth.MODELS["B"]
    weights, clips = synthetic_model("B", 0)
    sc = synth.make_scene(6, m["H"], m["W"], m["encoder_downsample"], m["model_channels"][-1], batch=2)
    uv = sc.uv_bias[0]
    write_refiner_dir(tmp_path, weights, clips, m["model_channels"], uv, encoder_downsample=8)
    a = Refiner.from_refiner_dir(tmp_path, batch=2)
    b = Refiner(_fp16_params(weights, 4), clips, "B", batch=2)
    try:
        args = (pinned(sc.point_coord), pinned(sc.lidar_depth), pinned(sc.lidar_conf), pinned(sc.encoder_feature))
        pa, fa = a.refine(*args)                             # baked UV planes
        pa = pa.clone()
        uvb = np.ascontiguousarray(np.broadcast_to(uv, sc.uv_bias.shape))
        pb, fb = b.refine(*args, uv_bias=pinned(uvb))
        assert torch.equal(pa, pb)
        assert fa == fb
        assert a.engine.status()[0] == 0
    finally:
        a.close()
        b.close()
