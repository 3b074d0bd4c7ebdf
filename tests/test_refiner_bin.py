"""The deployed refiner format (refiner.bin / refiner.json): this package's writer produces the bytes the reference's
exporter (promptmoge/export/refiner.py:28-111) produced for the same synthetic weights and clips (SHA-256 and block
index recorded by tests/golden/make_refiner_bin.py), and the reader returns the stored int8 weights, scales, fp16
parameters and clips unchanged."""
import hashlib
import json
import sys
from pathlib import Path

import numpy as np
import pytest

from promptmoge_b200 import synth
from promptmoge_b200.engine import quantise_weight, quantised_layer_names
from promptmoge_b200.refine import synthetic_model
from promptmoge_b200.refiner_bin import read_refiner_dir, write_refiner_dir

sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
import make_refiner_bin as mrb  # noqa: E402

G = json.loads((Path(__file__).resolve().parent / "golden" / "refiner_bin.json").read_text())


@pytest.mark.parametrize("model", ["B", "A"])
def test_writer_matches_reference_exporter(model, tmp_path):
    weights, clips = synthetic_model(model, 0)
    m = synth.MODELS[model]
    d = write_refiner_dir(tmp_path, weights, clips, m["model_channels"], mrb.uv_planes(model),
                          encoder_downsample=m["encoder_downsample"])
    blob = (d / "refiner.bin").read_bytes()
    assert len(blob) == G[model]["bin_bytes"]
    assert hashlib.sha256(blob).hexdigest() == G[model]["bin_sha256"]
    assert json.loads((d / "refiner.json").read_text()) == G[model]["refiner_json"]


def test_reader_round_trip(tmp_path):
    weights, clips = synthetic_model("B", 0)
    m = synth.MODELS["B"]
    uv = mrb.uv_planes("B")
    write_refiner_dir(tmp_path, weights, clips, m["model_channels"], uv, encoder_downsample=8)
    dep = read_refiner_dir(tmp_path)
    assert (dep.height, dep.width, dep.channels, dep.enc_channels) == (240, 320, m["model_channels"], 1024)
    np.testing.assert_array_equal(dep.uv_bias, uv)
    for name in quantised_layer_names(4):
        q, s = quantise_weight(weights[name + ".weight"])
        np.testing.assert_array_equal(dep.weights[name + ".weight_q8"], q)
        np.testing.assert_array_equal(dep.weights[name + ".weight_scale"], s)
        np.testing.assert_array_equal(dep.weights[name + ".bias"],
                                      weights[name + ".bias"].astype(np.float16).astype(np.float32))
        assert dep.clips[name] == np.float32(clips[name])
    for p in ("input_proj", "prompt_proj", "out_proj"):
        np.testing.assert_array_equal(dep.weights[p + ".weight"],
                                      weights[p + ".weight"].astype(np.float16).astype(np.float32))
    np.testing.assert_array_equal(dep.weights["bottleneck_stage.0.norm1.weight"],
                                  weights["bottleneck_stage.0.norm1.weight"].astype(np.float16).astype(np.float32))


def test_reader_rejects_truncated_file(tmp_path):
    weights, clips = synthetic_model("B", 0)
    write_refiner_dir(tmp_path, weights, clips, synth.MODELS["B"]["model_channels"], mrb.uv_planes("B"),
                      encoder_downsample=8)
    blob = (tmp_path / "refiner.bin").read_bytes()
    (tmp_path / "refiner.bin").write_bytes(blob[:-100])
    with pytest.raises(ValueError):
        read_refiner_dir(tmp_path)
