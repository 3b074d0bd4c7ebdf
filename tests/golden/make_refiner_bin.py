"""Golden record of the deployed refiner format (refiner.bin / refiner.json) written by the reference's own
exporter, promptmoge/export/refiner.py:28-111, for the synthetic Model A and Model B refiners of
promptmoge_b200.synth (seed 0) with the activation clips of promptmoge_b200/synth_clips.json.

    python tests/golden/make_refiner_bin.py /path/to/PromptMoGe

The exporter normally loads a trained checkpoint (load_model); here its ``load_model`` is replaced by a function
returning the reference's own Sparse3DUNet with the synthetic weights, QAT enabled (enable_refiner_qat) and each
activation quantiser's clip set, and the UV projection replaced by the synthetic scene's baked UV planes.  Everything
else -- the training quantiser, its bit-match assert, the block order, names, layouts and dtypes -- is the
exporter's unchanged code.  Writes tests/golden/refiner_bin.json: per model the exporter's refiner.json and the
SHA-256 and size of its refiner.bin (the binary itself is several MB and is not committed)."""
import hashlib
import json
import sys
import tempfile
import types
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(REPO))
from promptmoge_b200 import synth  # noqa: E402
from promptmoge_b200.refine import synthetic_model  # noqa: E402

UV_SEED = 77


def uv_planes(model: str) -> np.ndarray:
    """The baked UV conditioning [C_last, 30, 40] the fixture feeds the exporter (seeded)."""
    c_last = synth.MODELS[model]["model_channels"][-1]
    rng = np.random.default_rng(UV_SEED)
    return rng.normal(0, 0.3, (c_last, 30, 40)).astype(np.float32)


def main(ref: Path):
    sys.modules.setdefault("utils3d", types.ModuleType("utils3d"))
    sys.path.insert(0, str(ref / "promptmoge" / "_fallback"))
    sys.path.insert(0, str(ref))
    import torch
    from moge.model.modules.qat import enable_refiner_qat
    from moge.model.modules.sparse_unet import Sparse3DUNet
    import promptmoge.export.refiner as exporter

    out = {}
    for model in ("B", "A"):
        m = synth.MODELS[model]
        weights, clips = synthetic_model(model, 0)
        unet = Sparse3DUNet(in_channels=3, out_channels=1, encoder_channels=synth.ENC_CHANNELS,
                            model_channels=m["model_channels"], encoder_blocks_per_level=1,
                            decoder_blocks_per_level=1, bottleneck_blocks=1,
                            downsample_factors=m["downsample_factors"], encoder_downsample=m["encoder_downsample"],
                            prompt_channels=2)
        unet.load_state_dict({k: torch.from_numpy(v) for k, v in weights.items()}, strict=True)
        enable_refiner_qat(unet)
        for name, clip in clips.items():
            aq = getattr(unet, "aq_" + name.replace(".", "_"))
            aq.clip.fill_(clip)
            aq.observed.fill_(1)
        uvb = torch.from_numpy(uv_planes(model))
        fake = types.SimpleNamespace(refiner=unet.eval(), refiner_uv_fold=True, refiner_depth_resolution=256.0,
                                     refiner_uv_proj=lambda x, uvb=uvb: uvb[None])
        exporter.load_model = lambda name, base=None, fake=fake: fake
        with tempfile.TemporaryDirectory() as d:
            exporter.export(model, None, Path(d))
            blob = (Path(d) / "refiner.bin").read_bytes()
            index = json.loads((Path(d) / "refiner.json").read_text())
        out[model] = {"refiner_json": index, "bin_sha256": hashlib.sha256(blob).hexdigest(), "bin_bytes": len(blob)}
    dst = Path(__file__).resolve().parent / "refiner_bin.json"
    dst.write_text(json.dumps(out, indent=1))
    print("wrote", dst)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {sys.argv[0]} /path/to/PromptMoGe")
    main(Path(sys.argv[1]))
