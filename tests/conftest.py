import json
import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parents[1]
GOLDEN = REPO / "tests" / "golden"
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a) and the built extension")
    config.addinivalue_line("markers", "slow: full-size cases that take tens of seconds on CPU")


class Golden:
    """One committed fixture written by tests/golden/make_golden.py from the reference's own path."""

    def __init__(self, name: str):
        self.name = name
        self.z = np.load(GOLDEN / f"{name}.npz", allow_pickle=False)
        self.config = json.loads(str(self.z["config"]))
        self.digests = json.loads(str(self.z["digests"])) if "digests" in self.z.files else {}
        self.clips = json.loads(str(self.z["clips"])) if "clips" in self.z.files else {}

    def __getitem__(self, k):
        return self.z[k]

    def __contains__(self, k):
        return k in self.z.files

    def layer_names(self, step=0):
        p = f"s{step}_Q_"
        return sorted({k[len(p):].rsplit("_", 1)[0] for k in self.z.files if k.startswith(p) and k.endswith("_rows")
                       and not k.endswith("_acc_rows") and not k.endswith("_y_rows")})

    def scene(self):
        from promptmoge_b200 import synth
        c = self.config
        return synth.make_scene(c["seed"], c["H"], c["W"], c["encoder_downsample"],
                                synth.MODELS[c["model"]]["model_channels"][-1])

    def weights(self):
        from promptmoge_b200 import synth
        return synth.make_refiner_weights(self.config["model"], self.config["seed"])


@pytest.fixture(scope="session")
def golden():
    cache = {}

    def get(name):
        if name not in cache:
            cache[name] = Golden(name)
        return cache[name]
    return get


def sha(a: np.ndarray) -> str:
    import hashlib
    a = np.ascontiguousarray(a)
    return hashlib.sha256(a.dtype.str.encode() + str(a.shape).encode() + a.tobytes()).hexdigest()
