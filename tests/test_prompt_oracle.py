"""The LiDAR prompt oracle (oracle/prompt.py) against the reference's own outputs (tests/golden/prompt.npz, made by
tests/golden/make_prompt.py from promptmoge.nearest_fill and prompt_stem.build_prompt): the fill bit for bit, the
prompt's exact channels bit for bit, channel 0 and mu within an ulp of log."""
import hashlib
import sys
from pathlib import Path

import numpy as np
import pytest

from oracle import prompt as op

sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
import make_prompt as mp  # noqa: E402

G = np.load(Path(__file__).resolve().parent / "golden" / "prompt.npz")


def _sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.mark.parametrize("name", list(mp.small_cases()))
def test_fill_small_cases(name):
    d, c = mp.small_cases()[name]
    np.testing.assert_array_equal(G[f"fill_{name}_depth_in"], d)
    fd, fc = op.nearest_fill(d, c)
    np.testing.assert_array_equal(fd, G[f"fill_{name}_depth"])
    np.testing.assert_array_equal(fc, G[f"fill_{name}_conf"])


@pytest.mark.parametrize("name", list(mp.LARGE))
def test_fill_sensor_frames(name):
    d, c = mp.frame(name)
    fd, fc = op.nearest_fill(d, c)
    assert _sha(np.asarray(fd, np.float32)) == str(G[f"fill_{name}_depth_sha"])
    assert _sha(fc) == str(G[f"fill_{name}_conf_sha"])


def test_fill_tie_rule_brute_force():
    """Every hole's source is at the minimum squared distance; among ties the smallest column, then row."""
    rng = np.random.default_rng(3)
    for _ in range(40):
        h, w = rng.integers(1, 14, 2)
        valid = rng.random((h, w)) < rng.choice([0.05, 0.3, 0.7])
        if not valid.any():
            continue
        r, c = op.nearest_valid_index(valid)
        vi, vj = np.nonzero(valid)
        for i in range(h):
            for j in range(w):
                dist = (vi - i) ** 2 + (vj - j) ** 2
                k = np.lexsort((vi, vj, dist))[0]
                assert (r[i, j], c[i, j]) == (vi[k], vj[k])


@pytest.mark.parametrize("name", list(mp.PROMPTS))
def test_build_prompt(name):
    d, c, hw = mp.prompt_inputs(name)
    p, mu = op.build_prompt(d, c, hw)
    assert p.shape == (d.shape[0], 4) + tuple(hw)
    assert _sha(p[:, 1:]) == str(G[f"{name}_exact_sha"])
    ch0 = p[:, 0][:, ::3, ::3] if p.shape[-1] > 100 else p[:, 0]
    np.testing.assert_allclose(ch0, G[f"{name}_ch0"], rtol=0, atol=1e-6)
    np.testing.assert_allclose(mu, G[f"{name}_mu"], rtol=0, atol=1e-6)
    if f"{name}_prompt" in G:
        np.testing.assert_array_equal(p[:, 1:], G[f"{name}_prompt"][:, 1:])
