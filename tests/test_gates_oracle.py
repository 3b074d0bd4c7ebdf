"""The oracle's refiner-side gates (output gate, elastic anchor; moge/model/v3.py:565-573) against the reference's own
outputs (tests/golden/gates.npz, tests/golden/make_gates.py): the output gate bit for bit, the anchor (a fresh
trimmed least-squares fit and a log) within 5e-6."""
import sys
from pathlib import Path

import numpy as np
import pytest

from oracle import refiner as oref

sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
import make_gates as mg  # noqa: E402

G = np.load(Path(__file__).resolve().parent / "golden" / "gates.npz")


@pytest.mark.parametrize("name", list(mg.CASES))
def test_gates_match_reference(name):
    cur, refined, ld, lc, floor, beta = mg.case(name)
    got = oref.refiner_gates(cur, refined, ld, lc, floor, beta)
    if beta > 0:
        np.testing.assert_allclose(got, G[f"{name}_out"], rtol=0, atol=5e-6)
    else:
        np.testing.assert_array_equal(got, G[f"{name}_out"])
