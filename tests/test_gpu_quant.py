"""The quantiser's fast path (reciprocal estimate, exact IEEE divide near rounding boundaries) returns exactly
clamp(rint(fl(x / s)), -127, 127) -- the reference's fake-quant rounding (qat.py:28-37) -- on adversarial inputs:
values on and one to four ulps either side of every half-integer boundary, far outside the clamp range, zeros,
infinities and NaN."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _exact_q8(x: np.ndarray, s: np.float32) -> np.ndarray:
    with np.errstate(invalid="ignore", over="ignore"):
        q = np.rint(x.astype(np.float32) / np.float32(s))
    q = np.where(np.isnan(q), -127.0, q)          # fmaxf(NaN, -127) = -127, as the device's clamp
    return np.clip(q, -127, 127).astype(np.int8)


def _boundary_values(s: np.float32) -> np.ndarray:
    h = (np.arange(-130, 131, dtype=np.float64) + 0.5)
    centre = (h * np.float64(s)).astype(np.float32)
    vals = [centre]
    up, down = centre.copy(), centre.copy()
    for _ in range(4):
        up = np.nextafter(up, np.float32(np.inf))
        down = np.nextafter(down, np.float32(-np.inf))
        vals += [up, down]
    rng = np.random.default_rng(int(s * 1e6) % 1000)
    vals.append((rng.standard_normal(200000) * 60 * s).astype(np.float32))
    vals.append(np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 1e30, -1e30, 1e-30], np.float32))
    return np.concatenate(vals).astype(np.float32)


@pytest.mark.parametrize("s", [0.0123457, 0.5, 1.0 / 127, 3.3e-4, 7.77])
def test_quantize_fast_path_exact(s):
    from promptmoge_b200 import ops
    s = np.float32(s)
    x = _boundary_values(s)
    got = ops.quantize(torch.from_numpy(x).cuda(), float(s)).cpu().numpy()
    np.testing.assert_array_equal(got, _exact_q8(x, s))


@pytest.mark.parametrize("C", [32, 64, 128, 256])
def test_pool_mean_q8_exact(C):
    """Mean of 1..8 children then quantise: equals fl(sum / n) rounded by the exact rule (sums in child order)."""
    from promptmoge_b200 import ops
    rng = np.random.default_rng(C)
    M_out = 5000
    counts = rng.integers(1, 9, M_out)
    off = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
    M_in = int(off[-1])
    idx = rng.permutation(M_in).astype(np.int32)
    s = np.float32(0.037)
    x = (rng.standard_normal((M_in, C)) * 2.0).astype(np.float32)
    # push some means onto rounding boundaries: make every child of the first 500 outputs equal (k + 0.5) * s
    for o in range(500):
        v = np.float32((rng.integers(-120, 120) + 0.5) * np.float64(s))
        x[idx[off[o]:off[o + 1]]] = v
    acc = np.zeros((M_out, C), np.float32)
    for o in range(M_out):
        for j in range(off[o], off[o + 1]):
            acc[o] = (acc[o] + x[idx[j]]).astype(np.float32)
    mean = (acc / counts[:, None].astype(np.float32)).astype(np.float32)
    want = _exact_q8(mean, s)
    got = ops.pool_mean(torch.from_numpy(x).cuda(), torch.from_numpy(idx).cuda(), torch.from_numpy(off).cuda(),
                        M_out, scale=float(s)).cpu().numpy()
    np.testing.assert_array_equal(got, want)


@pytest.mark.parametrize("C", [32, 64, 128, 256])
def test_layernorm_silu_fast_requantise_equals_exact(C):
    """The row-parallel LayerNorm + SiLU + requantise kernel uses the reciprocal-estimate quantiser; the warp-per-row
    kernel (taken when a row pointer is not 16-byte aligned) uses the exact IEEE chain.  Same bits on the same rows."""
    from promptmoge_b200 import ops
    rng = np.random.default_rng(C)
    M = 20000
    base = torch.from_numpy((rng.standard_normal(M * C + 1) * 3).astype(np.float32)).cuda()
    gamma = torch.from_numpy(rng.uniform(0.5, 2.0, C).astype(np.float32)).cuda()
    beta = torch.from_numpy((rng.standard_normal(C) * 0.3).astype(np.float32)).cuda()
    x_aligned = base[:M * C].clone().view(M, C)                    # 16-byte aligned: row-parallel kernel
    x_odd = base[1:].view(M, C)                                     # 4-byte offset: warp-per-row kernel
    x_odd.copy_(x_aligned)
    for scale in (0.021, 0.0371, 0.11):
        q_fast = ops.ln_silu_q8(x_aligned, gamma, beta, scale)
        q_exact = ops.ln_silu_q8(x_odd, gamma, beta, scale)
        torch.cuda.synchronize()
        assert torch.equal(q_fast, q_exact), scale
