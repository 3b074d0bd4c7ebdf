"""The sparse 3-D operators the refiner's U-Net imports from ``flex_gemm``, on this package's CUDA kernels.

Same functions, classes, argument meanings, return values and errors as the reference's operator module
(promptmoge/_fallback/flex_gemm/_core.py and nn/__init__.py), so that ``moge.model.modules.flex_sparse_blocks`` and
``sparse_unet`` run unchanged once this package is importable as ``flex_gemm`` (see ``install()``):

  submanifold_conv   out[o] = bias + sum_v W[:, v, :] @ in[nmap[o, v]]            (_core.py:399-441)
                     fp32, taps accumulated in tap order by pmg_spconv_f32.
  build_submanifold_cache  nmap[o, v] = index of coords[o] + delta[v], -1 if absent (_core.py:307-336)
                     one warp-cooperative hash build (pmg_nmap_hash) for every coordinate set; the kernel keeps the
                     tap-major copy ([27][M] plus per-32-row tap masks) and ``NeighborCache.nmap`` is its [M, 27]
                     view, the reference's layout.
  build_pool_cache   perfect-partition pool (kernel == stride == 2, padding 0), out coords = unique floor(c / 2) in
                     key order, parent / seg_indices / seg_offsets (_core.py:339-392), on pmg_frame_csr +
                     pmg_pool_frames: the refiner's levels are sorted by (column, z) (pixel order at level 0, unique
                     sorted keys after each pool), which is the order those kernels take.
  sparse_pool        mean (or sum) over CSR children in ascending fine index, one rounding per add (_core.py:444-481)
  sparse_upsample    nearest: out[c] = in[parent[c]] from the transposed pool cache (_core.py:484-505)

What the refiner does not use is refused with the reference's own error types: kernels other than 3x3x3 with dilation
1, pools other than kernel == stride == 2 with padding 0, pooling onto caller-given output coordinates, upsampling
other than nearest, and gradients (this is an inference path).  Every computation is a kernel of libpmg_b200.so;
there is no CPU path: tensors must live on a CUDA device.
"""
from __future__ import annotations

import itertools
from typing import Any, Literal, Sequence

import torch
from torch import Tensor

from .. import ops

__all__ = [
    "NeighborCache",
    "NeighborCacheT",
    "build_submanifold_cache",
    "build_pool_cache",
    "submanifold_conv",
    "sparse_pool",
    "sparse_upsample",
    "make_conv_kernel_delta",
]


def _broadcast(arg, D: int, name: str):
    if arg is None:
        return None
    if isinstance(arg, int):
        return (arg,) * D
    arg = tuple(int(a) for a in arg)
    assert len(arg) == D, f"{name} must have length {D}, got {arg}"
    return arg


def make_conv_kernel_delta(kernel_size: Sequence[int], dilation: Sequence[int], batch_dims: int = 0,
                           dtype: torch.dtype = torch.int32, device: torch.device | None = None) -> Tensor:
    """Tap offsets in the reference's order (_core.py:65-82): the cartesian product over
    range(-(k//2)*d, (k//2+1)*d, d) per spatial dimension, last dimension fastest, batch dimensions 0."""
    axes = [range(-(k // 2) * d, (k // 2 + 1) * d, d) for k, d in zip(kernel_size, dilation)]
    rows = list(itertools.product(*([(0,)] * batch_dims), *axes))
    return torch.tensor(rows, dtype=dtype, device=device)


def _require_cuda(t: Tensor, name: str) -> None:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor: the B200 operators have no CPU path")


def _check_status(status: Tensor, what: str) -> None:
    code = int(status.item())
    if code != 0:
        raise ValueError(f"{what} failed on the device with status {code}")


# --------------------------------------------------------------------------------------------------------------- #
# NeighborCache
# --------------------------------------------------------------------------------------------------------------- #
class NeighborCache:
    """Adjacency between an input and an output coordinate set (_core.py:131-212): ``nmap`` for the submanifold
    conv, ``seg_indices`` / ``seg_offsets`` / ``parent`` for a pool, ``.T`` for the upsample.

    Besides the reference's fields it holds what the kernels read: ``nmap_tm`` (tap-major [27, M] int32),
    ``tile_mask`` (per 32 output rows, the OR of the occupied taps) and ``seg_offsets32`` (int32 offsets)."""

    is_transposed = False

    def __init__(self, input_coords: Tensor, output_coords: Tensor, *, nmap: Tensor | None = None,
                 seg_indices: Tensor | None = None, seg_offsets: Tensor | None = None,
                 parent: Tensor | None = None, num_kernels: int | None = None,
                 kernel_size: tuple[int, ...] | None = None, dilation: tuple[int, ...] | None = None,
                 stride: tuple[int, ...] | None = None, input_sparse_shape: Sequence[int] | None = None,
                 output_sparse_shape: Sequence[int] | None = None, symmetric: bool = False,
                 build_backend: str = "sorted", nmap_tm: Tensor | None = None, tile_mask: Tensor | None = None,
                 seg_offsets32: Tensor | None = None) -> None:
        self.input_coords = input_coords
        self.output_coords = output_coords
        self._nmap = nmap
        self.nmap_tm = nmap_tm
        self.tile_mask = tile_mask
        self.seg_indices = seg_indices
        self.seg_offsets = seg_offsets
        self.seg_offsets32 = seg_offsets32
        self.parent = parent
        self.num_kernels = num_kernels
        self.kernel_size = kernel_size
        self.dilation = dilation
        self.stride = stride
        self.input_sparse_shape = None if input_sparse_shape is None else torch.Size(input_sparse_shape)
        self.output_sparse_shape = None if output_sparse_shape is None else torch.Size(output_sparse_shape)
        self.symmetric = symmetric
        self.build_backend = build_backend
        self._T: NeighborCacheT | None = None

    @property
    def nmap(self) -> Tensor | None:
        """(num_out, V) int32, -1 where absent: a view of the tap-major map the kernels read."""
        if self._nmap is None and self.nmap_tm is not None:
            return self.nmap_tm[:, : self.num_output_coords].t()
        return self._nmap

    @property
    def num_input_coords(self) -> int:
        return int(self.input_coords.shape[0])

    @property
    def num_output_coords(self) -> int:
        return int(self.output_coords.shape[0])

    @property
    def T(self) -> "NeighborCacheT":
        if self._T is None:
            self._T = NeighborCacheT(self)
        return self._T

    def transpose(self) -> "NeighborCacheT":
        return self.T

    def assert_match(self, *, input_coords=None, output_coords=None, is_transposed=None, **_kw) -> None:
        """Staleness check of a reused cache (_core.py:195-204)."""
        if input_coords is not None:
            assert input_coords.shape[0] == self.input_coords.shape[0], "stale neighbor cache (input rows)"
            assert input_coords.data_ptr() == self.input_coords.data_ptr() or torch.equal(
                input_coords, self.input_coords), "stale neighbor cache (input coords)"
        if output_coords is not None:
            assert output_coords.shape[0] == self.output_coords.shape[0], "stale neighbor cache (output rows)"
        if is_transposed is not None:
            assert bool(is_transposed) == bool(self.is_transposed)

    def occupancy(self) -> dict[str, float]:
        """Mean / max / min occupied taps per output row (_core.py:207-218)."""
        assert self.nmap is not None
        occ = (self.nmap >= 0).sum(dim=1).float()
        return {"V": float(self.nmap.shape[1]), "mean": float(occ.mean()), "max": float(occ.max()),
                "min": float(occ.min()), "rows": float(self.nmap.shape[0])}


class NeighborCacheT:
    """Transposed view of a pool cache, used by the nearest upsample (_core.py:221-242)."""

    is_transposed = True

    def __init__(self, base: NeighborCache) -> None:
        self.base = base
        self.input_coords = base.output_coords
        self.output_coords = base.input_coords
        self.parent = base.parent
        self.input_sparse_shape = base.output_sparse_shape
        self.output_sparse_shape = base.input_sparse_shape
        self.kernel_size = base.kernel_size
        self.stride = base.stride

    @property
    def T(self) -> NeighborCache:
        return self.base

    def assert_match(self, **_kw) -> None:
        return None


# --------------------------------------------------------------------------------------------------------------- #
# Cache construction
# --------------------------------------------------------------------------------------------------------------- #
def _coords_ok(coords: Tensor, sparse_shape: Sequence[int]) -> None:
    _require_cuda(coords, "coords")
    if coords.dtype != torch.int32 or coords.dim() != 2 or coords.shape[1] != 4:
        raise ValueError(f"coords must be int32 [M, 4] (batch + 3 spatial), got {tuple(coords.shape)} {coords.dtype}")
    if len(sparse_shape) != 4:
        raise ValueError(f"sparse shape must have 4 entries (B, X, Y, Z), got {tuple(sparse_shape)}")


def build_submanifold_cache(coords: Tensor, sparse_shape: Sequence[int], kernel_size: Sequence[int],
                            dilation: Sequence[int] | None = None,
                            backend: Literal["auto", "column", "sorted"] = "auto") -> NeighborCache:
    """Neighbour map of a coordinate set onto itself (_core.py:307-336).  Any backend name the reference accepts
    builds the same map here (a hash build); "column" still checks the one-voxel-per-column precondition and raises
    ValueError when it does not hold, like the reference."""
    D = len(kernel_size)
    dilation = tuple(dilation) if dilation is not None else (1,) * D
    if tuple(kernel_size) != (3, 3, 3) or dilation != (1, 1, 1):
        raise NotImplementedError(f"kernel_size={tuple(kernel_size)}, dilation={dilation}: the refiner uses 3x3x3 "
                                  "with dilation 1")
    _coords_ok(coords, sparse_shape)
    coords = coords.contiguous()
    if backend == "column" and not _one_voxel_per_column(coords, sparse_shape):
        raise ValueError("column backend requested but coords are not one-per-column")
    nmap_tm, mask, status = ops.nmap_hash(coords, [int(s) for s in sparse_shape])
    _check_status(status, "neighbour map")
    return NeighborCache(coords, coords, num_kernels=27, kernel_size=tuple(kernel_size), dilation=dilation,
                         input_sparse_shape=sparse_shape, output_sparse_shape=sparse_shape, symmetric=True,
                         build_backend="hash", nmap_tm=nmap_tm, tile_mask=mask)


def _one_voxel_per_column(coords: Tensor, sparse_shape: Sequence[int]) -> bool:
    B, H, W, Z = (int(s) for s in sparse_shape[:4])
    if coords.shape[0] != B * H * W:
        return False
    col_start, _, status = ops.frame_csr(coords, B, H, W, Z)
    if int(status.item()) != 0:
        return False
    return bool(torch.equal(col_start, torch.arange(B * H * W + 1, dtype=torch.int32, device=coords.device)))


def build_pool_cache(coords: Tensor, sparse_shape: Sequence[int], kernel_size: Sequence[int],
                     stride: Sequence[int], padding: Sequence[int], output_coords: Tensor | None = None,
                     output_sparse_shape: Sequence[int] | None = None) -> NeighborCache:
    """Perfect-partition pool cache (_core.py:339-392): out coords = unique floor(coords / 2) in key order (first
    occurrence), parent = each input row's output row, seg_indices = input rows grouped by parent in ascending
    order, seg_offsets (int64) their CSR offsets."""
    assert tuple(kernel_size) == tuple(stride), "only kernel == stride supported"
    assert all(p == 0 for p in padding), "only padding == 0 supported"
    if tuple(stride) != (2, 2, 2):
        raise NotImplementedError(f"stride={tuple(stride)}: the refiner pools by 2 in every spatial dimension")
    if output_coords is not None:
        raise NotImplementedError("pooling onto given output coords is not used by the refiner")
    _coords_ok(coords, sparse_shape)
    coords = coords.contiguous()
    B, H, W, Z = (int(s) for s in sparse_shape[:4])
    if output_sparse_shape is None:
        output_sparse_shape = [B, -(-H // 2), -(-W // 2), -(-Z // 2)]
    M = coords.shape[0]
    dev = coords.device
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    col_start, z, status = ops.frame_csr(coords, B, H, W, Z, status=status)
    fine_count = torch.tensor([M], dtype=torch.int32, device=dev)
    p = ops.pool_frames(B, H, W, col_start, z, None, max(M, 1), fine_count=fine_count, with_coords=True,
                        status=status)
    _check_status(status, "pool cache (inputs must be sorted by (b, x, y, z) with coordinates inside the shape)")
    n_out = int(p["count"][0].item())
    seg32 = p["seg_offsets"][: n_out + 1]
    return NeighborCache(coords, p["coords"][:n_out], seg_indices=p["seg_indices"][:M],
                         seg_offsets=seg32.to(torch.int64), parent=p["parent"][:M], kernel_size=tuple(kernel_size),
                         stride=tuple(stride), input_sparse_shape=sparse_shape,
                         output_sparse_shape=output_sparse_shape, build_backend="frames", seg_offsets32=seg32)


# --------------------------------------------------------------------------------------------------------------- #
# Ops
# --------------------------------------------------------------------------------------------------------------- #
def _no_grad_check(*tensors) -> None:
    if torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in tensors):
        raise NotImplementedError("the B200 sparse operators are inference-only: run under torch.no_grad() / "
                                  "torch.inference_mode()")


def submanifold_conv(feats: Tensor, coords: Tensor, shape: torch.Size, weight: Tensor, bias: Tensor | None = None, *,
                     dilation: Sequence[int] | None = None, neighbor_cache: NeighborCache | None = None,
                     **_ignored) -> tuple[Tensor, NeighborCache]:
    """weight is (Co, 3, 3, 3, Ci); returns (out [M, Co] in feats' dtype, the cache)."""
    kernel_size = tuple(weight.shape[1:-1])
    sparse_shape = tuple(shape[: coords.shape[1]])
    if neighbor_cache is None:
        neighbor_cache = build_submanifold_cache(coords, sparse_shape, kernel_size, dilation)
    else:
        neighbor_cache.assert_match(input_coords=coords, output_coords=coords, is_transposed=False)
    _require_cuda(feats, "feats")
    _no_grad_check(feats, weight, bias)
    Co, Ci = int(weight.shape[0]), int(weight.shape[-1])
    V = int(neighbor_cache.nmap_tm.shape[0])
    w_tm = weight.detach().reshape(Co, V, Ci).permute(1, 0, 2).contiguous().float()
    b = bias.detach().float().contiguous() if bias is not None else None
    out = ops.spconv_f32(feats.detach().float().contiguous(), neighbor_cache.nmap_tm, neighbor_cache.tile_mask, w_tm,
                         b, rows=feats.shape[0])
    return out.to(feats.dtype), neighbor_cache


def submanifold_conv_int8(feats: Tensor, coords: Tensor, shape: torch.Size, weight: Tensor, bias: Tensor | None,
                          clip: float, *, dilation: Sequence[int] | None = None,
                          neighbor_cache: NeighborCache | None = None) -> tuple[Tensor, NeighborCache]:
    """The QAT conv as the deployed int8 layer (moge/model/modules/qat.py:28-57, promptmoge/export/refiner.py:40-46):
    q = clamp(rint(feats / s_a), +-127) with s_a = clip / 127, q_w = clamp(rint(w / s_w), +-127) with
    s_w = amax|w[n]| / 127 per output channel, exact int32 accumulation on the tcgen05 kernel, y = acc * s_a * s_w + b.
    weight is the fp32 master (Co, 3, 3, 3, Ci).  Returns (out [M, Co] in feats' dtype, the cache)."""
    kernel_size = tuple(weight.shape[1:-1])
    sparse_shape = tuple(shape[: coords.shape[1]])
    if neighbor_cache is None:
        neighbor_cache = build_submanifold_cache(coords, sparse_shape, kernel_size, dilation)
    else:
        neighbor_cache.assert_match(input_coords=coords, output_coords=coords, is_transposed=False)
    _require_cuda(feats, "feats")
    Co, Ci = int(weight.shape[0]), int(weight.shape[-1])
    V = int(neighbor_cache.nmap_tm.shape[0])
    if V != 27 or not ops.tc_supported(Ci, Co):
        raise NotImplementedError(f"int8 tensor-core conv for a {V}-tap {Ci}->{Co} layer")
    from ..engine import act_scale
    s_a = act_scale(clip)
    q_in = ops.quantize(feats.detach().float().contiguous(), s_a)
    w = weight.detach().float()
    # IEEE divides throughout (a tensor divisor: torch turns a division by a Python scalar into a multiply by its
    # reciprocal, which can differ in the last bit)
    amax = w.abs().reshape(Co, -1).amax(dim=1)
    s_w = (amax / torch.full_like(amax, 127.0)).clamp_min(1e-12)
    q_w = torch.clamp(torch.round(w / s_w.view(-1, 1, 1, 1, 1)), -127, 127).to(torch.int8)
    w_tm = q_w.reshape(Co, V, Ci).permute(1, 0, 2).contiguous()
    b = bias.detach().float().contiguous() if bias is not None else torch.zeros(Co, device=feats.device)
    out = ops.spconv_i8(q_in, neighbor_cache.nmap_tm, neighbor_cache.tile_mask, w_tm, s_w.contiguous(), b, s_a,
                        ops.EPI_F32, rows=feats.shape[0])
    return out.to(feats.dtype), neighbor_cache


def sparse_pool(feats: Tensor, coords: Tensor, shape: torch.Size, kernel_size, stride=None, padding=None,
                reduce: str = "mean", output_coords: Tensor | None = None, output_shape: torch.Size | None = None,
                neighbor_cache: NeighborCache | None = None) -> tuple[Tensor, Tensor, torch.Size, NeighborCache]:
    D = len(kernel_size)
    stride = tuple(stride) if stride is not None else tuple(kernel_size)
    padding = tuple(padding) if padding is not None else (0,) * D
    sparse_dim = coords.shape[1]
    sparse_in = tuple(shape[:sparse_dim])
    sparse_out = tuple(output_shape[:sparse_dim]) if output_shape is not None else None
    if neighbor_cache is None:
        neighbor_cache = build_pool_cache(coords, sparse_in, kernel_size, stride, padding, output_coords, sparse_out)
    if reduce not in ("mean", "sum"):
        raise NotImplementedError(f"reduce={reduce!r} not needed by MoGe")
    _require_cuda(feats, "feats")
    _no_grad_check(feats)
    out_coords = neighbor_cache.output_coords
    n_out = int(out_coords.shape[0])
    seg32 = neighbor_cache.seg_offsets32
    if seg32 is None:
        seg32 = neighbor_cache.seg_offsets.to(torch.int32)
    x = feats.detach().float().contiguous()
    if reduce == "mean":
        acc = ops.pool_mean(x, neighbor_cache.seg_indices, seg32, n_out)
    else:
        acc = ops.pool_sum(x, neighbor_cache.seg_indices, seg32, n_out)
    out_shape = torch.Size([*neighbor_cache.output_sparse_shape, feats.shape[1]])
    return acc.to(feats.dtype), out_coords, out_shape, neighbor_cache


def sparse_upsample(feats: Tensor, coords: Tensor, shape: torch.Size, scale_factor, *, mode: str = "nearest",
                    output_coords: Tensor | None = None, output_shape: torch.Size | None = None,
                    neighbor_cache: NeighborCacheT | None = None, **_ignored) -> tuple[Tensor, Tensor, torch.Size, Any]:
    assert mode == "nearest", "MoGe only uses nearest upsampling"
    assert neighbor_cache is not None and neighbor_cache.is_transposed, (
        "reference path requires the transposed pool cache (MoGe always supplies it)")
    assert output_coords is not None
    parent = neighbor_cache.parent
    assert parent.shape[0] == output_coords.shape[0]
    _require_cuda(feats, "feats")
    _no_grad_check(feats)
    out = ops.gather_rows(feats.detach().float().contiguous(), parent, rows=int(parent.shape[0]))
    out_shape = torch.Size([*tuple(output_shape[: output_coords.shape[1]]), feats.shape[1]])
    return out.to(feats.dtype), output_coords, out_shape, neighbor_cache
