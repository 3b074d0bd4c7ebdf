"""Oracle (test infrastructure): voxelisation, voxel dedup (pool cache) and neighbour maps in numpy.

Each function restates one reference function of PromptMoGe's bundled FlexGEMM fallback
(promptmoge/_fallback/flex_gemm/_core.py) or of moge/model/v3.py, with the same outputs and index conventions.
"""
from __future__ import annotations

import itertools

import numpy as np


def kernel_delta() -> np.ndarray:
    """[27, 4] int32 offsets (0, di, dj, dz), last dim fastest: tap v = (di+1)*9 + (dj+1)*3 + (dz+1).

    Follows make_conv_kernel_delta, _core.py:65-82 (itertools.product over range(-1, 2) per spatial dim, one batch
    dim of 0)."""
    return np.array([(0, a, b, c) for a, b, c in itertools.product(range(-1, 2), repeat=3)], dtype=np.int32)


def voxelize(point_coord: np.ndarray, res: float = 256.0):
    """MoGeModel._voxelize, moge/model/v3.py:305-344.

    point_coord [B, H, W, 3] fp32 (x/z, y/z, logz) -> feats [M, 3] fp32, coords [M, 4] int32 (b, i, j, z),
    shape (B, H, W, Z, 3), logz [B, H, W].  zq = round(logz * res) half-to-even in fp32, z = zq - per-frame min,
    Z = global max + 1 (v3.py:331-335)."""
    pc = np.asarray(point_coord, dtype=np.float32)
    B, H, W, _ = pc.shape
    logz = pc[..., 2]
    zq = np.rint(logz * np.float32(res)).astype(np.int64)
    z = zq - zq.min(axis=(1, 2), keepdims=True)
    Z = int(z.max()) + 1
    b = np.broadcast_to(np.arange(B).reshape(B, 1, 1), (B, H, W))
    i = np.broadcast_to(np.arange(H).reshape(1, H, 1), (B, H, W))
    j = np.broadcast_to(np.arange(W).reshape(1, 1, W), (B, H, W))
    coords = np.stack([b, i, j, z], axis=-1).reshape(-1, 4).astype(np.int32)
    return pc.reshape(-1, 3), coords, (B, H, W, Z, 3), logz


def linearise(coords: np.ndarray, sparse_shape) -> np.ndarray:
    """_linearise, _core.py:89-94: row-major int64 keys over sparse_shape."""
    key = np.zeros(coords.shape[0], dtype=np.int64)
    for d, extent in enumerate(sparse_shape):
        key = key * np.int64(extent) + coords[:, d].astype(np.int64)
    return key


def _in_bounds(coords, sparse_shape):
    """_in_bounds, _core.py:97-102."""
    ok = np.ones(coords.shape[0], dtype=bool)
    for d, extent in enumerate(sparse_shape):
        c = coords[:, d]
        ok &= (c >= 0) & (c < int(extent))
    return ok


def nmap_column(coords: np.ndarray, sparse_shape) -> np.ndarray:
    """Level-0 "column" backend, _core.py:269-295: one voxel per (b, i, j); the voxel at (b, i+di, j+dj) is the
    neighbour at tap (di, dj, dz) iff z[i+di, j+dj] == z[i, j] + dz.  Returns [M, 27] int32, -1 = absent."""
    B, H, W = (int(s) for s in sparse_shape[:3])
    z = coords[:, 3].astype(np.int64).reshape(B, H, W)
    flat = np.arange(B * H * W, dtype=np.int32).reshape(B, H, W)
    nmap = np.full((B, H, W, 27), -1, dtype=np.int32)
    NEG = np.iinfo(np.int64).min // 4
    for v, (_, di, dj, dz) in enumerate(kernel_delta()):
        zs = np.full_like(z, NEG)
        fs = np.full_like(flat, -1)
        si0, si1 = max(0, -di), min(H, H - di)
        ti0, ti1 = max(0, di), min(H, H + di)
        sj0, sj1 = max(0, -dj), min(W, W - dj)
        tj0, tj1 = max(0, dj), min(W, W + dj)
        if si1 > si0 and sj1 > sj0:
            zs[:, si0:si1, sj0:sj1] = z[:, ti0:ti1, tj0:tj1]
            fs[:, si0:si1, sj0:sj1] = flat[:, ti0:ti1, tj0:tj1]
        hit = zs == (z + dz)
        nmap[..., v] = np.where(hit, fs, -1)
    return nmap.reshape(B * H * W, 27)


def nmap_sorted(coords: np.ndarray, sparse_shape) -> np.ndarray:
    """Generic "sorted" backend, _core.py:105-124 (_SortedIndex) and :298-304: sort the linearised keys, look each of
    the 27 shifted coords up with searchsorted, out-of-bounds -> -1.  Returns [M, 27] int32."""
    keys = linearise(coords, sparse_shape)
    order = np.argsort(keys, kind="stable")
    skeys = keys[order]
    n = keys.shape[0]
    nmap = np.empty((coords.shape[0], 27), dtype=np.int32)
    for v, delta in enumerate(kernel_delta()):
        q = coords.astype(np.int64) + delta.astype(np.int64)
        ok = _in_bounds(q, sparse_shape)
        qk = np.where(ok, linearise(q, sparse_shape), -1)
        pos = np.searchsorted(skeys, qk)
        pos_c = np.minimum(pos, n - 1)
        hit = ok & (skeys[pos_c] == qk) & (pos < n)
        nmap[:, v] = np.where(hit, order[pos_c], -1).astype(np.int32)
    return nmap


def is_one_voxel_per_column(coords: np.ndarray, sparse_shape) -> bool:
    """_is_one_voxel_per_column, _core.py:249-266."""
    B, H, W = (int(s) for s in sparse_shape[:3])
    if coords.shape[0] != B * H * W or coords.shape[1] != 4:
        return False
    g = np.stack(np.meshgrid(np.arange(B), np.arange(H), np.arange(W), indexing="ij"), -1).reshape(-1, 3)
    return bool(np.array_equal(coords[:, :3], g))


def submanifold_nmap(coords: np.ndarray, sparse_shape) -> np.ndarray:
    """build_submanifold_cache's backend choice, _core.py:307-336 ("auto": column when one voxel per column)."""
    if is_one_voxel_per_column(coords, sparse_shape):
        return nmap_column(coords, sparse_shape)
    return nmap_sorted(coords, sparse_shape)


def pool(coords: np.ndarray, sparse_shape, factor: int = 2):
    """Perfect-partition pool cache = the voxel dedup, build_pool_cache _core.py:339-392 (output_coords=None) with
    the output shape of flex_sparse_blocks._ceil_downsample_shape (:40-46).

    Returns (out_coords [Mo, 4] int32, out_shape, parent [M] int32, seg_indices [M] int32, seg_offsets [Mo+1] int64).
    out_coords are the unique floor(coords / f) in sorted-key (lexicographic) order, parent = rank of each input's
    key among them, seg_indices = argsort(parent, stable), seg_offsets = prefix sums of the child counts."""
    div = np.array([1, factor, factor, factor], dtype=np.int64)
    down = np.floor_divide(coords.astype(np.int64), div)
    out_shape = tuple([int(sparse_shape[0])] + [-(-int(s) // factor) for s in sparse_shape[1:4]])
    keys = linearise(down, out_shape)
    uniq, first, inverse = np.unique(keys, return_index=True, return_inverse=True)
    out_coords = down[first].astype(np.int32)
    seg_indices = np.argsort(inverse, kind="stable").astype(np.int32)
    counts = np.bincount(inverse, minlength=uniq.shape[0])
    seg_offsets = np.zeros(uniq.shape[0] + 1, dtype=np.int64)
    seg_offsets[1:] = np.cumsum(counts)
    return out_coords, out_shape, inverse.astype(np.int32), seg_indices, seg_offsets


def build_levels(coords0: np.ndarray, shape0, factors):
    """The U-Net's structure for one forward (sparse_unet.py:217-225 builds each level's conv cache on its first
    block and each k -> k+1 pool cache in PoolDown): per level coords / shape / nmap, per transition the pool cache."""
    levels = [dict(coords=coords0, shape=tuple(shape0[:4]), nmap=submanifold_nmap(coords0, shape0[:4]))]
    pools = []
    for f in factors:
        c, s = levels[-1]["coords"], levels[-1]["shape"]
        oc, osh, parent, seg_idx, seg_off = pool(c, s, f)
        pools.append(dict(parent=parent, seg_indices=seg_idx, seg_offsets=seg_off))
        levels.append(dict(coords=oc, shape=osh, nmap=submanifold_nmap(oc, osh)))
    return levels, pools
