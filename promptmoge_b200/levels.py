"""The refiner's voxel hierarchy of one forward, built on the device (voxelise -> per-level dedup + neighbour maps).

Returns the structures in the reference's own layout (coords [M,4] int32, nmap [M,27] int32, parent, seg_indices,
seg_offsets) next to the device-native ones (tap-major nmap, column CSR), so callers that need NeighborCache-like
objects and the fused runtime share one builder.
"""
from __future__ import annotations

import torch

from . import ops


def build_levels(point_coord: torch.Tensor, levels: int, depth_resolution: float = 256.0, with_coords: bool = True):
    """point_coord [B,H,W,3] fp32 on CUDA -> list of level dicts and list of pool dicts (exact counts)."""
    B, H, W, _ = point_coord.shape
    N = B * H * W
    zq, zmin, zmax, nmap0, mask0 = ops.voxelize_l0(point_coord, depth_resolution)
    lv = [dict(count=N, H=H, W=W, z=zq, zmin=zmin, zmax=zmax, nmap_tm=nmap0, mask=mask0, col_start=None,
               coords=ops.l0_coords(zq, zmin, B, H, W) if with_coords else None)]
    pools = []
    status = torch.zeros(1, dtype=torch.int32, device=point_coord.device)
    for k in range(levels - 1):
        f = lv[-1]
        cap = f["count"]
        p = ops.pool_frames(B, f["H"], f["W"], f["col_start"], f["z"], zmin if k == 0 else None, cap,
                            with_coords=with_coords, status=status)
        M = int(p["count"][0])
        Hc, Wc = (f["H"] + 1) // 2, (f["W"] + 1) // 2
        nmap, mask = ops.nmap_frames(B, Hc, Wc, p["count"], p["z"], p["col"], p["col_start"], cap)
        pools.append(dict(parent=p["parent"][: f["count"]], seg_indices=p["seg_indices"][: f["count"]],
                          seg_offsets=p["seg_offsets"][: M + 1]))
        lv.append(dict(count=M, H=Hc, W=Wc, z=p["z"][:M], col=p["col"][:M], col_start=p["col_start"], nmap_tm=nmap,
                       mask=mask, coords=p["coords"][:M] if with_coords else None, count_dev=p["count"]))
    if int(status.item()) != 0:
        raise RuntimeError(f"level build failed with device status {int(status.item())}")
    for l in lv:
        l["nmap"] = l["nmap_tm"][:, : l["count"]].t()
    return lv, pools
