"""Post-refinement output of MoGeModel.infer on the device, with the reference's function names and arguments:

  recover_focal_shift(points, mask=None, focal=None, downsample_size=(64, 64))   moge/utils/geometry_torch.py:118-170
  normalized_view_plane_uv(width, height, aspect_ratio=None)                      moge/utils/geometry_torch.py:43-55
  postprocess(coords, image_hw, lidar_depth, lidar_conf=None, mask=None, fov_x=None, gauge_poly=2, apply_mask=True)
      the output path of infer(metric_from='lidar_ls') after the refine loop (v3.py:580-604, 739-832, 841-846):
      bilinear resize + 'exp' remap of the refined map, focal / shift recovery, shifted depth, the final robust
      LiDAR fit, the point map from depth and intrinsics, the mask (+inf), the polynomial gauge.

Every step runs as a CUDA kernel of libpmg_b200 on the current stream; nothing is copied to the host (the reference
moves the 64 x 64 samples to the CPU for scipy's least squares).  The trained model's optional ``prompt_calib``
rescale of the fit (v3.py:775-776) and the calibration LUT are model-specific and not part of this path.
"""
from __future__ import annotations

import torch

from . import ops
from ._lib import call


def _p(t):
    return ops._p(t)


def normalized_view_plane_uv(width: int, height: int, aspect_ratio: float | None = None, device="cuda"):
    """[H, W, 2] fp32 view-plane uv grid (torch.linspace, fused multiply-add form) -- built here with torch for
    callers that want it; the kernels compute the same values inline."""
    a = width / height if aspect_ratio is None else aspect_ratio
    sx, sy = a / (1 + a ** 2) ** 0.5, 1 / (1 + a ** 2) ** 0.5
    u = torch.linspace(-sx * (width - 1) / width, sx * (width - 1) / width, width, dtype=torch.float32, device=device)
    v = torch.linspace(-sy * (height - 1) / height, sy * (height - 1) / height, height, dtype=torch.float32,
                       device=device)
    uu, vv = torch.meshgrid(u, v, indexing="xy")
    return torch.stack([uu, vv], dim=-1)


def resize_remap(coords: torch.Tensor, image_hw) -> torch.Tensor:
    """coords [B,h,w,3] (x/z, y/z, log z) -> affine points [B,H,W,3] (bilinear resize, 'exp' remap)."""
    coords = ops._dev(coords.float().contiguous(), torch.float32, "coords")
    B, h, w, _ = coords.shape
    H, W = int(image_hw[0]), int(image_hw[1])
    out = torch.empty((B, H, W, 3), dtype=torch.float32, device=coords.device)
    call("pmg_resize_remap", _p(coords), B, h, w, H, W, _p(out), ops._stream())
    return out


def recover_focal_shift(points: torch.Tensor, mask: torch.Tensor | None = None, focal: torch.Tensor | None = None,
                        downsample_size=(64, 64)):
    """points [..., H, W, 3] -> (focal [...], shift [...]) fp32 on the device."""
    shape = points.shape
    H, W = shape[-3], shape[-2]
    pts = ops._dev(points.reshape(-1, H, W, 3).float().contiguous(), torch.float32, "points")
    B = pts.shape[0]
    mk = None
    if mask is not None:
        mk = ops._dev(mask.reshape(B, H, W).to(torch.uint8).contiguous(), torch.uint8, "mask")
    fin = None
    if focal is not None:
        fin = ops._dev(torch.as_tensor(focal, device=pts.device).reshape(B).float().contiguous(), torch.float32,
                       "focal")
    fo = torch.empty(B, dtype=torch.float32, device=pts.device)
    sh = torch.empty(B, dtype=torch.float32, device=pts.device)
    call("pmg_focal_shift", _p(pts), _p(mk), _p(fin), B, H, W, int(downsample_size[0]), int(downsample_size[1]),
         _p(fo), _p(sh), ops._stream())
    return fo.reshape(shape[:-3]), sh.reshape(shape[:-3])


def intrinsics_from_focal(focal: torch.Tensor, width: int, height: int) -> torch.Tensor:
    """[B,3,3] normalised intrinsics of infer (v3.py:741-742): fx = f/2 sqrt(1+a^2)/a, fy = f/2 sqrt(1+a^2), centre
    (0.5, 0.5)."""
    a = width / height
    fy = focal / 2 * (1 + a ** 2) ** 0.5
    fx = fy / a
    K = torch.zeros(focal.shape + (3, 3), dtype=torch.float32, device=focal.device)
    K[..., 0, 0], K[..., 1, 1] = fx, fy
    K[..., 0, 2], K[..., 1, 2], K[..., 2, 2] = 0.5, 0.5, 1.0
    return K


def postprocess(coords: torch.Tensor, image_hw, lidar_depth: torch.Tensor, lidar_conf: torch.Tensor | None = None,
                mask: torch.Tensor | None = None, fov_x=None, gauge_poly: int = 2, apply_mask: bool = True,
                fit_iters: int = 4, fit_trim: float = 0.2, fit_min_points: int = 32) -> dict:
    """The refined map coords [B,h,w,3] -> dict(points [B,H,W,3], depth [B,H,W], intrinsics [B,3,3], mask [B,H,W] or
    None, metric_fit [B,2] (s, t), focal [B], shift [B]) as infer(metric_from='lidar_ls') returns them.
    lidar_depth / lidar_conf [B,1,h',w'] fp32 (conf None = all 2); mask [B,H,W] bool (the mask head's > 0.5)."""
    H, W = int(image_hw[0]), int(image_hw[1])
    pts = resize_remap(coords, (H, W))
    B = pts.shape[0]
    dev = pts.device
    ld = ops._dev(lidar_depth.float().contiguous(), torch.float32, "lidar_depth")
    lc = torch.full_like(ld, 2.0) if lidar_conf is None else ops._dev(lidar_conf.float().contiguous(),
                                                                      torch.float32, "lidar_conf")
    focal_fixed = None
    if fov_x is not None:
        a = W / H
        fov = torch.as_tensor(fov_x, dtype=torch.float32, device=dev)
        focal_fixed = (a / (1 + a ** 2) ** 0.5 / torch.tan(torch.deg2rad(fov) / 2)).float().expand(B).contiguous()
    focal, shift = recover_focal_shift(pts, mask, focal_fixed)
    depth = torch.empty((B, H, W), dtype=torch.float32, device=dev)
    call("pmg_shift_depth", _p(pts), _p(shift), B, H, W, _p(depth), ops._stream())
    m01 = mask.float().contiguous() if mask is not None else None
    z, y, fl = ops.fit_prep_final(depth, ld, lc, m01)
    st = ops.fit_solve(z, y, fl, iters=fit_iters, trim=fit_trim, min_points=fit_min_points)
    ops.apply_affine(depth, st)
    fs = st.view(torch.float32)[:, :2].clone()          # pmg_fit_state starts with float s, t
    mask_out = None
    if mask is not None:
        mask_out = mask.to(torch.bool) & (depth > 0)
    mk = mask_out.to(torch.uint8).contiguous() if (mask_out is not None and apply_mask) else None
    points = torch.empty((B, H, W, 3), dtype=torch.float32, device=dev)
    call("pmg_depth_to_points", _p(depth), _p(focal), B, H, W, _p(mk), _p(points), _p(depth), ops._stream())
    if gauge_poly > 0:
        ops.gauge_poly(depth, ld.reshape(B, *ld.shape[-2:]).contiguous(), lc.reshape(B, *lc.shape[-2:]).contiguous(),
                       degree=gauge_poly, points=points, in_place=True)
    return {"points": points, "depth": depth, "intrinsics": intrinsics_from_focal(focal, W, H), "mask": mask_out,
            "metric_fit": fs, "focal": focal, "shift": shift}


__all__ = ["normalized_view_plane_uv", "resize_remap", "recover_focal_shift", "intrinsics_from_focal", "postprocess"]


class PostGraph:
    """postprocess captured once into a CUDA graph for fixed shapes (one launch per frame batch instead of a dozen
    kernel launches and allocations from Python); run() copies the inputs into the graph's static buffers and
    replays it.  The returned tensors are the graph's static outputs (overwritten by the next run)."""

    def __init__(self, batch: int, coords_hw, image_hw, lidar_hw=(192, 256), masked: bool = False,
                 gauge_poly: int = 2, device="cuda"):
        dev = torch.device(device)
        h, w = coords_hw
        lh, lw = lidar_hw
        self.coords = torch.zeros((batch, h, w, 3), dtype=torch.float32, device=dev)
        self.lidar = torch.ones((batch, 1, lh, lw), dtype=torch.float32, device=dev)
        self.conf = torch.full((batch, 1, lh, lw), 2.0, dtype=torch.float32, device=dev)
        self.mask = torch.ones((batch, image_hw[0], image_hw[1]), dtype=torch.bool, device=dev) if masked else None
        self.image_hw = tuple(image_hw)
        self.gauge_poly = gauge_poly
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            self._run()                                   # warm-up: attributes set, allocator primed
        torch.cuda.current_stream(dev).wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.out = self._run()

    def _run(self):
        return postprocess(self.coords, self.image_hw, self.lidar, self.conf, self.mask, gauge_poly=self.gauge_poly)

    def run(self, coords, lidar_depth, lidar_conf, mask=None) -> dict:
        self.coords.copy_(coords, non_blocking=True)
        self.lidar.copy_(lidar_depth, non_blocking=True)
        self.conf.copy_(lidar_conf, non_blocking=True)
        if self.mask is not None:
            self.mask.copy_(mask, non_blocking=True)
        self.graph.replay()
        return self.out
