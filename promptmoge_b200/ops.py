"""Op-level PyTorch wrappers over the C ABI (device tensors in, device tensors out, current CUDA stream).

PyTorch only provides the device memory and the stream here; every computation is a kernel of libpmg_b200.so.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib
from ._lib import EPI_ACC32, EPI_F32, EPI_F32_RESID, EPI_SILU_Q8, FitState, call  # noqa: F401


def _stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def _p(t):
    return C.c_void_p(t.data_ptr()) if t is not None else None


def _dev(t: torch.Tensor, dtype=None, name="tensor"):
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (no CPU path)")
    if dtype is not None and t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    return t


# ----------------------------------------------------------------------------------------------------------------- #
# Structure
# ----------------------------------------------------------------------------------------------------------------- #
def voxelize_l0(point_coord: torch.Tensor, depth_resolution: float = 256.0, ld: int | None = None):
    """Level 0 of a point map [B,H,W,3]: (zq [N], zmin [B], zmax [B], nmap [27, ld], tile_mask)."""
    _dev(point_coord, torch.float32, "point_coord")
    B, H, W, _ = point_coord.shape
    N = B * H * W
    ld = ld or N
    dev = point_coord.device
    zq = torch.empty(N, dtype=torch.int32, device=dev)
    zmin = torch.full((B,), 0x7F7F7F7F, dtype=torch.int32, device=dev)
    zmax = torch.full((B,), -0x7F7F7F80, dtype=torch.int32, device=dev)
    nmap = torch.empty((27, ld), dtype=torch.int32, device=dev)
    mask = torch.zeros((ld + 31) // 32 + 1, dtype=torch.int32, device=dev)
    call("pmg_voxelize_l0", _p(point_coord), B, H, W, float(depth_resolution), _p(zq), _p(zmin), _p(zmax), _p(nmap),
         ld, _p(mask), _stream())
    return zq, zmin, zmax, nmap, mask


def l0_coords(zq, zmin, B, H, W):
    coords = torch.empty((B * H * W, 4), dtype=torch.int32, device=zq.device)
    call("pmg_l0_coords", _p(zq), _p(zmin), B, H, W, _p(coords), _stream())
    return coords


def pool_frames(B, Hf, Wf, fine_col_start, fine_z, zmin, cap, fine_count=None, with_coords=True, status=None):
    """One 2x2x2 pool transition of a frame grid.  Returns a dict with count (int32[2]: stored, required),
    z, col, col_start, coords, parent, seg_indices, seg_offsets (device tensors, capacity-sized)."""
    dev = fine_z.device
    Hc, Wc = (Hf + 1) // 2, (Wf + 1) // 2
    M_f = fine_z.shape[0]
    out = dict(
        count=torch.zeros(2, dtype=torch.int32, device=dev),
        z=torch.empty(cap, dtype=torch.int32, device=dev),
        col=torch.empty(cap, dtype=torch.int32, device=dev),
        col_start=torch.empty(B * Hc * Wc + 1, dtype=torch.int32, device=dev),
        coords=torch.empty((cap, 4), dtype=torch.int32, device=dev) if with_coords else None,
        parent=torch.empty(M_f, dtype=torch.int32, device=dev),
        seg_indices=torch.empty(M_f, dtype=torch.int32, device=dev),
        seg_offsets=torch.empty(cap + 1, dtype=torch.int32, device=dev),
    )
    nbytes = _lib.load().pmg_pool_frames_workspace_bytes(B, Hc, Wc)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    st = status if status is not None else torch.zeros(1, dtype=torch.int32, device=dev)
    call("pmg_pool_frames", B, Hf, Wf, _p(fine_count), _p(fine_col_start), _p(fine_z), _p(zmin), _p(out["count"]),
         _p(out["z"]), _p(out["col"]), _p(out["col_start"]), _p(out["coords"]), cap, _p(out["parent"]),
         _p(out["seg_indices"]), _p(out["seg_offsets"]), _p(ws), nbytes, _p(st), _stream())
    out["status"] = st
    return out


def nmap_frames(B, H, W, count, z, col, col_start, ld):
    dev = z.device
    nmap = torch.empty((27, ld), dtype=torch.int32, device=dev)
    mask = torch.zeros((ld + 31) // 32 + 1, dtype=torch.int32, device=dev)
    call("pmg_nmap_frames", B, H, W, _p(count), _p(z), _p(col), _p(col_start), _p(nmap), ld, _p(mask), _stream())
    return nmap, mask


def nmap_hash(coords: torch.Tensor, extents, row_major: bool = False, ld: int | None = None, status=None):
    """Generic neighbour map of coords [M,4] int32 within the sparse shape `extents` (4 ints)."""
    _dev(coords, torch.int32, "coords")
    M = coords.shape[0]
    dev = coords.device
    ld = ld or M
    nmap = torch.empty((M, 27) if row_major else (27, ld), dtype=torch.int32, device=dev)
    mask = torch.zeros((max(M, ld) + 31) // 32 + 1, dtype=torch.int32, device=dev)
    nbytes = _lib.load().pmg_nmap_hash_workspace_bytes(max(M, 1))
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    st = status if status is not None else torch.zeros(1, dtype=torch.int32, device=dev)
    ext = (C.c_int64 * 4)(*[int(e) for e in extents])
    call("pmg_nmap_hash", _p(coords), M, ext, _p(nmap), ld, int(row_major), _p(mask), _p(ws), nbytes, _p(st),
         _stream())
    return nmap, mask, st


# ----------------------------------------------------------------------------------------------------------------- #
# int8 layers
# ----------------------------------------------------------------------------------------------------------------- #
def _epi_out(mode, rows, n, dev):
    if mode == EPI_ACC32:
        return torch.empty((rows, n), dtype=torch.int32, device=dev)
    if mode == EPI_SILU_Q8:
        return torch.empty((rows, n), dtype=torch.int8, device=dev)
    return torch.empty((rows, n), dtype=torch.float32, device=dev)


FLAG_SIMT = 1


def tc_supported(Ci: int, Co: int) -> bool:
    """Shapes the tcgen05 path covers."""
    return Co in (32, 64, 128, 256) and (Ci in (32, 64) or (Ci >= 128 and Ci % 128 == 0))


def grid0_supported(Ci: int, Co: int) -> bool:
    """Widths the level-0 frame-grid tensor-core conv covers."""
    return Ci == Co and Ci in (32, 64)


def spconv_i8(q_in, nmap, tile_mask, weight_tap_major, w_scale=None, bias=None, act_scale=1.0, mode=EPI_ACC32,
              out_scale=1.0, resid=None, count=None, rows=None, tensor_cores=True, status=None, split: int = 1):
    """Submanifold conv: q_in [M_in, Ci] int8, nmap [27, ld] int32, weight [27, Co, Ci] int8.  The tcgen05 kernel
    runs where the shape allows unless tensor_cores is False; split > 1 allows split-K (up to `split` CTAs per output
    tile, same results)."""
    _dev(q_in, torch.int8, "q_in")
    _dev(weight_tap_major, torch.int8, "weight")
    ld = nmap.shape[1]
    rows = ld if rows is None else rows
    Co, Ci = weight_tap_major.shape[1], weight_tap_major.shape[2]
    out = _epi_out(mode, rows, Co, q_in.device)
    if split > 1 and tensor_cores:
        nbytes = _lib.load().pmg_spconv_i8_split_workspace_bytes(rows, Co, split)
        ws = torch.empty(nbytes, dtype=torch.uint8, device=q_in.device)
        call("pmg_spconv_i8_split", _p(q_in), q_in.shape[0], _p(nmap), ld, _p(tile_mask), _p(count), rows, Ci, Co,
             _p(weight_tap_major), _p(w_scale), _p(bias), float(act_scale), mode, float(out_scale), _p(resid),
             _p(out), int(split), _p(ws), nbytes, _p(status), _stream())
        return out
    call("pmg_spconv_i8", _p(q_in), q_in.shape[0], _p(nmap), ld, _p(tile_mask), _p(count), rows, Ci, Co,
         _p(weight_tap_major), _p(w_scale), _p(bias), float(act_scale), mode, float(out_scale), _p(resid), _p(out),
         0 if tensor_cores else FLAG_SIMT, _p(status), _stream())
    return out


def l0_tap_lanes(zq, B, H, W):
    """Per-tile tap masks of level 0 ([ceil(B*H*W/128), 27, 4] int32 view of the uint32 words) from zq."""
    _dev(zq, torch.int32, "zq")
    n = (B * H * W + 127) // 128
    lanes = torch.empty((n, 27, 4), dtype=torch.int32, device=zq.device)
    call("pmg_l0_tap_lanes", _p(zq), B, H, W, _p(lanes), _stream())
    return lanes


def spconv_i8_grid0(q_in, lanes, B, H, W, weight_tap_major, w_scale=None, bias=None, act_scale=1.0, mode=EPI_ACC32,
                    out_scale=1.0, resid=None, status=None):
    """Level-0 submanifold conv of a B x H x W frame grid (one voxel per pixel) without a neighbour map:
    q_in [B*H*W, C] int8, lanes from l0_tap_lanes, weight [27, C, C] int8, C in {32, 64}."""
    _dev(q_in, torch.int8, "q_in")
    _dev(lanes, torch.int32, "lanes")
    _dev(weight_tap_major, torch.int8, "weight")
    rows = B * H * W
    Co, Ci = weight_tap_major.shape[1], weight_tap_major.shape[2]
    out = _epi_out(mode, rows, Co, q_in.device)
    call("pmg_spconv_i8_grid0", _p(q_in), _p(lanes), B, H, W, Ci, Co, _p(weight_tap_major), _p(w_scale), _p(bias),
         float(act_scale), mode, float(out_scale), _p(resid), _p(out), _p(status), _stream())
    return out


def dense_i8(a, weight, w_scale=None, bias=None, act_scale=1.0, mode=EPI_ACC32, out_scale=1.0, resid=None,
             count=None, rows=None, tensor_cores=True, status=None):
    """Dense int8 layer: a [M, K] int8, weight [N, K] int8."""
    _dev(a, torch.int8, "a")
    _dev(weight, torch.int8, "weight")
    rows = a.shape[0] if rows is None else rows
    N, K = weight.shape
    out = _epi_out(mode, rows, N, a.device)
    call("pmg_dense_i8", _p(a), _p(count), rows, K, N, _p(weight), _p(w_scale), _p(bias), float(act_scale), mode,
         float(out_scale), _p(resid), _p(out), 0 if tensor_cores else FLAG_SIMT, _p(status), _stream())
    return out


def quantize(x, scale):
    _dev(x, torch.float32, "x")
    q = torch.empty(x.shape, dtype=torch.int8, device=x.device)
    call("pmg_quantize", _p(x), x.numel(), float(scale), _p(q), _stream())
    return q


def ln_silu_q8(x, gamma, beta, scale, eps=1e-6, up_src=None, parent=None, skip=None, count=None, rows=None):
    C_ = gamma.shape[0]
    ref = x if x is not None else skip
    rows = ref.shape[0] if rows is None else rows
    q = torch.empty((rows, C_), dtype=torch.int8, device=ref.device)
    x_out = torch.empty((rows, C_), dtype=torch.float32, device=ref.device) if up_src is not None else None
    call("pmg_ln_silu_q8", _p(x), _p(up_src), _p(parent), _p(skip), _p(x_out), _p(count), rows, C_, _p(gamma),
         _p(beta), float(eps), float(scale), _p(q), _stream())
    return (q, x_out) if up_src is not None else q


def frame_csr(coords, B, H, W, Z, status=None):
    """Column CSR (col_start [B*H*W+1], z [M]) of coords [M,4] sorted by (column, z)."""
    _dev(coords, torch.int32, "coords")
    M = coords.shape[0]
    dev = coords.device
    col_start = torch.empty(B * H * W + 1, dtype=torch.int32, device=dev)
    z = torch.empty(max(M, 1), dtype=torch.int32, device=dev)
    st = status if status is not None else torch.zeros(1, dtype=torch.int32, device=dev)
    call("pmg_frame_csr", _p(coords), M, B, H, W, int(Z), _p(col_start), _p(z), _p(st), _stream())
    return col_start, z[:M], st


def pool_sum(x, seg_indices, seg_offsets, rows, count=None):
    C_ = x.shape[1]
    out = torch.empty((rows, C_), dtype=torch.float32, device=x.device)
    call("pmg_pool_sum_f32", _p(x), _p(seg_indices), _p(seg_offsets), _p(count), rows, C_, _p(out), _stream())
    return out


def pool_mean(x, seg_indices, seg_offsets, rows, scale=None, count=None):
    C_ = x.shape[1]
    if scale is None:
        out = torch.empty((rows, C_), dtype=torch.float32, device=x.device)
        call("pmg_pool_mean_f32", _p(x), _p(seg_indices), _p(seg_offsets), _p(count), rows, C_, _p(out), _stream())
    else:
        out = torch.empty((rows, C_), dtype=torch.int8, device=x.device)
        call("pmg_pool_mean_q8", _p(x), _p(seg_indices), _p(seg_offsets), _p(count), rows, C_, float(scale), _p(out),
             _stream())
    return out


def gather_rows(x, parent, rows=None, count=None):
    _dev(x, torch.float32, "x")
    rows = parent.shape[0] if rows is None else rows
    out = torch.empty((rows, x.shape[1]), dtype=torch.float32, device=x.device)
    call("pmg_gather_rows_f32", _p(x), _p(parent), _p(count), rows, x.shape[1], _p(out), _stream())
    return out


def spconv_f32(x, nmap, tile_mask, weight_tap_major, bias=None, rows=None, count=None):
    _dev(x, torch.float32, "x")
    _dev(weight_tap_major, torch.float32, "weight")
    ld = nmap.shape[1]
    rows = ld if rows is None else rows
    Co, Ci = weight_tap_major.shape[1], weight_tap_major.shape[2]
    out = torch.empty((rows, Co), dtype=torch.float32, device=x.device)
    call("pmg_spconv_f32", _p(x), _p(nmap), ld, _p(tile_mask), _p(count), rows, Ci, Co, _p(weight_tap_major),
         _p(bias), _p(out), _stream())
    return out


# ----------------------------------------------------------------------------------------------------------------- #
# Fit
# ----------------------------------------------------------------------------------------------------------------- #
def _fit_state(B, dev):
    return torch.zeros((B, 18), dtype=torch.int32, device=dev)   # 72 bytes per frame (pmg_fit_state)


def fit_state_view(state: torch.Tensor):
    """Host copy of device fit states -> list of dicts."""
    raw = state.cpu().numpy().tobytes()
    n = len(raw) // C.sizeof(FitState)
    arr = (FitState * n).from_buffer_copy(raw)
    return [dict(s=a.s, t=a.t, thr=a.thr, count=a.count, k=a.k, ok=a.ok, sums=list(a.sums)) for a in arr]


def fit_solve(z, target, flags, iters=4, trim=0.2, min_points=32):
    B, N = z.shape
    dev = z.device
    st = _fit_state(B, dev)
    nbytes = _lib.load().pmg_fit_workspace_bytes(B, N)
    ws = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
    call("pmg_fit_solve", _p(z), _p(target), _p(flags), B, N, iters, float(trim), min_points, _p(st), _p(ws), nbytes,
         _stream())
    return st


def fit_prep_prompt(logz, lidar, conf):
    """logz [B,H,W] (contiguous) or a point map [B,H,W,3] (logz read with stride 3)."""
    if logz.dim() == 4:
        base, stride = logz[..., 2], 3
        ptr = C.c_void_p(logz.data_ptr() + 8)
        B, H, W = logz.shape[:3]
    else:
        base, stride = logz, 1
        ptr = _p(logz)
        B, H, W = logz.shape
    h, w = lidar.shape[-2:]
    dev = logz.device
    N = B * H * W
    z = torch.empty((B, H * W), dtype=torch.float32, device=dev)
    y = torch.empty((B, H * W), dtype=torch.float32, device=dev)
    fl = torch.empty((B, H * W), dtype=torch.uint8, device=dev)
    del base
    call("pmg_fit_prep_prompt", ptr, stride, _p(lidar), _p(conf), B, H, W, h, w, _p(z), _p(y), _p(fl), _stream())
    return z, y, fl


def fit_prep_final(depth, lidar, conf, mask01=None):
    B, H, W = depth.shape
    h, w = lidar.shape[-2:]
    dev = depth.device
    z = torch.empty((B, h * w), dtype=torch.float32, device=dev)
    y = torch.empty((B, h * w), dtype=torch.float32, device=dev)
    fl = torch.empty((B, h * w), dtype=torch.uint8, device=dev)
    call("pmg_fit_prep_final", _p(depth), _p(mask01), _p(lidar), _p(conf), B, H, W, h, w, _p(z), _p(y), _p(fl),
         _stream())
    return z, y, fl


def fit_prompt_fused(logz, lidar, conf, soft_gate=True, iters=4, trim=0.2, min_points=32):
    """The one-launch per-step fit (pmg_fit_prompt_fused): (state [B,18] int32 view of pmg_fit_state, prompt
    features [B*H*W,2]) from logz [B,H,W] (contiguous or a point map's logz channel) and the LiDAR."""
    lz, st = _elem_strided(logz)
    B, H, W = logz.shape
    h, w = lidar.shape[-2:]
    state = _fit_state(B, logz.device)
    out = torch.empty((B * H * W, 2), dtype=torch.float32, device=logz.device)
    nbytes = _lib.load().pmg_fit_prompt_fused_workspace_bytes(B, H, W)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=logz.device)
    call("pmg_fit_prompt_fused", _p(lz), st, _p(lidar), _p(conf), B, H, W, h, w, iters, float(trim), min_points,
         int(soft_gate), _p(state), _p(out), None, None, _p(ws), nbytes, _stream())
    return state, out


def prompt_feats(logz, lidar, conf, state, soft_gate=True):
    B, H, W = logz.shape
    h, w = lidar.shape[-2:]
    out = torch.empty((B * H * W, 2), dtype=torch.float32, device=logz.device)
    call("pmg_prompt_feats", _p(logz), 1, _p(lidar), _p(conf), _p(state), B, H, W, h, w, int(soft_gate), _p(out),
         _stream())
    return out


def _elem_strided(t: torch.Tensor):
    """(tensor, element stride) for a [B,H,W] tensor whose elements sit at a constant stride (a contiguous map, or
    the logz channel of a contiguous [B,H,W,3] point map); anything else is copied to a contiguous tensor."""
    B, H, W = t.shape
    for st in (1, 3):
        if t.stride() == (H * W * st, W * st, st):
            return t, st
    return t.contiguous(), 1


def affine_frame(logz, lidar, conf, state, soft_gate=True):
    """(log_d_aff [B,H,W], gate [B,H,W]) of MoGeModel._lidar_in_affine_frame (moge/model/v3.py:362-383) from a solved
    fit state."""
    B, H, W = logz.shape
    h, w = lidar.shape[-2:]
    lz, st = _elem_strided(logz)
    log_d_aff = torch.empty((B, H, W), dtype=torch.float32, device=logz.device)
    gate = torch.empty((B, H, W), dtype=torch.float32, device=logz.device)
    call("pmg_affine_frame", _p(lz), st, _p(lidar), _p(conf), _p(state), B, H, W, h, w, int(soft_gate), _p(log_d_aff),
         _p(gate), _stream())
    return log_d_aff, gate


def lidar_in_affine_frame(logz, lidar, conf, soft_gate=False, iters=4, trim=0.2, min_points=32, fused=True):
    """MoGeModel._lidar_in_affine_frame (moge/model/v3.py:362-383) on the device: the trimmed least-squares fit of the
    nearest-resized confident LiDAR to exp(logz) (prompt_stem.fit_scale_shift, prompt_stem.py:211-240), then the
    LiDAR in the affine log-depth frame.  logz [B,H,W] fp32 (a strided view of a point map's logz channel is read in
    place), lidar / conf [B,1,h,w] fp32.  Returns (log_d_aff [B,H,W], gate [B,H,W], s [B], t [B]).  fused: one
    cluster launch per frame (pmg_fit_prompt_fused) where the frame size allows, else the multi-launch kernels."""
    if not logz.is_cuda or logz.dtype != torch.float32:
        raise ValueError("logz must be a float32 CUDA tensor (no CPU path)")
    _dev(lidar, torch.float32, "lidar")
    _dev(conf, torch.float32, "conf")
    lz, st = _elem_strided(logz)
    B, H, W = logz.shape
    h, w = lidar.shape[-2:]
    dev = logz.device
    if fused:
        state = _fit_state(B, dev)
        log_d_aff = torch.empty((B, H, W), dtype=torch.float32, device=dev)
        gate = torch.empty((B, H, W), dtype=torch.float32, device=dev)
        nbytes = _lib.load().pmg_fit_prompt_fused_workspace_bytes(B, H, W)
        ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        rc = _lib.load().pmg_fit_prompt_fused(_p(lz), st, _p(lidar), _p(conf), B, H, W, h, w, iters, float(trim),
                                               min_points, int(soft_gate), _p(state), None, _p(log_d_aff), _p(gate),
                                               _p(ws), nbytes, _stream())
        if rc == 0:
            sv = state.view(torch.float32)[:, :2]
            return log_d_aff, gate, sv[:, 0].clone(), sv[:, 1].clone()
        if rc != 5:          # PMG_ERR_UNSUPPORTED: this frame size / device takes the multi-launch fit below
            raise _lib.PmgError("pmg_fit_prompt_fused", rc)
    z = torch.empty((B, H * W), dtype=torch.float32, device=dev)
    y = torch.empty((B, H * W), dtype=torch.float32, device=dev)
    fl = torch.empty((B, H * W), dtype=torch.uint8, device=dev)
    call("pmg_fit_prep_prompt", _p(lz), st, _p(lidar), _p(conf), B, H, W, h, w, _p(z), _p(y), _p(fl), _stream())
    state = fit_solve(z, y, fl, iters, trim, min_points)
    log_d_aff, gate = affine_frame(logz, lidar, conf, state, soft_gate)
    sv = state.view(torch.float32)[:, :2]       # pmg_fit_state starts with (s, t) fp32
    return log_d_aff, gate, sv[:, 0].clone(), sv[:, 1].clone()


def apply_affine(depth, state):
    B = depth.shape[0]
    call("pmg_apply_affine", _p(depth), _p(state), B, depth[0].numel(), _stream())
    return depth


# ----------------------------------------------------------------------------------------------------------------- #
# Polynomial prompt gauge
# ----------------------------------------------------------------------------------------------------------------- #
def gauge_poly(depth, lidar, conf=None, degree: int = 2, iters: int = 3, points=None, in_place: bool = False):
    """Per-frame gauge of depth [B,H,W] to lidar [B,h,w] (conf [B,h,w] or None).  Returns (corr [B,H,W],
    corrected depth [B,H,W] (depth itself when in_place), coef [B,8] = 6 coefficients, ok, count); points
    [B,H,W,3], when given, is multiplied by corr in place."""
    _dev(depth, torch.float32, "depth")
    _dev(lidar, torch.float32, "lidar")
    B, H, W = depth.shape
    h, w = lidar.shape[-2:]
    dev = depth.device
    corr = torch.empty((B, H, W), dtype=torch.float32, device=dev)
    out = depth if in_place else torch.empty_like(depth)
    coef = torch.empty((B, 8), dtype=torch.float32, device=dev)
    nbytes = _lib.load().pmg_gauge_workspace_bytes(B, h, w)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    call("pmg_gauge_poly", _p(depth), _p(lidar.contiguous()), _p(conf.contiguous() if conf is not None else None), B,
         H, W, h, w, degree, iters, _p(corr), _p(out), _p(points), _p(coef), _p(ws), nbytes, _stream())
    return corr, out, coef


# ----------------------------------------------------------------------------------------------------------------- #
# LiDAR prompt preparation
# ----------------------------------------------------------------------------------------------------------------- #
def _frames(t: torch.Tensor, name: str):
    if t.dim() < 2:
        raise ValueError(f"{name} must be [..., h, w]")
    h, w = t.shape[-2:]
    return max(1, t.numel() // max(1, h * w)), h, w


def nearest_fill(depth: torch.Tensor, conf: torch.Tensor | None = None, out=None):
    """promptmoge.nearest_fill (promptmoge/model.py:61-72) on the GPU, per frame of [..., h, w] fp32 tensors: every
    missing pixel (depth <= 0 or NaN) takes the depth of its Euclidean-nearest present pixel and confidence 1.
    conf None means all-high (2), as promptmoge.infer does.  Returns (depth, conf) tensors of the input shape: new
    ones, or `out` = (depth_out, conf_out) (contiguous fp32, not aliasing the inputs)."""
    _dev(depth, torch.float32, "depth")
    if conf is None:
        conf = torch.full_like(depth, 2.0)
    _dev(conf, torch.float32, "conf")
    if conf.shape != depth.shape:
        raise ValueError("conf must have depth's shape")
    B, h, w = _frames(depth, "depth")
    if out is None:
        d_out, c_out = torch.empty_like(depth), torch.empty_like(conf)
    else:
        d_out, c_out = _dev(out[0], torch.float32, "depth_out"), _dev(out[1], torch.float32, "conf_out")
        if d_out.shape != depth.shape or c_out.shape != depth.shape:
            raise ValueError("out tensors must have depth's shape")
    if depth.numel() == 0:
        return d_out, c_out
    nbytes = _lib.load().pmg_prompt_workspace_bytes(B, h, w)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=depth.device)
    call("pmg_nearest_fill", _p(depth), _p(conf), B, h, w, _p(d_out), _p(c_out), _p(ws), nbytes, _stream())
    return d_out, c_out


def build_prompt(depth: torch.Tensor, conf: torch.Tensor, out_hw, conf_levels: float = 2.0, mono_z=None,
                 prefill=None, conf_phase: bool = False):
    """build_prompt (moge/model/modules/prompt_stem.py:45-105) on the GPU: depth, conf [B,1,h,w] fp32 -> (prompt
    [B,4,H,W] fp32, {"mu": [B]}).  The optional mono / prefill / phase channels are not part of the deployed
    4-channel prompt and are not implemented here."""
    if mono_z is not None or prefill is not None or conf_phase:
        raise NotImplementedError("only the 4-channel prompt (no mono_z / prefill / conf_phase) is implemented")
    depth = _dev(depth.float().contiguous(), torch.float32, "depth")
    conf = _dev(conf.float().contiguous(), torch.float32, "conf")
    if depth.dim() != 4 or depth.shape[1] != 1 or conf.shape != depth.shape:
        raise ValueError("depth and conf must be [B,1,h,w]")
    B, _, h, w = depth.shape
    H, W = int(out_hw[0]), int(out_hw[1])
    prompt = torch.empty((B, 4, H, W), dtype=torch.float32, device=depth.device)
    mu = torch.empty(B, dtype=torch.float32, device=depth.device)
    nbytes = _lib.load().pmg_prompt_workspace_bytes(B, h, w)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=depth.device)
    call("pmg_build_prompt", _p(depth), _p(conf), B, h, w, H, W, float(conf_levels), _p(prompt), _p(mu), _p(ws),
         nbytes, _stream())
    return prompt, {"mu": mu}


# ----------------------------------------------------------------------------------------------------------------- #
# Optional refiner-side gates (moge/model/v3.py:565-573)
# ----------------------------------------------------------------------------------------------------------------- #
def output_gate(cur_logz, refined_logz, lidar, conf, floor: float = 0.1):
    """cur + g (refined - cur), g = floor + (1 - floor) u (the refiner output gate).  logz [B,H,W]."""
    cur = _dev(cur_logz.contiguous(), torch.float32, "cur_logz")
    ref = _dev(refined_logz.contiguous(), torch.float32, "refined_logz")
    out = torch.empty_like(ref)
    B, H, W = ref.shape
    h, w = lidar.shape[-2:]
    call("pmg_output_gate", _p(cur), _p(ref), _p(out), 1, _p(lidar.contiguous()), _p(conf.contiguous()), B, H, W, h,
         w, float(floor), _stream())
    return out


def anchor(logz, lidar, conf, beta: float, iters: int = 4, trim: float = 0.2, min_points: int = 32):
    """The elastic anchor: a fresh _lidar_in_affine_frame fit of logz, then logz + beta gate (log d_aff - logz)."""
    lz = _dev(logz.contiguous(), torch.float32, "logz")
    z, y, fl = fit_prep_prompt(lz, lidar.contiguous(), conf.contiguous())
    st = fit_solve(z, y, fl, iters=iters, trim=trim, min_points=min_points)
    out = lz.clone()
    B, H, W = lz.shape
    h, w = lidar.shape[-2:]
    call("pmg_anchor_apply", _p(out), 1, _p(lidar.contiguous()), _p(conf.contiguous()), _p(st), B, H, W, h, w,
         float(beta), _stream())
    return out
