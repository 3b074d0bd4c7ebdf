"""ctypes binding of the C ABI in include/pmg_b200.h (libpmg_b200.so, built in-tree by promptmoge_b200.build).

There is no fallback: if the library is missing or was built for another architecture, importing the ops raises.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "libpmg_b200.so"

P = C.c_void_p
I32 = C.c_int32
I64 = C.c_int64
F32 = C.c_float
SZ = C.c_size_t


class FitState(C.Structure):
    """pmg_fit_state (72 bytes)."""
    _fields_ = [("s", C.c_float), ("t", C.c_float), ("thr", C.c_float), ("count", C.c_int32), ("k", C.c_int32),
                ("ok", C.c_int32), ("prefix", C.c_uint32), ("remaining", C.c_int32), ("sums", C.c_double * 5)]


class RefinerConfig(C.Structure):
    _fields_ = [("batch", I32), ("height", I32), ("width", I32), ("levels", I32), ("channels", I32 * 8),
                ("enc_channels", I32), ("lidar_h", I32), ("lidar_w", I32), ("depth_resolution", F32),
                ("soft_gate", I32), ("fit_iters", I32), ("fit_trim", F32), ("fit_min_points", I32),
                ("use_prompt", I32), ("capacity", I64 * 8), ("use_tensor_cores", I32), ("max_split", I32),
                ("output_gate", I32), ("anchor_beta", F32), ("output_gate_floor", C.c_double), ("use_pdl", I32),
                ("multi_launch_fit", I32), ("multi_launch_transitions", I32)]


# name -> (restype, argtypes)
SIGNATURES = {
    "pmg_abi_version": (I32, []),
    "pmg_status_string": (C.c_char_p, [I32]),
    "pmg_last_cuda_error": (I32, []),
    "pmg_check_device": (I32, []),
    "pmg_voxelize_l0": (I32, [P, I32, I32, I32, F32, P, P, P, P, I64, P, P]),
    "pmg_l0_coords": (I32, [P, P, I32, I32, I32, P, P]),
    "pmg_pool_frames_workspace_bytes": (SZ, [I32, I32, I32]),
    "pmg_pool_frames": (I32, [I32, I32, I32, P, P, P, P, P, P, P, P, P, I64, P, P, P, P, SZ, P, P]),
    "pmg_nmap_frames": (I32, [I32, I32, I32, P, P, P, P, P, I64, P, P]),
    "pmg_nmap_hash_workspace_bytes": (SZ, [I64]),
    "pmg_nmap_hash": (I32, [P, I64, C.POINTER(I64), P, I64, I32, P, P, SZ, P, P]),
    "pmg_nmap_hash_noalloc": (I32, [P, I64, C.POINTER(I64), P, I64, I32, P, P, P]),
    "pmg_frame_csr": (I32, [P, I64, I32, I32, I32, I64, P, P, P, P]),
    "pmg_gauge_workspace_bytes": (SZ, [I32, I32, I32]),
    "pmg_gauge_poly": (I32, [P, P, P, I32, I32, I32, I32, I32, I32, I32, P, P, P, P, P, SZ, P]),
    "pmg_prompt_workspace_bytes": (SZ, [I32, I32, I32]),
    "pmg_nearest_fill": (I32, [P, P, I32, I32, I32, P, P, P, SZ, P]),
    "pmg_build_prompt": (I32, [P, P, I32, I32, I32, I32, I32, F32, P, P, P, SZ, P]),
    "pmg_resize_remap": (I32, [P, I32, I32, I32, I32, I32, P, P]),
    "pmg_focal_shift": (I32, [P, P, P, I32, I32, I32, I32, I32, P, P, P]),
    "pmg_shift_depth": (I32, [P, P, I32, I32, I32, P, P]),
    "pmg_depth_to_points": (I32, [P, P, I32, I32, I32, P, P, P, P]),
    "pmg_output_gate": (I32, [P, P, P, I64, P, P, I32, I32, I32, I32, I32, C.c_double, P]),
    "pmg_anchor_apply": (I32, [P, I64, P, P, P, I32, I32, I32, I32, I32, F32, P]),
    "pmg_spconv_i8": (I32, [P, I64, P, I64, P, P, I64, I32, I32, P, P, P, F32, I32, F32, P, P, I32, P, P]),
    "pmg_spconv_i8_split_workspace_bytes": (SZ, [I64, I32, I32]),
    "pmg_spconv_i8_split": (I32, [P, I64, P, I64, P, P, I64, I32, I32, P, P, P, F32, I32, F32, P, P, I32, P, SZ, P, P]),
    "pmg_l0_tap_lanes_bytes": (SZ, [I32, I32, I32]),
    "pmg_l0_tap_lanes": (I32, [P, I32, I32, I32, P, P]),
    "pmg_spconv_i8_grid0": (I32, [P, P, I32, I32, I32, I32, I32, P, P, P, F32, I32, F32, P, P, P, P]),
    "pmg_dense_i8": (I32, [P, P, I64, I32, I32, P, P, P, F32, I32, F32, P, P, I32, P, P]),
    "pmg_quantize": (I32, [P, I64, F32, P, P]),
    "pmg_ln_silu_q8": (I32, [P, P, P, P, P, P, I64, I32, P, P, F32, F32, P, P]),
    "pmg_pool_mean_q8": (I32, [P, P, P, P, I64, I32, F32, P, P]),
    "pmg_pool_mean_f32": (I32, [P, P, P, P, I64, I32, P, P]),
    "pmg_pool_sum_f32": (I32, [P, P, P, P, I64, I32, P, P]),
    "pmg_gather_rows_f32": (I32, [P, P, P, I64, I32, P, P]),
    "pmg_spconv_f32": (I32, [P, P, I64, P, P, I64, I32, I32, P, P, P, P]),
    "pmg_fit_workspace_bytes": (SZ, [I32, I64]),
    "pmg_fit_prep_prompt": (I32, [P, I64, P, P, I32, I32, I32, I32, I32, P, P, P, P]),
    "pmg_fit_prep_final": (I32, [P, P, P, P, I32, I32, I32, I32, I32, P, P, P, P]),
    "pmg_fit_solve": (I32, [P, P, P, I32, I64, I32, F32, I32, P, P, SZ, P]),
    "pmg_prompt_feats": (I32, [P, I64, P, P, P, I32, I32, I32, I32, I32, I32, P, P]),
    "pmg_affine_frame": (I32, [P, I64, P, P, P, I32, I32, I32, I32, I32, I32, P, P, P]),
    "pmg_fit_prompt_fused_workspace_bytes": (SZ, [I32, I32, I32]),
    "pmg_fit_prompt_fused": (I32, [P, I64, P, P, I32, I32, I32, I32, I32, I32, F32, I32, I32, P, P, P, P, P, SZ, P]),
    "pmg_apply_affine": (I32, [P, P, I32, I64, P]),
    "pmg_refiner_create": (I32, [C.POINTER(RefinerConfig), C.POINTER(P)]),
    "pmg_refiner_destroy": (None, [P]),
    "pmg_refiner_set_qlayer": (I32, [P, C.c_char_p, P, P, P, F32]),
    "pmg_refiner_set_norm": (I32, [P, C.c_char_p, P, P]),
    "pmg_refiner_set_proj": (I32, [P, C.c_char_p, P, P]),
    "pmg_refiner_set_frame": (I32, [P, P, P, P]),
    "pmg_refiner_set_inputs": (I32, [P, P, P, P]),
    "pmg_refiner_set_prompt": (I32, [P, P]),
    "pmg_refiner_enqueue": (I32, [P, I32, P, P, P]),
    "pmg_refiner_capture": (I32, [P, I32, P, P, P]),
    "pmg_refiner_launch": (I32, [P, P]),
    "pmg_refiner_status": (I32, [P, P, I32, P]),
    "pmg_refiner_set_capacity": (I32, [P, C.POINTER(I64)]),
    "pmg_refiner_launches_per_step": (I32, [P]),
    "pmg_refiner_level_info": (I32, [P, I32, C.POINTER(I64), C.POINTER(I32), C.POINTER(I32), C.POINTER(I32)]),
    "pmg_refiner_debug_ptr": (P, [P, C.c_char_p, I32]),
}

STATUS = {0: "ok", 1: "bad argument", 2: "CUDA runtime error", 3: "hash table full", 4: "level capacity overflow",
          5: "unsupported configuration", 6: "coordinate outside the key range", 7: "no sm_100 device",
          8: "bounded wait expired inside a kernel"}

EPI_ACC32, EPI_F32, EPI_F32_RESID, EPI_SILU_Q8 = 0, 1, 2, 3


class PmgError(RuntimeError):
    def __init__(self, fn: str, code: int):
        extra = ""
        if code == 2 and _lib is not None:
            extra = f" (cudaError {_lib.pmg_last_cuda_error()})"
        super().__init__(f"{fn} failed: {STATUS.get(code, code)}{extra}")
        self.code = code


_lib = None


def load(path: str | os.PathLike | None = None) -> C.CDLL:
    """Load (once) the in-tree library and attach the prototypes.  Raises if it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise ImportError(f"{p} is missing: build it with `python -m promptmoge_b200.build` (nvcc, sm_100a)")
    lib = C.CDLL(str(p))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def call(name: str, *args) -> int:
    """Call a status-returning entry point and raise PmgError on failure."""
    rc = getattr(load(), name)(*args)
    if rc != 0:
        raise PmgError(name, rc)
    return rc


def header_functions(header: str | os.PathLike | None = None) -> list:
    """Names of the functions declared in include/pmg_b200.h."""
    import re
    h = Path(header) if header else _PKG.parent / "include" / "pmg_b200.h"
    text = h.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(pmg_[a-z0-9_]+)\s*\(", text)))
