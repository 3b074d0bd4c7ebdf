"""The allocation-free neighbour map (pmg_nmap_hash_noalloc) against the workspace one (pmg_nmap_hash).

Callers such as a real-time capture loop that reserved its device memory at start-up, or a host that routes all
device memory through its own allocator, cannot let the library allocate.  The no-alloc entry point keeps its hash
table in a fixed array inside the library instead of a caller workspace; this file checks, through the C ABI, that it
returns exactly what the workspace entry point returns, on two different inputs called back to back (the second
call must not see the first call's table contents), and that an input above its fixed limit is refused.

Kept in its own file, named to be collected last, so that a failure here comes after every other GPU test ran.
"""
import ctypes as C

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

MAX_VOXELS = 1 << 18


def _noalloc(coords: torch.Tensor, extents, row_major: bool):
    from promptmoge_b200 import _lib
    lib = _lib.load()
    M = coords.shape[0]
    nmap = torch.full((M, 27) if row_major else (27, M), -7, dtype=torch.int32, device=coords.device)
    mask = torch.zeros((M + 31) // 32 + 1, dtype=torch.int32, device=coords.device)
    status = torch.zeros(1, dtype=torch.int32, device=coords.device)
    ext = (C.c_int64 * 4)(*[int(e) for e in extents])
    rc = lib.pmg_nmap_hash_noalloc(C.c_void_p(coords.data_ptr()), M, ext, C.c_void_p(nmap.data_ptr()), M,
                                   int(row_major), C.c_void_p(mask.data_ptr()), C.c_void_p(status.data_ptr()),
                                   C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, lib.pmg_status_string(rc)
    return nmap, mask, status


def _inputs():
    from promptmoge_b200 import synth
    shell = torch.from_numpy(synth.make_surface_voxels(60000, seed=21)).cuda()        # 2^21 grid, ~60k voxels
    room = synth.make_scene(3, 48, 64, 16, 256)
    from promptmoge_b200.levels import build_levels
    lv, _ = build_levels(torch.from_numpy(room.point_coord).cuda(), 5)
    c1 = lv[1]["coords"].contiguous()                                               # a refiner level, other grid
    ext1 = [1, lv[1]["H"], lv[1]["W"], int(c1[:, 3].max().item()) + 1]
    return [(shell, [1, 1 << 21, 1 << 21, 1 << 21]), (c1, ext1)]


def test_noalloc_equals_workspace_entry_point_on_consecutive_calls():
    from promptmoge_b200 import ops
    cases = _inputs()
    for row_major in (True, False):
        results = [_noalloc(c, e, row_major) for c, e in cases]          # two calls in a row, then compare
        torch.cuda.synchronize()
        for (coords, ext), (nm, mask, st) in zip(cases, results):
            want, want_mask, want_st = ops.nmap_hash(coords, ext, row_major=row_major)
            torch.cuda.synchronize()
            assert int(st.item()) == 0 and int(want_st.item()) == 0
            assert torch.equal(nm, want)
            n_groups = (coords.shape[0] + 31) // 32
            assert torch.equal(mask[:n_groups], want_mask[:n_groups])


def test_noalloc_at_its_size_limit_then_a_smaller_call():
    """M equal to the fixed limit (a dense 64^3 block: 262,144 voxels, so the table's slots are all in use and
    the values end at the array's last byte), then a smaller set on the same table: both equal pmg_nmap_hash."""
    from promptmoge_b200 import ops, synth
    r = torch.arange(64, dtype=torch.int32)
    x, y, z = torch.meshgrid(r, r, r, indexing="ij")
    cube = torch.stack([torch.zeros_like(x), x, y, z], -1).reshape(-1, 4).contiguous().cuda()
    assert cube.shape[0] == MAX_VOXELS
    small = torch.from_numpy(synth.make_surface_voxels(20000, seed=5)).cuda()
    cases = [(cube, [1, 64, 64, 64]), (small, [1, 1 << 21, 1 << 21, 1 << 21])]
    results = [_noalloc(c, e, False) for c, e in cases]
    torch.cuda.synchronize()
    for (coords, ext), (nm, mask, st) in zip(cases, results):
        want, want_mask, want_st = ops.nmap_hash(coords, ext, row_major=False)
        torch.cuda.synchronize()
        assert int(st.item()) == 0 and int(want_st.item()) == 0
        assert torch.equal(nm, want)
        n_groups = (coords.shape[0] + 31) // 32
        assert torch.equal(mask[:n_groups], want_mask[:n_groups])


def test_noalloc_refuses_inputs_above_its_fixed_table():
    from promptmoge_b200 import _lib
    lib = _lib.load()
    coords = torch.zeros((4, 4), dtype=torch.int32, device="cuda")
    ext = (C.c_int64 * 4)(1, 16, 16, 16)
    out = torch.empty(4, dtype=torch.int32, device="cuda")
    rc = lib.pmg_nmap_hash_noalloc(C.c_void_p(coords.data_ptr()), MAX_VOXELS + 1, ext, C.c_void_p(out.data_ptr()),
                                   MAX_VOXELS + 1, 1, None, None, None)
    assert rc == 1      # PMG_ERR_BAD_ARG, before any device work
