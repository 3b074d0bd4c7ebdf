"""The C-ABI library builds, loads and exports every function include/pmg_b200.h declares.  CPU only: no compute
call is made without a GPU."""
import ctypes

import pytest

from promptmoge_b200 import _lib


def test_library_builds_and_loads():
    from promptmoge_b200 import build
    lib_path = build.build()
    assert lib_path.exists()
    lib = _lib.load()
    assert lib.pmg_abi_version() == 1


def test_every_header_function_is_exported_and_bound():
    lib = _lib.load()
    declared = _lib.header_functions()
    assert len(declared) >= 40
    for name in declared:
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes prototype"
    assert set(_lib.SIGNATURES) <= set(declared)


def test_status_strings_and_struct_layout():
    lib = _lib.load()
    assert lib.pmg_status_string(0) == b"ok"
    assert lib.pmg_status_string(4) == b"level capacity overflow"
    assert ctypes.sizeof(_lib.FitState) == 72


def test_workspace_queries_are_pure_host():
    lib = _lib.load()
    assert lib.pmg_pool_frames_workspace_bytes(1, 240, 320) >= 2 * 240 * 320 * 4
    assert lib.pmg_nmap_hash_workspace_bytes(100000) >= 200000 * 12
    assert lib.pmg_fit_workspace_bytes(2, 307200) > 0


def test_bad_arguments_rejected_without_device_work():
    lib = _lib.load()
    # null pointers / bad sizes are refused before any launch
    assert lib.pmg_voxelize_l0(None, 1, 4, 4, 256.0, None, None, None, None, 16, None, None) == 1
    assert lib.pmg_spconv_i8(None, 0, None, 0, None, None, 0, 16, 16, None, None, None, 1.0, 0, 1.0, None, None, 0,
                             None, None) == 1
    assert lib.pmg_dense_i8(None, None, 0, 16, 16, None, None, None, 1.0, 0, 1.0, None, None, 0, None, None) == 1


def test_product_path_has_no_cpu_fallback(monkeypatch, tmp_path):
    """A missing library is an ImportError, never a silent CPU path."""
    monkeypatch.setattr(_lib, "_lib", None)
    with pytest.raises(ImportError):
        _lib.load(tmp_path / "missing.so")
