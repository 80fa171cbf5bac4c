"""The C-ABI library loads, exports every symbol include/pairformer_b200.h declares, and
validates arguments on the host (no GPU needed for any of these calls)."""
import ctypes
import os
import re

import pytest

from opendde_b200 import _abi

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include",
                      "pairformer_b200.h")


def declared_symbols():
    txt = open(HEADER).read()
    return sorted(set(re.findall(r"^PF_API\s+[\w\s\*]+?\b(pf_\w+)\s*\(", txt, flags=re.M)))


def test_header_declares_the_binding_table():
    assert declared_symbols() == sorted(_abi.EXPORTED)


def test_library_exports_every_declared_symbol():
    lib = _abi.load()
    for name in declared_symbols():
        assert hasattr(lib, name), name


def test_abi_version_and_error_strings():
    lib = _abi.load()
    assert lib.pf_abi_version() == 1
    assert lib.pf_set_option(12345, 1) == _abi.PF_EINVAL_ARG
    assert b"unknown option" in lib.pf_last_error_string()


def test_workspace_queries_and_validation_without_gpu():
    lib = _abi.load()
    n = _abi.workspace_bytes("pf_trimul_workspace_size", 64, 64, 64, 128, 128, _abi.PF_F32)
    assert n > 64 * 64 * 128 * 4
    with pytest.raises(_abi.PFError) as e:
        _abi.workspace_bytes("pf_trimul_workspace_size", -1, 64, 64, 128, 128, _abi.PF_F32)
    assert e.value.status == _abi.PF_EINVAL_SHAPE
    with pytest.raises(_abi.PFError) as e:
        _abi.workspace_bytes("pf_trimul_workspace_size", 4, 4, 4, 128, 128, 7)
    assert e.value.status == _abi.PF_EINVAL_DTYPE
    # null weights are rejected before any launch
    v = _abi.PairView(None, 0, 0)
    mv = _abi.MaskView(None, 0, 0)
    st = lib.pf_trimul_fwd(ctypes.byref(_abi.TrimulParams()), v, v, mv, mv, v, v, 4, 4, 4, 128, 128,
                           1, _abi.PF_F32, None, 0, None)
    assert st == _abi.PF_EINVAL_ARG
    # q columns outside the slab
    p = _abi.TriattParams(*([1] * 8))
    good = _abi.PairView(16, 128 * 8, 128)
    st = lib.pf_triatt_fwd(ctypes.byref(p), good, mv, None, 0, 0, good, 8, 8, 8, 4, 8, 128, 4, 32,
                           1e9, 1, _abi.PF_F32, None, 0, None)
    assert st == _abi.PF_EINVAL_SHAPE
    assert b"outside the slab" in lib.pf_last_error_string()


def test_split_trimul_and_peer_entry_points_validate_on_the_host():
    """The Fold-CP entry points reject bad arguments before touching a device."""
    lib = _abi.load()
    v = _abi.PairView(None, 0, 0)
    mv = _abi.MaskView(None, 0, 0)
    st = lib.pf_trimul_project(ctypes.byref(_abi.TrimulParams()), v, mv, 4, 4, 128, 128, _abi.PF_BF16,
                               None, None, 8, None, 0, None)
    assert st == _abi.PF_EINVAL_ARG                      # null weights
    w = _abi.TrimulParams(*([16] * 10))
    good = _abi.PairView(16, 128 * 8, 128)
    st = lib.pf_trimul_project(ctypes.byref(w), good, mv, 4, 16, 128, 128, _abi.PF_BF16, 16, 16, 8, None, 0, None)
    assert st == _abi.PF_EINVAL_SHAPE                    # ld < n_cols
    st = lib.pf_trimul_combine(ctypes.byref(w), 16, 16, 4, 4, 4, 8, good, good, 128, 128, 1, _abi.PF_BF16,
                               None, 0, None)
    assert st == _abi.PF_EINVAL_SHAPE                    # ld < n_k
    assert _abi.workspace_bytes("pf_trimul_combine_workspace_size", 64, 64, 64, 128, 128, _abi.PF_F32) > 0
    with pytest.raises(_abi.PFError):
        _abi.workspace_bytes("pf_trimul_project_workspace_size", -1, 4, 128, 128, _abi.PF_F32)
    # copy regions: count, sizes and pitches are checked first
    assert lib.pf_copy_regions(None, 33, None) == _abi.PF_EINVAL_ARG
    assert lib.pf_copy_regions(None, 0, None) == _abi.PF_OK
    bad_pitch = (_abi.CopyRegion * 1)(_abi.CopyRegion(16, 32, 1, 4, 64, 32, 64, 0, 0))
    assert lib.pf_copy_regions(bad_pitch, 1, None) == _abi.PF_EINVAL_SHAPE
    bad_plane = (_abi.CopyRegion * 1)(_abi.CopyRegion(16, 32, 2, 4, 64, 64, 64, 100, 256))
    assert lib.pf_copy_regions(bad_plane, 1, None) == _abi.PF_EINVAL_SHAPE
    null_src = (_abi.CopyRegion * 1)(_abi.CopyRegion(None, 32, 1, 1, 16, 16, 16, 0, 0))
    assert lib.pf_copy_regions(null_src, 1, None) == _abi.PF_EINVAL_ARG
    empty = (_abi.CopyRegion * 1)(_abi.CopyRegion(None, None, 0, 5, 16, 16, 16, 0, 0))
    assert lib.pf_copy_regions(empty, 1, None) == _abi.PF_OK   # empty boxes are skipped
    # peer windows
    assert lib.pf_peer_handle_bytes() == 64
    assert lib.pf_peer_window_alloc(0, None, None) == _abi.PF_EINVAL_ARG
    assert lib.pf_peer_window_open(None, None) == _abi.PF_EINVAL_ARG
    assert lib.pf_peer_window_close(None) == _abi.PF_EINVAL_ARG
    assert lib.pf_peer_window_free(None) == _abi.PF_EINVAL_ARG
