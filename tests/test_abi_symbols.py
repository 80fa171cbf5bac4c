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
