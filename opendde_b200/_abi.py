"""ctypes binding of ``libpairformer_b200.so`` (the C ABI in ``include/pairformer_b200.h``).

This is the only module that touches the shared library. Every call returns a status
code; :func:`check` turns non-zero codes into Python exceptions carrying the library's
thread-local message. The library never allocates device memory: callers pass
workspaces (allocated here from torch's caching allocator).
"""

from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, Structure, c_char_p, c_float, c_int, c_int32, c_int64, c_size_t, c_void_p

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libpairformer_b200.so")

PF_OK = 0
PF_EINVAL_SHAPE = 1
PF_EINVAL_DTYPE = 2
PF_EUNSUPPORTED = 3
PF_ECUDA = 4
PF_ENCCL = 5
PF_ETIMEOUT = 6
PF_EINVAL_ARG = 7
PF_EWORKSPACE = 8
PF_F32 = 0
PF_BF16 = 1
PF_OPT_FORCE_SIMT = 1
PF_OPT_SM_RESERVE = 2

_STATUS_NAMES = {
    PF_EINVAL_SHAPE: "PF_EINVAL_SHAPE", PF_EINVAL_DTYPE: "PF_EINVAL_DTYPE",
    PF_EUNSUPPORTED: "PF_EUNSUPPORTED", PF_ECUDA: "PF_ECUDA", PF_ENCCL: "PF_ENCCL",
    PF_ETIMEOUT: "PF_ETIMEOUT", PF_EINVAL_ARG: "PF_EINVAL_ARG", PF_EWORKSPACE: "PF_EWORKSPACE",
}

# Every symbol the header declares (checked by tests/test_abi_symbols.py).
EXPORTED = (
    "pf_abi_version", "pf_last_error_string", "pf_set_option", "pf_last_path", "pf_device_status",
    "pf_device_status_async",
    "pf_launch_count", "pf_profile_enable", "pf_profile_report", "pf_selftest_bounded_wait",
    "pf_layernorm_fwd",
    "pf_trimul_workspace_size", "pf_trimul_fwd",
    "pf_trimul_project_workspace_size", "pf_trimul_project", "pf_trimul_combine_workspace_size",
    "pf_trimul_combine",
    "pf_static_scratch_bytes", "pf_trimul_fwd_static_scratch",
    "pf_triatt_bias_workspace_size", "pf_triatt_bias", "pf_triatt_workspace_size", "pf_triatt_fwd",
    "pf_transition_workspace_size", "pf_transition_fwd",
    "pf_apb_pair_bias_workspace_size", "pf_apb_pair_bias", "pf_apb_workspace_size", "pf_apb_fwd",
    "pf_apb_rows_workspace_size", "pf_apb_rows_fwd",
    "pf_peer_handle_bytes", "pf_peer_window_alloc", "pf_peer_window_free", "pf_peer_window_open",
    "pf_peer_window_close", "pf_copy_regions",
    "pf_opm_workspace_size", "pf_opm_fwd",
    "pf_trunk_init_workspace_size", "pf_trunk_init_fwd", "pf_pair_ln_linear_workspace_size",
    "pf_pair_ln_linear_fwd",
    "pf_copy_regions_dma",
    "pf_pair_head_workspace_size", "pf_pair_head_fwd",
    "pf_confidence_pair_init_workspace_size", "pf_confidence_pair_init_fwd",
    "pf_diffusion_pair_cond_workspace_size", "pf_diffusion_pair_cond_fwd",
)

# pf_pair_head_fwd forms (include/pairformer_b200.h)
PF_HEAD_PLAIN, PF_HEAD_SYM_IN, PF_HEAD_SYM_OUT = 0, 1, 2


class PFError(RuntimeError):
    """A non-zero pf_status from the library."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{_STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


class PairView(Structure):
    _fields_ = [("ptr", c_void_p), ("row_stride", c_int64), ("col_stride", c_int64)]


class MaskView(Structure):
    _fields_ = [("ptr", c_void_p), ("row_stride", c_int64), ("col_stride", c_int64)]


class TrimulParams(Structure):
    _fields_ = [(n, c_void_p) for n in (
        "ln_in_w", "ln_in_b", "w_ap", "w_ag", "w_bp", "w_bg", "ln_out_w", "ln_out_b", "w_z", "w_g")]


class TriattParams(Structure):
    _fields_ = [(n, c_void_p) for n in ("ln_w", "ln_b", "w_bias", "w_q", "w_k", "w_v", "w_g", "w_o")]


class TransitionParams(Structure):
    _fields_ = [(n, c_void_p) for n in ("ln_w", "ln_b", "w_a", "w_b", "w_o")]


class CopyRegion(Structure):
    _fields_ = [("src", c_void_p), ("dst", c_void_p), ("planes", c_int64), ("rows", c_int64),
                ("row_bytes", c_int64), ("src_pitch", c_int64), ("dst_pitch", c_int64),
                ("src_plane_pitch", c_int64), ("dst_plane_pitch", c_int64)]


PF_MAX_COPY_REGIONS = 32


class ApbParams(Structure):
    _fields_ = [(n, c_void_p) for n in (
        "ln_a_w", "ln_a_b", "w_q", "b_q", "w_k", "w_v", "w_g", "w_o", "ln_z_w", "ln_z_b", "w_z")]


class OpmParams(Structure):
    _fields_ = [(n, c_void_p) for n in ("ln_w", "ln_b", "w_1", "w_2", "w_out", "b_out")]


class TrunkInitParams(Structure):
    _fields_ = [(n, c_void_p) for n in ("w_zinit1", "w_zinit2", "w_relp", "w_bond")]


class TokenIds(Structure):
    _fields_ = [(n, c_void_p) for n in ("asym_id", "residue_index", "entity_id", "token_index", "sym_id")]


class PairLinearParams(Structure):
    _fields_ = [(n, c_void_p) for n in ("ln_w", "ln_b", "w")]


class PairHeadParams(Structure):
    _fields_ = [(n, c_void_p) for n in ("ln_w", "ln_b", "w", "b")]


class ConfidenceInitParams(Structure):
    _fields_ = [(n, c_void_p) for n in ("w_s1", "w_s2", "w_d", "w_d0", "lower_bins", "upper_bins")]


class DiffusionPairParams(Structure):
    _fields_ = [(n, c_void_p) for n in ("ln_zt_w", "w_zt", "w_relp", "ln_z_w", "w_z")] + [
        ("t1", TransitionParams), ("t2", TransitionParams)]


_lib = None


def load(path: str = LIB_PATH):
    """Load the library once and declare the argument types of every entry point."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise RuntimeError(
            f"{path} is missing: build it with `make -C opendde_b200/csrc` "
            "(or __graft_entry__.build()); there is no fallback implementation")
    lib = ctypes.CDLL(path)
    sz = POINTER(c_size_t)
    sig = {
        "pf_abi_version": ([], c_int),
        "pf_last_error_string": ([], c_char_p),
        "pf_last_path": ([], c_char_p),
        "pf_set_option": ([c_int, c_int64], c_int),
        "pf_device_status": ([POINTER(c_int), c_int], c_int),
        "pf_device_status_async": ([c_void_p, c_void_p], c_int),
        "pf_launch_count": ([], ctypes.c_longlong),
        "pf_profile_enable": ([c_int], c_int),
        "pf_profile_report": ([ctypes.c_char_p, c_size_t], c_int),
        "pf_selftest_bounded_wait": ([c_int64, c_void_p], c_int),
        "pf_layernorm_fwd": ([c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int32, c_float, c_int32, c_void_p], c_int),
        "pf_trimul_workspace_size": ([c_int64, c_int64, c_int64, c_int32, c_int32, c_int32, sz], c_int),
        "pf_trimul_fwd": ([POINTER(TrimulParams), PairView, PairView, MaskView, MaskView, PairView, PairView,
                           c_int64, c_int64, c_int64, c_int32, c_int32, c_int32, c_int32, c_void_p, c_size_t, c_void_p], c_int),
        "pf_trimul_project_workspace_size": ([c_int64, c_int64, c_int32, c_int32, c_int32, sz], c_int),
        "pf_trimul_project": ([POINTER(TrimulParams), PairView, MaskView, c_int64, c_int64, c_int32, c_int32,
                               c_int32, c_void_p, c_void_p, c_int64, c_void_p, c_size_t, c_void_p], c_int),
        "pf_trimul_combine_workspace_size": ([c_int64, c_int64, c_int64, c_int32, c_int32, c_int32, sz], c_int),
        "pf_trimul_combine": ([POINTER(TrimulParams), c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64,
                               PairView, PairView, c_int32, c_int32, c_int32, c_int32, c_void_p, c_size_t,
                               c_void_p], c_int),
        "pf_static_scratch_bytes": ([], c_size_t),
        "pf_trimul_fwd_static_scratch": ([POINTER(TrimulParams), PairView, PairView, MaskView, MaskView, PairView,
                                          PairView, c_int64, c_int64, c_int64, c_int32, c_int32, c_int32, c_int32,
                                          c_void_p], c_int),
        "pf_triatt_bias_workspace_size": ([c_int64, c_int64, c_int32, c_int32, c_int32, sz], c_int),
        "pf_triatt_bias": ([POINTER(TriattParams), PairView, c_int64, c_int64, c_void_p, c_int64, c_int64,
                            c_int32, c_int32, c_int32, c_void_p, c_size_t, c_void_p], c_int),
        "pf_triatt_workspace_size": ([c_int64, c_int64, c_int64, c_int32, c_int32, c_int32, c_int32, sz], c_int),
        "pf_triatt_fwd": ([POINTER(TriattParams), PairView, MaskView, c_void_p, c_int64, c_int64, PairView,
                           c_int64, c_int64, c_int64, c_int64, c_int64, c_int32, c_int32, c_int32, c_float,
                           c_int32, c_int32, c_void_p, c_size_t, c_void_p], c_int),
        "pf_transition_workspace_size": ([c_int64, c_int32, c_int32, c_int32, sz], c_int),
        "pf_transition_fwd": ([POINTER(TransitionParams), c_void_p, c_int64, c_void_p, c_int64, c_int64, c_int32,
                               c_int32, c_int32, c_int32, c_void_p, c_size_t, c_void_p], c_int),
        "pf_apb_pair_bias_workspace_size": ([c_int64, c_int64, c_int32, c_int32, c_int32, sz], c_int),
        "pf_apb_pair_bias": ([POINTER(ApbParams), PairView, c_int64, c_int64, c_void_p, c_int64, c_int64,
                              c_int32, c_int32, c_int32, c_void_p, c_size_t, c_void_p], c_int),
        "pf_apb_workspace_size": ([c_int64, c_int32, c_int32, c_int32, c_int32, sz], c_int),
        "pf_apb_fwd": ([POINTER(ApbParams), c_void_p, c_void_p, PairView, c_void_p, c_int64, c_int32, c_int32,
                        c_int32, c_int32, c_int32, c_void_p, c_size_t, c_void_p], c_int),
        "pf_apb_rows_workspace_size": ([c_int64, c_int64, c_int32, c_int32, c_int32, sz], c_int),
        "pf_apb_rows_fwd": ([POINTER(ApbParams), c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64,
                             c_int64, c_int32, c_int32, c_int32, c_int32, c_void_p, c_size_t, c_void_p], c_int),
        "pf_peer_handle_bytes": ([], c_size_t),
        "pf_peer_window_alloc": ([c_size_t, POINTER(c_void_p), c_void_p], c_int),
        "pf_peer_window_free": ([c_void_p], c_int),
        "pf_peer_window_open": ([c_void_p, POINTER(c_void_p)], c_int),
        "pf_peer_window_close": ([c_void_p], c_int),
        "pf_copy_regions": ([POINTER(CopyRegion), c_int32, c_void_p], c_int),
        "pf_copy_regions_dma": ([POINTER(CopyRegion), c_int32, c_void_p], c_int),
        "pf_trunk_init_workspace_size": ([c_int64, c_int64, c_int32, c_int32, c_int32, c_int32, c_int32, sz], c_int),
        "pf_trunk_init_fwd": ([POINTER(TrunkInitParams), c_void_p, c_int64, TokenIds, MaskView, PairView, c_int64,
                               c_int64, c_int64, c_int64, c_int64, c_int32, c_int32, c_int32, c_int32, c_int32,
                               c_void_p, c_size_t, c_void_p], c_int),
        "pf_pair_ln_linear_workspace_size": ([c_int64, c_int64, c_int32, c_int32, c_int32, sz], c_int),
        "pf_pair_ln_linear_fwd": ([POINTER(PairLinearParams), PairView, PairView, c_int64, c_int64, c_int32, c_int32,
                                   c_int32, c_int32, c_void_p, c_size_t, c_void_p], c_int),
        "pf_pair_head_workspace_size": ([c_int64, c_int64, c_int32, c_int32, c_int32, sz], c_int),
        "pf_pair_head_fwd": ([POINTER(PairHeadParams), c_int32, PairView, PairView, c_int64, c_int64, c_int32, c_int32,
                              PairView, c_int32, c_void_p, c_int64, c_int64, c_int32, c_int32, c_void_p, c_size_t,
                              c_void_p], c_int),
        "pf_confidence_pair_init_workspace_size": ([c_int64, c_int64, c_int32, c_int32, c_int32, c_int32, sz], c_int),
        "pf_confidence_pair_init_fwd": ([POINTER(ConfidenceInitParams), c_void_p, c_int64, c_void_p, PairView,
                                         PairView, c_int64, c_int64, c_int64, c_int64, c_int64, c_int32, c_int32,
                                         c_int32, c_int32, c_void_p, c_size_t, c_void_p], c_int),
        "pf_diffusion_pair_cond_workspace_size": ([c_int64, c_int64, c_int32, c_int32, c_int32, c_int32, c_int32, sz],
                                                  c_int),
        "pf_diffusion_pair_cond_fwd": ([POINTER(DiffusionPairParams), PairView, TokenIds, PairView, c_int64, c_int64,
                                        c_int64, c_int64, c_int64, c_int32, c_int32, c_int32, c_int32, c_int32,
                                        c_void_p, c_size_t, c_void_p], c_int),
        "pf_opm_workspace_size": ([c_int64, c_int64, c_int64, c_int64, c_int32, c_int32, c_int32, c_int32, sz], c_int),
        "pf_opm_fwd": ([POINTER(OpmParams), PairView, MaskView, PairView, c_int64, c_int64, c_int64, c_int64, c_int64,
                        c_int64, c_int32, c_int32, c_int32, c_float, c_int32, c_int32, c_void_p, c_size_t, c_void_p],
                       c_int),
    }
    for name, (args, res) in sig.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    _lib = lib
    return lib


def check(status: int) -> None:
    if status != PF_OK:
        msg = load().pf_last_error_string().decode(errors="replace")
        raise PFError(status, msg)


def last_path() -> str:
    return load().pf_last_path().decode()


def set_force_simt(flag: bool) -> None:
    check(load().pf_set_option(PF_OPT_FORCE_SIMT, 1 if flag else 0))


def set_sm_reserve(n: int) -> None:
    """Leave ``n`` SMs out of the persistent kernels this thread launches next (see
    PF_OPT_SM_RESERVE); 0 restores every SM."""
    check(load().pf_set_option(PF_OPT_SM_RESERVE, int(n)))


def device_status(clear: bool = False) -> int:
    """Read (and optionally clear) the device status word; synchronises the device."""
    v = c_int(0)
    check(load().pf_device_status(ctypes.byref(v), 1 if clear else 0))
    if clear:  # forget copies taken before the clear
        for w in _WATCH.values():
            w.buf.zero_()
            w.event = None
    return int(v.value)


class _StatusWatch:
    """A pinned host copy of one device's status word, refreshed stream-ordered."""

    def __init__(self):
        import torch
        self.buf = torch.zeros(1, dtype=torch.int32).pin_memory()
        self.event = None


_WATCH = {}

STATUS_BITS = {
    1: "a device-side bounded wait of an opendde_b200 kernel timed out (the kernels drained instead of "
       "hanging)",
    2: "a triangle-attention logit exceeded the f16 range of the bf16 path's logit accumulator "
       "(|q.k| log2(e)/sqrt(d) > 65504); run such inputs in fp32 mode",
    4: "a tensor-core kernel's shared-memory layout did not fit the dynamic shared memory it was "
       "given (the kernel returned without writing its outputs)",
}


def status_message(word: int) -> str:
    what = "; ".join(m for b, m in STATUS_BITS.items() if word & b) or f"status word {word:#x}"
    return (f"{what}: the outputs of the launches since then are invalid. The status word stays set "
            "until it is cleared with device_status(clear=True).")


def status_checkpoint(device) -> None:
    """Raise if a copy of ``device``'s status word made at an earlier checkpoint has completed
    and shows a timed-out wait, then enqueue a fresh copy on the current stream.

    No device synchronisation: a timed-out wait is reported at the first checkpoint after the
    copy that saw it completes, i.e. at most one checkpoint late. Skipped inside CUDA graph
    capture (a captured graph's caller checks with :func:`device_status`).
    """
    import torch
    if torch.cuda.is_current_stream_capturing():
        return
    idx = device.index if device.index is not None else torch.cuda.current_device()
    w = _WATCH.get(idx)
    if w is None:
        w = _WATCH[idx] = _StatusWatch()
    if w.event is not None and w.event.query() and int(w.buf[0]) != 0:
        word = int(w.buf[0])
        w.event = None
        raise PFError(PF_ETIMEOUT, status_message(word))
    if w.event is None or w.event.query():
        stream = torch.cuda.current_stream(device)
        check(load().pf_device_status_async(w.buf.data_ptr(), stream.cuda_stream))
        w.event = torch.cuda.Event()
        w.event.record(stream)


def launch_count() -> int:
    return int(load().pf_launch_count())


def profile_enable(on: bool) -> None:
    check(load().pf_profile_enable(1 if on else 0))


def profile_report() -> dict:
    """Per-kernel {name: (launches, total_ms, total_work, unit)} since the last report
    (synchronises). ``total_work`` is the algorithmic work the launches stated: flops of their
    contractions (unit "flop") or the minimum HBM bytes they move (unit "byte"); 0 and "" for
    kernels without a work model."""
    import json
    buf = ctypes.create_string_buffer(1 << 16)
    check(load().pf_profile_report(buf, len(buf)))
    return {k: (int(v[0]), float(v[1]), float(v[2]), str(v[3])) for k, v in json.loads(buf.value.decode()).items()}


def workspace_bytes(fn_name: str, *args) -> int:
    out = c_size_t(0)
    check(getattr(load(), fn_name)(*args, ctypes.byref(out)))
    return int(out.value)
