"""Torch-facing wrappers over the C ABI: validation, pair views, weight packs, workspaces.

Every function here launches CUDA work through ``libpairformer_b200.so`` on
``torch.cuda.current_stream()``. CPU tensors are rejected (there is no CPU fallback).
The compute mode follows the pair tensor's dtype: float32 -> PF_F32 (SIMT fp32),
bfloat16 -> PF_BF16 (tcgen05 tensor cores where the shape is covered).
"""

from __future__ import annotations

import ctypes
from typing import Dict, Optional

import torch

from . import _abi
from ._abi import ApbParams, MaskView, PairView, TransitionParams, TriattParams, TrimulParams, check

_DTYPES = {torch.float32: _abi.PF_F32, torch.bfloat16: _abi.PF_BF16}


def dtype_code(t: torch.Tensor) -> int:
    try:
        return _DTYPES[t.dtype]
    except KeyError:
        raise TypeError(f"opendde_b200 supports float32 and bfloat16 pair tensors, got {t.dtype}") from None


def require_cuda(*ts: Optional[torch.Tensor]) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("opendde_b200 kernels need CUDA tensors; there is no CPU fallback "
                               "(use the reference modules for CPU execution)")


def stream_ptr() -> int:
    return torch.cuda.current_stream().cuda_stream


def pair_view(t: torch.Tensor) -> PairView:
    """[R, C, ch] tensor (any row/col strides, contiguous channels) -> PairView."""
    if t.dim() != 3:
        raise ValueError(f"pair tensor must be [R, C, ch], got shape {tuple(t.shape)}")
    if t.stride(2) != 1 and t.shape[2] > 1:
        raise ValueError("pair tensor channel dim must be contiguous")
    return PairView(t.data_ptr(), t.stride(0), t.stride(1))


def mask_view(m: Optional[torch.Tensor]) -> MaskView:
    if m is None:
        return MaskView(None, 0, 0)
    if m.dtype != torch.float32:
        raise TypeError("mask views are float32")
    return MaskView(m.data_ptr(), m.stride(0), m.stride(1))


def prepare_mask(mask: Optional[torch.Tensor], n_rows: int, n_cols: int, device) -> torch.Tensor:
    """Float32 CUDA mask of shape [n_rows, n_cols] (ones when None)."""
    if mask is None:
        return torch.ones((n_rows, n_cols), device=device, dtype=torch.float32)
    return mask.to(device=device, dtype=torch.float32)


def workspace(nbytes: int, device) -> torch.Tensor:
    return torch.empty((max(int(nbytes), 1),), dtype=torch.uint8, device=device)


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


# ------------------------------------------------------------------------------ weight packs

class WeightPack:
    """Weights converted once to the compute dtype (LayerNorm parameters stay fp32).

    Built from a module's parameters; rebuilt when any parameter's storage or version
    counter changes (e.g. after ``load_state_dict``).
    """

    def __init__(self, key, tensors: Dict[str, torch.Tensor], struct):
        self.key = key
        self.tensors = tensors  # keeps the converted storage alive
        self.struct = struct


def pack_key(params, dtype, device):
    return (dtype, str(device)) + tuple((p.data_ptr(), p._version) for p in params)


def _conv(p: Optional[torch.Tensor], dtype, device) -> Optional[torch.Tensor]:
    if p is None:
        return None
    return p.detach().to(device=device, dtype=dtype).contiguous()


def make_pack(struct_cls, spec: Dict[str, Optional[torch.Tensor]], f32_names, dtype, device, key):
    tensors = {}
    for name, p in spec.items():
        tensors[name] = _conv(p, torch.float32 if name in f32_names else dtype, device)
    struct = struct_cls(**{n: _ptr(t) for n, t in tensors.items()})
    return WeightPack(key, tensors, struct)


# ------------------------------------------------------------------------------ ops

def layernorm(x: torch.Tensor, weight: Optional[torch.Tensor], bias: Optional[torch.Tensor],
              eps: float = 1e-5) -> torch.Tensor:
    require_cuda(x)
    code = dtype_code(x)
    x = x.contiguous()
    y = torch.empty_like(x)
    c = x.shape[-1]
    w = None if weight is None else weight.detach().float().contiguous()
    b = None if bias is None else bias.detach().float().contiguous()
    check(_abi.load().pf_layernorm_fwd(x.data_ptr(), y.data_ptr(), _ptr(w), _ptr(b),
                                       x.numel() // c, c, eps, code, stream_ptr()))
    return y


def trimul(pack: WeightPack, za: torch.Tensor, zb: torch.Tensor, ma: torch.Tensor,
           mb: torch.Tensor, zg: torch.Tensor, zo: torch.Tensor, c_h: int, accumulate: bool) -> None:
    """zo (+)= TriangleMultiplicativeUpdate on views (see pf_trimul_fwd); gate source zg."""
    require_cuda(za, zb, zg, zo, ma, mb)
    code = dtype_code(zo)
    n_i, n_k, c_z = za.shape
    n_j = zb.shape[0]
    if zb.shape[1] != n_k or zo.shape[:2] != (n_i, n_j) or zg.shape[:2] != (n_i, n_j):
        raise ValueError(f"trimul view shapes disagree: za {tuple(za.shape)} zb {tuple(zb.shape)} zo {tuple(zo.shape)}")
    nbytes = _abi.workspace_bytes("pf_trimul_workspace_size", n_i, n_j, n_k, c_z, c_h, code)
    ws = workspace(nbytes, zo.device)
    check(_abi.load().pf_trimul_fwd(ctypes.byref(pack.struct), pair_view(za), pair_view(zb),
                                    mask_view(ma), mask_view(mb), pair_view(zg), pair_view(zo),
                                    n_i, n_j, n_k,
                                    c_z, c_h, int(accumulate), code, ws.data_ptr(), ws.numel(),
                                    stream_ptr()))


def triatt_bias(pack: WeightPack, z: torch.Tensor, heads: int, out: torch.Tensor) -> None:
    """out[h, r, s] = triangle bias of z(r, s) (fp32 natural units, or bf16 x log2(e))."""
    require_cuda(z, out)
    code = dtype_code(z)
    n_r, n_c, c = z.shape
    nbytes = _abi.workspace_bytes("pf_triatt_bias_workspace_size", n_r, n_c, c, heads, code)
    ws = workspace(nbytes, z.device)
    check(_abi.load().pf_triatt_bias(ctypes.byref(pack.struct), pair_view(z), n_r, n_c,
                                     out.data_ptr(), out.stride(0), out.stride(1), c, heads, code,
                                     ws.data_ptr(), ws.numel(), stream_ptr()))


def triatt(pack: WeightPack, zs: torch.Tensor, m: torch.Tensor, zo: torch.Tensor, heads: int,
           head_dim: int, inf: float, accumulate: bool, bias: Optional[torch.Tensor] = None,
           q_col0: int = 0, n_q: Optional[int] = None, n_valid_keys: Optional[int] = None) -> None:
    """zo (+)= starting-node triangle attention of slab zs (see pf_triatt_fwd)."""
    require_cuda(zs, zo, m, bias)
    code = dtype_code(zs)
    n_rows, n_keys, c = zs.shape
    n_q = n_keys if n_q is None else n_q
    n_valid = n_keys if n_valid_keys is None else n_valid_keys
    nbytes = _abi.workspace_bytes("pf_triatt_workspace_size", n_rows, n_keys, n_q, c, heads, head_dim, code)
    ws = workspace(nbytes, zs.device)
    b_ptr, b_hs, b_rs = (None, 0, 0) if bias is None else (bias.data_ptr(), bias.stride(0), bias.stride(1))
    check(_abi.load().pf_triatt_fwd(ctypes.byref(pack.struct), pair_view(zs), mask_view(m), b_ptr,
                                    b_hs, b_rs, pair_view(zo), n_rows, n_keys, n_valid, q_col0, n_q,
                                    c, heads, head_dim, inf, int(accumulate), code, ws.data_ptr(),
                                    ws.numel(), stream_ptr()))


def transition(pack: WeightPack, x2d: torch.Tensor, out2d: torch.Tensor, n_mult: int,
               accumulate: bool) -> None:
    """out (+)= Transition(x) over rows of 2-D views (row strides allowed, contiguous channels)."""
    require_cuda(x2d, out2d)
    code = dtype_code(x2d)
    rows, c = x2d.shape
    if x2d.stride(1) != 1 or out2d.stride(1) != 1:
        raise ValueError("transition rows must have contiguous channels")
    nbytes = _abi.workspace_bytes("pf_transition_workspace_size", rows, c, n_mult, code)
    ws = workspace(nbytes, x2d.device)
    check(_abi.load().pf_transition_fwd(ctypes.byref(pack.struct), x2d.data_ptr(), x2d.stride(0),
                                        out2d.data_ptr(), out2d.stride(0), rows, c, n_mult,
                                        int(accumulate), code, ws.data_ptr(), ws.numel(), stream_ptr()))


def apb_pair_bias(pack: WeightPack, z: torch.Tensor, heads: int, out: torch.Tensor) -> None:
    """out[h, r, s] (fp32) = linear_nobias_z(layernorm_z(z(r, s)))."""
    require_cuda(z, out)
    code = dtype_code(z)
    n_r, n_c, c_z = z.shape
    nbytes = _abi.workspace_bytes("pf_apb_pair_bias_workspace_size", n_r, n_c, c_z, heads, code)
    ws = workspace(nbytes, z.device)
    check(_abi.load().pf_apb_pair_bias(ctypes.byref(pack.struct), pair_view(z), n_r, n_c,
                                       out.data_ptr(), out.stride(0), out.stride(1), c_z, heads,
                                       code, ws.data_ptr(), ws.numel(), stream_ptr()))


def opm(pack: WeightPack, m: torch.Tensor, mask: Optional[torch.Tensor], z_out: torch.Tensor, row0: int,
        col0: int, c_hidden: int, eps: float, accumulate: bool) -> None:
    """z_out (+)= the OuterProductMean update of rows [row0, row0 + R) x cols [col0, col0 + C)
    (z_out is [R, C, c_z]) from the MSA representation ``m`` [S, N, c_m] and its mask [S, N]
    (see pf_opm_fwd)."""
    require_cuda(m, z_out, mask)
    code = dtype_code(m)
    if z_out.dtype != m.dtype:
        raise TypeError("the pair update must be in the MSA representation's dtype")
    n_seq, n_res, c_m = m.shape
    n_rows, n_cols, c_z = z_out.shape
    nbytes = _abi.workspace_bytes("pf_opm_workspace_size", n_seq, n_res, n_rows, n_cols, c_m, c_hidden, c_z, code)
    ws = workspace(nbytes, m.device)
    check(_abi.load().pf_opm_fwd(ctypes.byref(pack.struct), pair_view(m), mask_view(mask), pair_view(z_out), n_seq,
                                 n_res, row0, n_rows, col0, n_cols, c_m, c_hidden, c_z, float(eps), int(accumulate),
                                 code, ws.data_ptr(), ws.numel(), stream_ptr()))


def trunk_init(pack: WeightPack, s_init: torch.Tensor, ids, token_bonds: Optional[torch.Tensor],
               z_out: torch.Tensor, row0: int, col0: int, r_max: int, s_max: int) -> None:
    """z_out [R, C, c_z] = the trunk's pair input on rows [row0, row0 + R) x cols [col0, col0 + C)
    (see pf_trunk_init_fwd). ``ids``: int32 CUDA tensors asym_id, residue_index, entity_id,
    token_index, sym_id (in that order)."""
    require_cuda(s_init, z_out, token_bonds, *ids)
    code = dtype_code(s_init)
    if z_out.dtype != s_init.dtype or s_init.stride(-1) != 1:
        raise TypeError("s_init (contiguous channels) and the pair output must share the storage dtype")
    n_token, c_s = s_init.shape
    n_rows, n_cols, c_z = z_out.shape
    nbytes = _abi.workspace_bytes("pf_trunk_init_workspace_size", n_rows, n_cols, c_s, c_z, r_max, s_max, code)
    ws = workspace(nbytes, s_init.device)
    tid = _abi.TokenIds(*[t.data_ptr() for t in ids])
    check(_abi.load().pf_trunk_init_fwd(ctypes.byref(pack.struct), s_init.data_ptr(), s_init.stride(0), tid,
                                        mask_view(token_bonds), pair_view(z_out), n_token, row0, n_rows, col0,
                                        n_cols, c_s, c_z, r_max, s_max, code, ws.data_ptr(), ws.numel(),
                                        stream_ptr()))


def pair_ln_linear(pack: WeightPack, z_in: torch.Tensor, z_out: torch.Tensor, accumulate: bool) -> None:
    """z_out (+)= W LN(z_in) over the positions of two pair views (see pf_pair_ln_linear_fwd)."""
    require_cuda(z_in, z_out)
    code = dtype_code(z_in)
    if z_out.dtype != z_in.dtype:
        raise TypeError("pair views must share the dtype")
    n_rows, n_cols, c_in = z_in.shape
    c_out = z_out.shape[2]
    if z_out.shape[:2] != (n_rows, n_cols):
        raise ValueError("pair views must cover the same positions")
    nbytes = _abi.workspace_bytes("pf_pair_ln_linear_workspace_size", n_rows, n_cols, c_in, c_out, code)
    ws = workspace(nbytes, z_in.device)
    check(_abi.load().pf_pair_ln_linear_fwd(ctypes.byref(pack.struct), pair_view(z_in), pair_view(z_out), n_rows,
                                            n_cols, c_in, c_out, int(accumulate), code, ws.data_ptr(), ws.numel(),
                                            stream_ptr()))


def apb(pack: WeightPack, s_in: torch.Tensor, s_out: torch.Tensor, z: Optional[torch.Tensor],
        bias: Optional[torch.Tensor], heads: int, accumulate: bool) -> None:
    """s_out (+)= AttentionPairBias(s_in, z) (bias from z when ``bias`` is None)."""
    require_cuda(s_in, s_out, z, bias)
    code = dtype_code(s_in)
    n, c_s = s_in.shape
    c_z = z.shape[-1] if z is not None else 0
    if bias is not None and (bias.dtype != torch.float32 or not bias.is_contiguous()):
        raise ValueError("apb bias must be a contiguous float32 [H, N, N] tensor")
    nbytes = _abi.workspace_bytes("pf_apb_workspace_size", n, c_s, c_z, heads, code)
    ws = workspace(nbytes, s_in.device)
    zv = pair_view(z) if z is not None else PairView(None, 0, 0)
    check(_abi.load().pf_apb_fwd(ctypes.byref(pack.struct), s_in.data_ptr(), s_out.data_ptr(), zv,
                                 _ptr(bias), n, c_s, c_z, heads, int(accumulate), code,
                                 ws.data_ptr(), ws.numel(), stream_ptr()))


def apb_rows(pack: WeightPack, s_in: torch.Tensor, s_out: torch.Tensor, bias: torch.Tensor, q_row0: int,
             heads: int, accumulate: bool) -> None:
    """s_out (+)= AttentionPairBias query rows [q_row0, q_row0 + len(s_out)) of s_in.

    ``bias`` is the fp32 pair bias of those query rows over all keys, [H, n_q, n] with a
    contiguous key dimension (any head/row strides).
    """
    require_cuda(s_in, s_out, bias)
    code = dtype_code(s_in)
    n, c_s = s_in.shape
    n_q = s_out.shape[0]
    if not s_out.is_contiguous() or s_out.shape[1] != c_s or s_out.dtype != s_in.dtype:
        raise ValueError("apb_rows output must be a contiguous [n_q, c_s] tensor of the input dtype")
    if bias.dtype != torch.float32 or bias.dim() != 3 or bias.shape[1] < n_q or bias.shape[2] < n or bias.stride(2) != 1:
        raise ValueError("apb_rows bias must be float32 [H, n_q, n] with contiguous keys")
    nbytes = _abi.workspace_bytes("pf_apb_rows_workspace_size", n, n_q, c_s, heads, code)
    ws = workspace(nbytes, s_in.device)
    check(_abi.load().pf_apb_rows_fwd(ctypes.byref(pack.struct), s_in.data_ptr(), s_out.data_ptr(),
                                      bias.data_ptr(), bias.stride(0), bias.stride(1), n, q_row0, n_q, c_s,
                                      heads, int(accumulate), code, ws.data_ptr(), ws.numel(), stream_ptr()))


def copy_regions(regions, dma: bool = False) -> None:
    """Copy byte boxes ``(src_ptr, dst_ptr, planes, rows, row_bytes, src_pitch, dst_pitch,
    src_plane_pitch, dst_plane_pitch)`` on the current stream (sources may be peers' windows):
    by a kernel, one launch per PF_MAX_COPY_REGIONS boxes, or (``dma``) by the copy engines."""
    lib = _abi.load()
    if dma:
        if regions:
            arr = (_abi.CopyRegion * len(regions))(*[_abi.CopyRegion(*r) for r in regions])
            check(lib.pf_copy_regions_dma(arr, len(regions), stream_ptr()))
        return
    step = _abi.PF_MAX_COPY_REGIONS
    for i in range(0, len(regions), step):
        chunk = regions[i:i + step]
        arr = (_abi.CopyRegion * len(chunk))(*[_abi.CopyRegion(*r) for r in chunk])
        check(lib.pf_copy_regions(arr, len(chunk), stream_ptr()))


def trimul_project(pack: WeightPack, z: torch.Tensor, m: torch.Tensor, c_h: int, a_ptr: int, b_ptr: int,
                   ld: int) -> None:
    """a, b projections of the pair view ``z`` [R, C, c_z] (mask ``m`` [R, C]) written
    channel-major [c_h][R][ld] at the raw device addresses ``a_ptr`` / ``b_ptr`` (storage dtype:
    fp32 for fp32 z, bf16 for bf16 z)."""
    require_cuda(z, m)
    code = dtype_code(z)
    rows, cols, c_z = z.shape
    nbytes = _abi.workspace_bytes("pf_trimul_project_workspace_size", rows, cols, c_z, c_h, code)
    ws = workspace(nbytes, z.device)
    check(_abi.load().pf_trimul_project(ctypes.byref(pack.struct), pair_view(z), mask_view(m), rows, cols, c_z,
                                        c_h, code, a_ptr, b_ptr, ld, ws.data_ptr(), ws.numel(), stream_ptr()))


def trimul_combine(pack: WeightPack, a: torch.Tensor, b: torch.Tensor, n_k: int, zg: torch.Tensor,
                   zo: torch.Tensor, accumulate: bool) -> None:
    """zo (+)= the triangle update from channel-major projections a [c_h][n_i][ld] and
    b [c_h][n_j][ld] contracted over k < n_k, gated by LN_in(zg)."""
    require_cuda(a, b, zg, zo)
    code = dtype_code(zo)
    c_h, n_i, ld = a.shape
    n_j = b.shape[1]
    if b.shape[0] != c_h or b.shape[2] != ld or not a.is_contiguous() or not b.is_contiguous():
        raise ValueError("trimul_combine takes contiguous [c_h, n, ld] projections with one ld")
    if a.dtype != zo.dtype or b.dtype != zo.dtype:
        raise TypeError("projections must be in the pair tensor's dtype")
    c_z = zo.shape[2]
    nbytes = _abi.workspace_bytes("pf_trimul_combine_workspace_size", n_i, n_j, n_k, c_z, c_h, code)
    ws = workspace(nbytes, zo.device)
    check(_abi.load().pf_trimul_combine(ctypes.byref(pack.struct), a.data_ptr(), b.data_ptr(), ld, n_i, n_j, n_k,
                                        pair_view(zg), pair_view(zo), c_z, c_h, int(accumulate), code,
                                        ws.data_ptr(), ws.numel(), stream_ptr()))


def pair_head(pack: WeightPack, mode: int, z: torch.Tensor, zt: Optional[torch.Tensor], logits: torch.Tensor,
              contact: Optional[torch.Tensor] = None, contact_bins: int = 0) -> None:
    """logits [R, C, n_bins] (fp32, or z's dtype) of a pair tile and optionally the contact
    probabilities [R, C] (fp32): see pf_pair_head_fwd. ``zt`` holds z^T at the tile's positions
    (forms PF_HEAD_SYM_IN / PF_HEAD_SYM_OUT)."""
    require_cuda(z, zt, logits, contact)
    code = dtype_code(z)
    lcode = dtype_code(logits)
    n_rows, n_cols, c_z = z.shape
    n_bins = logits.shape[2]
    if logits.shape[:2] != (n_rows, n_cols) or (zt is not None and zt.shape != z.shape):
        raise ValueError("pair head views must cover the same positions")
    if zt is not None and zt.dtype != z.dtype:
        raise TypeError("z and zt must share the dtype")
    if contact is not None and (contact.dtype != torch.float32 or tuple(contact.shape) != (n_rows, n_cols)):
        raise ValueError("contact must be a float32 [R, C] tensor")
    nbytes = _abi.workspace_bytes("pf_pair_head_workspace_size", n_rows, n_cols, c_z, n_bins, code)
    ws = workspace(nbytes, z.device)
    ztv = pair_view(zt) if zt is not None else PairView(None, 0, 0)
    crs, ccs = (contact.stride(0), contact.stride(1)) if contact is not None else (0, 0)
    check(_abi.load().pf_pair_head_fwd(ctypes.byref(pack.struct), mode, pair_view(z), ztv, n_rows, n_cols, c_z,
                                       n_bins, pair_view(logits), lcode, _ptr(contact), crs, ccs, contact_bins, code,
                                       ws.data_ptr(), ws.numel(), stream_ptr()))


def confidence_pair_init(pack: WeightPack, s_inputs: torch.Tensor, coords: torch.Tensor, z_trunk: torch.Tensor,
                         z_out: torch.Tensor, row0: int, col0: int, n_dist_bins: int) -> None:
    """z_out [R, C, c_z] = the confidence head's pair input on rows [row0, row0 + R) x cols
    [col0, col0 + C) (see pf_confidence_pair_init_fwd); z_out may be z_trunk."""
    require_cuda(s_inputs, coords, z_trunk, z_out)
    code = dtype_code(z_trunk)
    if z_out.dtype != z_trunk.dtype or s_inputs.dtype != z_trunk.dtype or s_inputs.stride(-1) != 1:
        raise TypeError("s_inputs (contiguous channels) and the pair views must share the storage dtype")
    if coords.dtype != torch.float32 or not coords.is_contiguous() or coords.shape[-1] != 3:
        raise ValueError("coords must be a contiguous float32 [N_token, 3] tensor")
    n_token, c_s = s_inputs.shape
    n_rows, n_cols, c_z = z_out.shape
    if z_trunk.shape != z_out.shape:
        raise ValueError("z_trunk and z_out must cover the same positions")
    nbytes = _abi.workspace_bytes("pf_confidence_pair_init_workspace_size", n_rows, n_cols, c_s, c_z, n_dist_bins,
                                  code)
    ws = workspace(nbytes, z_out.device)
    check(_abi.load().pf_confidence_pair_init_fwd(ctypes.byref(pack.struct), s_inputs.data_ptr(), s_inputs.stride(0),
                                                  coords.data_ptr(), pair_view(z_trunk), pair_view(z_out), n_token,
                                                  row0, n_rows, col0, n_cols, c_s, c_z, n_dist_bins, code,
                                                  ws.data_ptr(), ws.numel(), stream_ptr()))


def diffusion_pair_cond(pack: WeightPack, z_trunk: torch.Tensor, ids, z_out: torch.Tensor, row0: int, col0: int,
                        n_token: int, r_max: int, s_max: int) -> None:
    """z_out [R, C, c_zd] = the diffusion pair conditioning on rows [row0, row0 + R) x cols
    [col0, col0 + C) (see pf_diffusion_pair_cond_fwd). ``ids``: int32 CUDA tensors asym_id,
    residue_index, entity_id, token_index, sym_id."""
    require_cuda(z_trunk, z_out, *ids)
    code = dtype_code(z_trunk)
    if z_out.dtype != z_trunk.dtype:
        raise TypeError("pair views must share the dtype")
    n_rows, n_cols, c_z = z_trunk.shape
    c_zd = z_out.shape[2]
    if z_out.shape[:2] != (n_rows, n_cols):
        raise ValueError("z_trunk and z_out must cover the same positions")
    nbytes = _abi.workspace_bytes("pf_diffusion_pair_cond_workspace_size", n_rows, n_cols, c_z, c_zd, r_max, s_max,
                                  code)
    ws = workspace(nbytes, z_out.device)
    tid = _abi.TokenIds(*[t.data_ptr() for t in ids])
    check(_abi.load().pf_diffusion_pair_cond_fwd(ctypes.byref(pack.struct), pair_view(z_trunk), tid,
                                                 pair_view(z_out), n_token, row0, n_rows, col0, n_cols, c_z, c_zd,
                                                 r_max, s_max, code, ws.data_ptr(), ws.numel(), stream_ptr()))
