"""pf_trimul_fwd_static_scratch against pf_trimul_fwd, through the C ABI.

The static-scratch entry point exists for callers that cannot allocate device memory or hand
the library a workspace (a plugin living inside a runtime that owns all device allocations,
or a foreign-language binding that only holds its input and output pointers). It runs the same
kernels as the workspace entry point, so its results must be bit-identical to it, call after
call, although every call reuses (and finds stale data in) the same fixed array inside the
library. The calls below go from the largest accepted problem (N = 256 fills the 48 MiB array
exactly) to smaller, odd, non-square ones, so stale contents of padded rows and tiles from an
earlier, larger call would show up as a difference.

This file is named to be collected last, so that a run stopping at the first failure has
already run every other test.
"""
import ctypes

import pytest
import torch

from opendde_b200 import _abi, kernels
from opendde_b200.model import TriangleMultiplicationIncoming, TriangleMultiplicationOutgoing
from opendde_b200.utils import make_inputs, ragged_pair_mask, seeded_init_

pytestmark = pytest.mark.gpu

SCRATCH = 48 * 1024 * 1024


def _static_call(pack, za, zb, ma, mb, zg, zo, dtype, c_h=128):
    n_i, n_k, c_z = za.shape
    n_j = zb.shape[0]
    return _abi.load().pf_trimul_fwd_static_scratch(
        ctypes.byref(pack.struct), kernels.pair_view(za), kernels.pair_view(zb), kernels.mask_view(ma),
        kernels.mask_view(mb), kernels.pair_view(zg), kernels.pair_view(zo), n_i, n_j, n_k, c_z, c_h, 0,
        dtype, kernels.stream_ptr())


def _module(outgoing, device):
    mod = (TriangleMultiplicationOutgoing if outgoing else TriangleMultiplicationIncoming)(c_z=128, c_hidden=128)
    seeded_init_(mod, seed=0, perturb_1d=True)
    return mod.to(device)


def _pair(n_rows, n_cols, seed, device, dtype):
    g = torch.Generator().manual_seed(seed)
    return torch.randn((n_rows, n_cols, 128), generator=g).to(device, dtype)


def _compare(pack, za, zb, ma, mb, zg, dtype, what):
    """Run both entry points on the same views; the outputs must be bit-identical."""
    n_i, n_j = za.shape[0], zb.shape[0]
    tdt = torch.bfloat16 if dtype == _abi.PF_BF16 else torch.float32
    want = torch.empty((n_i, n_j, 128), device=za.device, dtype=tdt)
    kernels.trimul(pack, za, zb, ma, mb, zg, want, 128, accumulate=False)  # pf_trimul_fwd
    got = torch.full_like(want, float("nan"))
    status = _static_call(pack, za, zb, ma, mb, zg, got, dtype)
    assert status == _abi.PF_OK, _abi.load().pf_last_error_string()
    torch.cuda.synchronize()
    assert _abi.device_status(clear=True) == 0
    assert torch.isfinite(got.float()).all(), what
    assert torch.equal(got, want), f"{what}: max |diff| {(got.float() - want.float()).abs().max().item():.3e}"


@pytest.mark.parametrize("outgoing", [True, False])
def test_static_scratch_matches_workspace_entry_point(outgoing, cuda_device):
    mod = _module(outgoing, cuda_device)
    pack = mod.weight_pack(torch.bfloat16, cuda_device)
    assert _abi.load().pf_static_scratch_bytes() == SCRATCH
    # 1) the largest accepted square problem: its scratch is the whole array
    n = 256
    assert _abi.workspace_bytes("pf_trimul_workspace_size", n, n, n, 128, 128, _abi.PF_BF16) == SCRATCH
    for seed in (1, 2):  # two calls in a row, different inputs
        _, z, _ = make_inputs(n, seed=seed, with_s=False)
        z = z.to(cuda_device, torch.bfloat16)
        m = ragged_pair_mask(n, seed=seed + 10, drop=0.1, full_rows=[3]).to(cuda_device)
        if outgoing:
            _compare(pack, z, z, m, m, z, _abi.PF_BF16, f"N=256 seed {seed}")
        else:
            zt, mt = z.transpose(0, 1), m.t()
            _compare(pack, zt, zt, mt, mt, z, _abi.PF_BF16, f"N=256 seed {seed}")
    # 2) then a smaller, odd, non-square problem (n_i = 131, n_j = 97, n_k = 113): partial
    # tiles and padded pitches land on scratch that the previous call filled
    n_i, n_j, n_k = 131, 97, 113
    za, zb, zg = _pair(n_i, n_k, 5, cuda_device, torch.bfloat16), _pair(n_j, n_k, 6, cuda_device, torch.bfloat16), \
        _pair(n_i, n_j, 7, cuda_device, torch.bfloat16)
    ma = ragged_pair_mask(max(n_i, n_j, n_k), seed=21, drop=0.15)[:n_i, :n_k].contiguous().to(cuda_device)
    mb = ragged_pair_mask(max(n_i, n_j, n_k), seed=22, drop=0.15)[:n_j, :n_k].contiguous().to(cuda_device)
    if outgoing:
        _compare(pack, za, zb, ma, mb, zg, _abi.PF_BF16, "131x97x113")
    else:  # incoming reads transposed views: a(k, i), b(k, j)
        zat = _pair(n_k, n_i, 8, cuda_device, torch.bfloat16).transpose(0, 1)
        zbt = _pair(n_k, n_j, 9, cuda_device, torch.bfloat16).transpose(0, 1)
        _compare(pack, zat, zbt, ma, mb, zg, _abi.PF_BF16, "131x97x113 transposed views")


def test_static_scratch_fp32_path(cuda_device):
    """The fp32 (SIMT) kernels through the static array, after the bf16 calls above."""
    mod = _module(True, cuda_device)
    pack = mod.weight_pack(torch.float32, cuda_device)
    n_i, n_j, n_k = 61, 45, 77
    assert _abi.workspace_bytes("pf_trimul_workspace_size", n_i, n_j, n_k, 128, 128, _abi.PF_F32) <= SCRATCH
    za, zb, zg = _pair(n_i, n_k, 11, cuda_device, torch.float32), _pair(n_j, n_k, 12, cuda_device, torch.float32), \
        _pair(n_i, n_j, 13, cuda_device, torch.float32)
    ma = ragged_pair_mask(128, seed=23, drop=0.2)[:n_i, :n_k].contiguous().to(cuda_device)
    mb = ragged_pair_mask(128, seed=24, drop=0.2)[:n_j, :n_k].contiguous().to(cuda_device)
    for call in range(2):
        _compare(pack, za, zb, ma, mb, zg, _abi.PF_F32, f"fp32 call {call}")


def test_static_scratch_rejects_problems_beyond_the_array(cuda_device):
    mod = TriangleMultiplicationOutgoing(c_z=128, c_hidden=128).to(cuda_device)
    pack = mod.weight_pack(torch.bfloat16, cuda_device)
    n = 257  # the first square size past the array: 3 x 128 x 257 x 264 x 2 bytes > 48 MiB
    z = torch.zeros((n, n, 128), device=cuda_device, dtype=torch.bfloat16)
    m = torch.ones((n, n), device=cuda_device)
    status = _static_call(pack, z, z, m, m, z, z, _abi.PF_BF16)
    assert status == _abi.PF_EINVAL_SHAPE
    msg = _abi.load().pf_last_error_string().decode()
    assert "fixed" in msg and str(SCRATCH) in msg
