"""pf_trimul_fwd_static_scratch against pf_trimul_fwd, through the C ABI.

The static-scratch entry point exists for callers that cannot allocate device memory or hand
the library a workspace (a plugin living inside a runtime that owns all device allocations,
or a foreign-language binding that only holds its input and output pointers). It must give
the same result as the workspace entry point, call after call, although every call reuses
(and finds stale data in) the same fixed array inside the library.

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

BF16_TOL = 2e-2  # relative L2, the bf16 tolerance used by every parity test


def _rel_l2(a, b):
    a, b = a.double(), b.double()
    return ((a - b).norm() / b.norm()).item()


def _static_call(pack, za, zb, ma, mb, zg, zo, c_h=128):
    n_i, n_k, c_z = za.shape
    n_j = zb.shape[0]
    return _abi.load().pf_trimul_fwd_static_scratch(
        ctypes.byref(pack.struct), kernels.pair_view(za), kernels.pair_view(zb), kernels.mask_view(ma),
        kernels.mask_view(mb), kernels.pair_view(zg), kernels.pair_view(zo), n_i, n_j, n_k, c_z, c_h, 0,
        _abi.PF_BF16, kernels.stream_ptr())


@pytest.mark.parametrize("outgoing", [True, False])
def test_static_scratch_matches_workspace_entry_point(outgoing, cuda_device):
    n = 200
    mod = (TriangleMultiplicationOutgoing if outgoing else TriangleMultiplicationIncoming)(c_z=128, c_hidden=128)
    seeded_init_(mod, seed=0, perturb_1d=True)
    mod = mod.to(cuda_device)
    pack = mod.weight_pack(torch.bfloat16, cuda_device)
    assert _abi.load().pf_static_scratch_bytes() == 48 * 1024 * 1024
    for call, seed in enumerate((1, 2)):  # two calls in a row, different inputs
        _, z, _ = make_inputs(n, seed=seed, with_s=False)
        z = z.to(cuda_device, torch.bfloat16)
        m = ragged_pair_mask(n, seed=seed + 10, drop=0.1, full_rows=[3]).to(cuda_device)
        if outgoing:
            za = zb = z
            ma = mb = m
        else:
            za = zb = z.transpose(0, 1)
            ma = mb = m.t()
        want = torch.empty_like(z)
        kernels.trimul(pack, za, zb, ma, mb, z, want, 128, accumulate=False)  # pf_trimul_fwd
        got = torch.full_like(z, float("nan"))
        status = _static_call(pack, za, zb, ma, mb, z, got)
        assert status == _abi.PF_OK, _abi.load().pf_last_error_string()
        torch.cuda.synchronize()
        assert _abi.device_status(clear=True) == 0
        assert torch.isfinite(got.float()).all()
        err = _rel_l2(got.float().cpu(), want.float().cpu())
        assert err <= BF16_TOL, f"call {call}: rel-L2 {err:.3e}"


def test_static_scratch_rejects_problems_beyond_the_array(cuda_device):
    mod = TriangleMultiplicationOutgoing(c_z=128, c_hidden=128).to(cuda_device)
    pack = mod.weight_pack(torch.bfloat16, cuda_device)
    n = 300  # 3 * 128 * n^2 * 2 bytes > 48 MiB
    z = torch.zeros((n, n, 128), device=cuda_device, dtype=torch.bfloat16)
    m = torch.ones((n, n), device=cuda_device)
    status = _static_call(pack, z, z, m, m, z, z)
    assert status == _abi.PF_EINVAL_SHAPE
    msg = _abi.load().pf_last_error_string().decode()
    assert "fixed" in msg and str(48 * 1024 * 1024) in msg
