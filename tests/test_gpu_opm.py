"""OuterProductMean (pf_opm_fwd) on the GPU against the oracle and the reference's outputs.

* bf16 (tensor-core path: projections, the outer product over the sequences as one channel of
  the per-channel contraction, W_out over the 32 x 32 outer-product channels read through a
  4-D tensor map): rel-L2 <= 2e-2 against the fp32 oracle, with a ragged MSA mask (fully masked
  sequence and residue column) and without a mask, at sizes with partial tiles.
* fp32 (SIMT): the reference's own outputs (tests/golden/opm) within 1e-4 of max |out|.
* Fold-CP tiles (``tile_update`` on 2 x 3 and 3 x 2 meshes, and the tile entry point's
  row / col offsets) bit-identical to the matching slice of the one-call update.
"""
import os
import sys

import numpy as np
import pytest
import torch

from gpu_helpers import rel_l2
from oracle import pairformer_oracle as O
from opendde_b200 import _abi
from opendde_b200.model import OuterProductMean
from opendde_b200.utils import seeded_init_

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
from make_opm_golden import opm_inputs  # noqa: E402

pytestmark = pytest.mark.gpu

BF16_TOL = 2e-2


def _module(c_m, c_hidden, c_z, device, seed=0):
    mod = OuterProductMean(c_m=c_m, c_z=c_z, c_hidden=c_hidden)
    params = seeded_init_(mod, seed=seed, perturb_1d=True)
    return mod.to(device), params


def _dev(params, device):
    return {k: v.to(device) for k, v in params.items()}


@pytest.mark.parametrize("n_seq,n_res,masked", [(37, 130, True), (200, 70, False), (5, 11, True)])
def test_opm_bf16_against_oracle(n_seq, n_res, masked, cuda_device):
    c_m, c_hidden, c_z = 64, 32, 128
    mod, params = _module(c_m, c_hidden, c_z, cuda_device)
    m, mask = opm_inputs(n_seq, n_res, c_m, masked)
    mb = m.to(cuda_device, torch.bfloat16)
    md = mask.to(cuda_device) if mask is not None else None
    with torch.no_grad():
        got = mod(mb, mask=md)
        assert _abi.last_path() == "tc.rows"
        old = torch.backends.cuda.matmul.allow_tf32
        torch.backends.cuda.matmul.allow_tf32 = False
        try:
            want = O.outer_product_mean(mb.float(), md, _dev(params, cuda_device))
        finally:
            torch.backends.cuda.matmul.allow_tf32 = old
    assert _abi.device_status(clear=True) == 0
    err = rel_l2(got, want)
    print(f"OPM bf16 S={n_seq} N={n_res} masked={masked}: rel-L2 {err:.3e}")
    assert err <= BF16_TOL


@pytest.mark.parametrize("name", ["opm_s7_n13_masked", "opm_s5_n11_nomask"])
def test_opm_fp32_against_reference_outputs(name, cuda_device):
    rec = dict(np.load(os.path.join(HERE, "golden", "opm", f"{name}.npz")))
    n_seq, n_res, c_m, c_h, c_z = (int(rec[k]) for k in ("n_seq", "n_res", "c_m", "c_hidden", "c_z"))
    mod, _ = _module(c_m, c_h, c_z, cuda_device)
    m, mask = opm_inputs(n_seq, n_res, c_m, bool(rec["masked"]))
    with torch.no_grad():
        got = mod(m.to(cuda_device), mask=mask.to(cuda_device) if mask is not None else None)
    assert _abi.last_path() == "simt"
    want = torch.from_numpy(rec["out"])
    err = (got.cpu() - want).abs().max().item()
    scale = max(1.0, want.abs().max().item())
    print(f"OPM fp32 {name}: max-abs {err:.3e} (max |out| {scale:.1f})")
    assert err <= 1e-4 * scale


@pytest.mark.parametrize("mesh", [(2, 3), (3, 2)])
def test_opm_tiles_match_the_full_update(mesh, cuda_device):
    c_m, c_hidden, c_z = 64, 32, 128
    n_seq, n_res = 41, 131
    mod, _ = _module(c_m, c_hidden, c_z, cuda_device, seed=3)
    m, mask = opm_inputs(n_seq, n_res, c_m, True)
    mb, md = m.to(cuda_device, torch.bfloat16), mask.to(cuda_device)
    with torch.no_grad():
        full = mod(mb, mask=md)
        rows, cols = mesh
        rt, ct = -(-n_res // rows), -(-n_res // cols)
        for r in range(rows):
            for c in range(cols):
                tile = mod.tile_update(mb, mesh, (r, c), mask=md)
                assert tile.shape == (rt, ct, c_z)
                r1, c1 = min(n_res, (r + 1) * rt), min(n_res, (c + 1) * ct)
                assert torch.equal(tile[: r1 - r * rt, : c1 - c * ct], full[r * rt:r1, c * ct:c1])
                assert not tile[r1 - r * rt:].any() and not tile[:, c1 - c * ct:].any()
    assert _abi.device_status(clear=True) == 0


def test_opm_accumulates_into_a_strided_view(cuda_device):
    """z(i, j) += OPM(i, j) through apply_ on a transposed view of an existing pair tensor."""
    c_m, c_hidden, c_z, n_seq, n_res = 64, 32, 128, 19, 77
    mod, _ = _module(c_m, c_hidden, c_z, cuda_device, seed=5)
    m, mask = opm_inputs(n_seq, n_res, c_m, True)
    mb, md = m.to(cuda_device, torch.bfloat16), mask.to(cuda_device)
    g = torch.Generator().manual_seed(4)
    z = torch.randn((n_res, n_res, c_z), generator=g).to(cuda_device, torch.bfloat16)
    with torch.no_grad():
        upd = mod(mb, mask=md)
        want = (z.float() + upd.float().transpose(0, 1)).to(torch.bfloat16)
        zt = z.clone()
        mod.apply_(mb, md, zt.transpose(0, 1), accumulate=True)
    assert _abi.device_status(clear=True) == 0
    assert rel_l2(zt, want) <= 1e-2
