"""The trunk's pair input (pf_trunk_init_fwd) and recycling step (pf_pair_ln_linear_fwd) on the
GPU: against the reference's own outputs (tests/golden/trunk) in fp32, against the fp32 oracle
in bf16, and the Fold-CP local construction (per-rank tiles) against the full plane."""
import os
import sys
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from gpu_helpers import rel_l2
from oracle import pairformer_oracle as O
from opendde_b200 import _abi
from opendde_b200.distributed.foldcp import apply_trunk_z_cycle_local, build_trunk_z_init_local
from opendde_b200.model import (LayerNorm, LazyRelativePositionEncodingFeatures, RelativePositionEncoding,
                                trunk_pair_cycle, trunk_pair_init)
from opendde_b200.model.primitives import LinearNoBias

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
from make_trunk_golden import trunk_inputs, trunk_param_shapes  # noqa: E402

from opendde_b200.utils import seeded_params  # noqa: E402

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(HERE, "golden", "trunk", "trunk_init_n23.npz")


def _modules(c_s, c_z, r_max, s_max, device, dtype, seed=0):
    params = seeded_params(trunk_param_shapes(c_s, c_z, r_max, s_max), seed=seed, perturb_1d=True)
    z1, z2, bond = LinearNoBias(c_s, c_z), LinearNoBias(c_s, c_z), LinearNoBias(1, c_z)
    relpe = RelativePositionEncoding(r_max=r_max, s_max=s_max, c_z=c_z)
    ln, cyc = LayerNorm(c_z), LinearNoBias(c_z, c_z)
    with torch.no_grad():
        z1.weight.copy_(params["linear_no_bias_zinit1.weight"])
        z2.weight.copy_(params["linear_no_bias_zinit2.weight"])
        relpe.linear_no_bias.weight.copy_(params["relative_position_encoding.linear_no_bias.weight"])
        bond.weight.copy_(params["linear_no_bias_token_bond.weight"])
        ln.weight.copy_(params["layernorm_z_cycle.weight"])
        ln.bias.copy_(params["layernorm_z_cycle.bias"])
        cyc.weight.copy_(params["linear_no_bias_z_cycle.weight"])
    mods = [m.to(device) for m in (z1, z2, relpe, bond, ln, cyc)]
    return mods, params


def _feats(feats, r_max, s_max, device):
    return LazyRelativePositionEncodingFeatures(*[feats[k].to(device) for k in
                                                  ("asym_id", "residue_index", "entity_id", "token_index", "sym_id")],
                                                r_max=r_max, s_max=s_max)


def test_trunk_init_fp32_matches_reference_outputs(cuda_device):
    rec = dict(np.load(GOLDEN))
    r_max, s_max = int(rec["r_max"]), int(rec["s_max"])
    (z1, z2, relpe, bond, ln, cyc), _ = _modules(int(rec["c_s"]), int(rec["c_z"]), r_max, s_max, cuda_device,
                                                 torch.float32)
    feats, bonds, s_init, z_prev = trunk_inputs()
    with torch.no_grad():
        z_init = trunk_pair_init(s_init.to(cuda_device), z1, z2, relpe, bond, _feats(feats, r_max, s_max, cuda_device),
                                 bonds.to(cuda_device))
        z_cyc = trunk_pair_cycle(z_init, z_prev.to(cuda_device), ln, cyc)
    assert _abi.device_status(clear=True) == 0
    e1 = (z_init.cpu() - torch.from_numpy(rec["z_init"])).abs().max().item()
    e2 = (z_cyc.cpu() - torch.from_numpy(rec["z_cycle"])).abs().max().item()
    print(f"trunk init fp32: max-abs {e1:.2e}, recycle {e2:.2e}")
    assert e1 <= 1e-4 and e2 <= 1e-4


@pytest.mark.parametrize("n,c_s,c_z", [(23, 32, 64), (300, 384, 128)])
def test_trunk_init_bf16_against_oracle(n, c_s, c_z, cuda_device):
    r_max, s_max = (4, 2) if n == 23 else (32, 2)
    (z1, z2, relpe, bond, ln, cyc), params = _modules(c_s, c_z, r_max, s_max, cuda_device, torch.bfloat16)
    if n == 23:
        feats, bonds, s_init, z_prev = trunk_inputs()
    else:
        g = torch.Generator().manual_seed(3)
        chain = torch.repeat_interleave(torch.arange(5), torch.tensor([90, 60, 60, 50, 40]))
        feats = {"asym_id": chain, "entity_id": chain % 3, "sym_id": chain // 3,
                 "residue_index": torch.cat([torch.arange(k) * (1 + (k % 2)) for k in (90, 60, 60, 50, 40)]),
                 "token_index": torch.arange(n)}
        bonds = (torch.rand((n, n), generator=g) < 0.02).float()
        s_init = torch.randn((n, c_s), generator=g)
        z_prev = torch.randn((n, n, c_z), generator=g)
    for m in (z1, z2, relpe, bond, ln, cyc):
        m.to(torch.bfloat16)
    ln.float()
    sb, zpb = s_init.to(cuda_device, torch.bfloat16), z_prev.to(cuda_device, torch.bfloat16)
    with torch.no_grad():
        z_init = trunk_pair_init(sb, z1, z2, relpe, bond, _feats(feats, r_max, s_max, cuda_device), bonds.to(cuda_device))
        assert _abi.last_path() == "simt"
        z_cyc = trunk_pair_cycle(z_init, zpb, ln, cyc)
        assert _abi.last_path() == "tc.rows"
        pd = {k: v.to(cuda_device) for k, v in params.items()}
        want = O.trunk_z_init(sb.float(), {k: v.to(cuda_device) for k, v in feats.items()}, bonds.to(cuda_device), pd,
                              r_max, s_max)
        want_c = O.trunk_z_cycle(z_init.float(), zpb.float(), pd)
    assert _abi.device_status(clear=True) == 0
    e1, e2 = rel_l2(z_init, want), rel_l2(z_cyc, want_c)
    print(f"trunk init bf16 N={n}: rel-L2 {e1:.3e}, recycle {e2:.3e}")
    assert e1 <= 2e-2 and e2 <= 2e-2


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("mesh_shape", [(2, 3), (2, 2)])
def test_foldcp_local_tiles_assemble_the_plane(dtype, mesh_shape, cuda_device):
    rec = dict(np.load(GOLDEN))
    r_max, s_max = int(rec["r_max"]), int(rec["s_max"])
    (z1, z2, relpe, bond, ln, cyc), _ = _modules(int(rec["c_s"]), int(rec["c_z"]), r_max, s_max, cuda_device, dtype)
    if dtype == torch.bfloat16:
        for m in (z1, z2, relpe, bond, cyc):
            m.to(dtype)
    feats, bonds, s_init, z_prev = trunk_inputs()
    s, zp = s_init.to(cuda_device, dtype), z_prev.to(cuda_device, dtype)
    lazy = _feats(feats, r_max, s_max, cuda_device)
    n = s.shape[0]
    with torch.no_grad():
        full = trunk_pair_init(s, z1, z2, relpe, bond, lazy, bonds.to(cuda_device))
        full_c = trunk_pair_cycle(full, zp, ln, cyc)
        R, C = mesh_shape
        for r in range(R):
            for c in range(C):
                mesh = SimpleNamespace(layout=SimpleNamespace(shape=mesh_shape), coord=(r, c))
                z_loc, spec = build_trunk_z_init_local(s_init=s, linear_zinit1=z1, linear_zinit2=z2,
                                                       relative_position_encoding=relpe, linear_token_bond=bond,
                                                       relp_feature=lazy, token_bonds=bonds.to(cuda_device), mesh=mesh)
                (r0, r1), (c0, c1) = spec.row_range, spec.col_range
                vr, vc = min(r1, n) - r0, min(c1, n) - c0
                assert torch.equal(z_loc[:vr, :vc], full[r0:r0 + vr, c0:c0 + vc])
                assert not z_loc[vr:].any() and not z_loc[:, vc:].any()
                zp_loc = torch.zeros_like(z_loc)
                zp_loc[:vr, :vc] = zp[r0:r0 + vr, c0:c0 + vc]
                z_c = apply_trunk_z_cycle_local(z_init_local=z_loc, z_local=zp_loc, layernorm_z_cycle=ln,
                                                linear_z_cycle=cyc, z_spec=spec)
                assert torch.equal(z_c[:vr, :vc], full_c[r0:r0 + vr, c0:c0 + vc])
    assert _abi.device_status(clear=True) == 0
