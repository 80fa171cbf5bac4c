"""Generate the trunk pair-initialisation golden vectors from the OpenDDE reference modules (CPU).

Run in a container that has the reference source tree (it is NOT needed at test time):

    python tests/golden/make_trunk_golden.py --reference <path-to-OpenDDE-checkout>

The reference pieces are run as opendde/model/opendde.py:812-835 composes them:
LinearNoBias zinit1 / zinit2 (c_s -> c_z), RelativePositionEncoding (both the dense features of
generate_relp and the lazy ones of LazyRelativePositionEncodingFeatures), LinearNoBias token
bond (1 -> c_z), and one recycling step LayerNorm + LinearNoBias z_cycle. Weights are seeded with
``opendde_b200.utils.seeded_params`` under the reference's parameter names; inputs come from
``trunk_inputs`` below (also imported by the tests).
"""

from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
sys.path.insert(0, HERE)

from opendde_b200.utils import seeded_params  # noqa: E402

N, C_S, C_Z, R_MAX, S_MAX = 23, 32, 64, 4, 2


def trunk_param_shapes(c_s=C_S, c_z=C_Z, r_max=R_MAX, s_max=S_MAX):
    n_feat = 4 * r_max + 2 * s_max + 7
    return [("linear_no_bias_zinit1.weight", (c_z, c_s)), ("linear_no_bias_zinit2.weight", (c_z, c_s)),
            ("relative_position_encoding.linear_no_bias.weight", (c_z, n_feat)),
            ("linear_no_bias_token_bond.weight", (c_z, 1)), ("layernorm_z_cycle.weight", (c_z,)),
            ("layernorm_z_cycle.bias", (c_z,)), ("linear_no_bias_z_cycle.weight", (c_z, c_z))]


def trunk_inputs(n=N, c_s=C_S, c_z=C_Z):
    """Four chains (two copies of one entity), residue gaps, several tokens in one residue, a
    residue offset beyond r_max; symmetric sparse token bonds; s_init and a previous z."""
    g = torch.Generator().manual_seed(5)
    asym = torch.tensor([0] * 8 + [1] * 6 + [2] * 6 + [3] * (n - 20))
    entity = torch.tensor([0] * 8 + [1] * 6 + [0] * 6 + [2] * (n - 20))
    sym = torch.tensor([0] * 8 + [0] * 6 + [1] * 6 + [0] * (n - 20))
    residue = torch.cat([torch.tensor([1, 2, 3, 3, 3, 4, 10, 11]), torch.arange(1, 7), torch.arange(1, 7),
                         torch.arange(1, n - 19)])
    token = torch.arange(n)
    feats = {"asym_id": asym, "residue_index": residue, "entity_id": entity, "token_index": token, "sym_id": sym}
    bonds = (torch.rand((n, n), generator=g) < 0.1).float()
    bonds = torch.maximum(bonds, bonds.t())
    s_init = torch.randn((n, c_s), generator=g)
    z_prev = torch.randn((n, n, c_z), generator=g)
    return feats, bonds, s_init, z_prev


def checksum(t: torch.Tensor) -> np.ndarray:
    t = t.double()
    return np.array([t.sum().item(), t.abs().sum().item(), (t * t).sum().item()])


@torch.no_grad()
def run():
    from opendde.model.modules.embedders import RelativePositionEncoding
    from opendde.model.modules.primitives import LayerNorm, LinearNoBias
    params = seeded_params(trunk_param_shapes(), seed=0, perturb_1d=True)
    zinit1, zinit2 = LinearNoBias(C_S, C_Z), LinearNoBias(C_S, C_Z)
    bond = LinearNoBias(1, C_Z)
    relpe = RelativePositionEncoding(r_max=R_MAX, s_max=S_MAX, c_z=C_Z)
    ln, cyc = LayerNorm(C_Z), LinearNoBias(C_Z, C_Z)
    zinit1.weight.copy_(params["linear_no_bias_zinit1.weight"])
    zinit2.weight.copy_(params["linear_no_bias_zinit2.weight"])
    relpe.linear_no_bias.weight.copy_(params["relative_position_encoding.linear_no_bias.weight"])
    bond.weight.copy_(params["linear_no_bias_token_bond.weight"])
    ln.weight.copy_(params["layernorm_z_cycle.weight"])
    ln.bias.copy_(params["layernorm_z_cycle.bias"])
    cyc.weight.copy_(params["linear_no_bias_z_cycle.weight"])
    feats, bonds, s_init, z_prev = trunk_inputs()
    dense = relpe.generate_relp(dict(feats), lazy=False)["relp"]
    lazy = relpe.generate_relp(dict(feats), lazy=True)["relp"]
    z_init = zinit1(s_init)[..., None, :] + zinit2(s_init)[..., None, :, :]
    z_init = z_init + relpe(dense)
    z_init = z_init + bond(bonds.unsqueeze(dim=-1))
    z_lazy = zinit1(s_init)[..., None, :] + zinit2(s_init)[..., None, :, :] + relpe(lazy) + bond(bonds.unsqueeze(-1))
    assert torch.equal(z_init, z_lazy)
    z_cycle = z_init + cyc(ln(z_prev))
    return {"relp": dense.numpy().astype(np.float32), "z_init": z_init.numpy().astype(np.float32),
            "z_cycle": z_cycle.numpy().astype(np.float32), "chk_s": checksum(s_init), "chk_z_prev": checksum(z_prev),
            "chk_bonds": checksum(bonds), "chk_params": np.stack([checksum(params[k]) for k in sorted(params)]),
            "param_names": np.array(sorted(params))}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path to the OpenDDE source tree")
    args = ap.parse_args()
    sys.path.insert(0, os.path.abspath(args.reference))
    from make_golden import _stub_imports
    _stub_imports()
    rec = run()
    path = os.path.join(HERE, "trunk", "trunk_init_n23.npz")
    np.savez_compressed(path, n=np.array(N), c_s=np.array(C_S), c_z=np.array(C_Z), r_max=np.array(R_MAX),
                        s_max=np.array(S_MAX), **rec)
    print("wrote", path, os.path.getsize(path))


if __name__ == "__main__":
    main()
