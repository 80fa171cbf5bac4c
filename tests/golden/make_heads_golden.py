"""Generate the golden vectors of the pair heads and the diffusion pair conditioning by running the
OpenDDE reference modules on CPU.

Run in a container that has the reference source tree (it is NOT needed at test time):

    python tests/golden/make_heads_golden.py --reference <path-to-OpenDDE-checkout>

The reference's import chain is stubbed exactly as in make_golden.py (``optree``, ``rdkit``).
Three fixtures, each the reference's own code path:

* distogram: ``DistogramHead.forward`` (opendde/model/modules/head.py:33-46) and the contact
  probabilities of ``distogram_contact_probs_local`` (opendde/distributed/foldcp/distogram.py:133-167),
  run on a one-rank gloo group with a 1 x 1 mesh;
* confidence: ``ConfidenceHead.forward`` with zero Pairformer blocks (confidence.py:204-383,
  488-637): the pair input (s_inputs projections, distance embedding) is captured as the stack's
  input, and pae / pde are the head's outputs;
* diffusion: ``DiffusionConditioning.prepare_cache`` (diffusion.py:828-847) with and without the
  c_z -> c_z_pair_diffusion compression.

Each fixture also records the names and shapes of the reference module's pair-side state
(``ref_state``). N = 23 keeps torch.cdist on its direct (non-matrix-product) form. Weights are
seeded with ``opendde_b200.utils.seeded_params`` under the reference's parameter names; inputs
come from ``heads_inputs`` below (also imported by the tests).
"""

from __future__ import annotations

import argparse
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
sys.path.insert(0, HERE)

from opendde_b200.utils import seeded_params  # noqa: E402

N, C_Z, C_S_IN = 23, 32, 40
NB_DIST, MIN_BIN, MAX_BIN, THRES = 24, 2.25, 25.75, 8.0
B_PAE, B_PDE = 16, 24
C_ZD = 16                # c_z_pair_diffusion of the compressing case
R_MAX, S_MAX = 32, 2     # RelativePositionEncoding defaults (used by DiffusionConditioning)


def distogram_param_shapes(c_z=C_Z, nb=NB_DIST):
    return [("linear.weight", (nb, c_z)), ("linear.bias", (nb,))]


def confidence_param_shapes(c_z=C_Z, c_s_inputs=C_S_IN, b_pae=B_PAE, b_pde=B_PDE, n_dist=39):
    return [("linear_no_bias_s1.weight", (c_z, c_s_inputs)), ("linear_no_bias_s2.weight", (c_z, c_s_inputs)),
            ("linear_no_bias_d.weight", (c_z, n_dist)), ("linear_no_bias_d_wo_onehot.weight", (c_z, 1)),
            ("linear_no_bias_pae.weight", (b_pae, c_z)), ("linear_no_bias_pde.weight", (b_pde, c_z)),
            ("pae_ln.weight", (c_z,)), ("pae_ln.bias", (c_z,)), ("pde_ln.weight", (c_z,)), ("pde_ln.bias", (c_z,))]


def distance_bins(start=3.25, end=52.0, step=1.25):
    """lower / upper bins of ConfidenceHead (confidence.py:83-88)."""
    lower = torch.arange(start, end, step)
    upper = torch.cat([lower[1:], lower.new_tensor([1e6])], dim=-1)
    return lower, upper


def diffusion_param_shapes(c_z=C_Z, c_zd=C_ZD, r_max=R_MAX, s_max=S_MAX):
    n_feat = 4 * r_max + 2 * s_max + 7
    shapes = [("relpe.linear_no_bias.weight", (c_zd, n_feat)), ("layernorm_z.weight", (2 * c_zd,)),
              ("linear_no_bias_z.weight", (c_zd, 2 * c_zd))]
    if c_zd != c_z:
        shapes += [("layernorm_z_trunk.weight", (c_z,)), ("linear_no_bias_z_trunk.weight", (c_zd, c_z))]
    for t in ("transition_z1", "transition_z2"):
        shapes += [(f"{t}.layernorm1.weight", (c_zd,)), (f"{t}.layernorm1.bias", (c_zd,)),
                   (f"{t}.linear_no_bias_a.weight", (2 * c_zd, c_zd)),
                   (f"{t}.linear_no_bias_b.weight", (2 * c_zd, c_zd)),
                   (f"{t}.linear_no_bias.weight", (c_zd, 2 * c_zd))]
    return shapes


def heads_inputs(n=N, c_z=C_Z, c_s_inputs=C_S_IN):
    """z (the stack's output), s_inputs, representative-atom coordinates spread over the distance
    bins (about 3 to 50 A), and the token ids of four chains (two copies of one entity)."""
    g = torch.Generator().manual_seed(7)
    z = torch.randn((n, n, c_z), generator=g)
    s_inputs = torch.randn((n, c_s_inputs), generator=g)
    coords = torch.randn((n, 3), generator=g) * 12.0
    asym = torch.tensor([0] * 8 + [1] * 6 + [2] * 6 + [3] * (n - 20))
    entity = torch.tensor([0] * 8 + [1] * 6 + [0] * 6 + [2] * (n - 20))
    sym = torch.tensor([0] * 8 + [0] * 6 + [1] * 6 + [0] * (n - 20))
    residue = torch.cat([torch.tensor([1, 2, 3, 3, 3, 4, 10, 11]), torch.arange(1, 7), torch.arange(1, 7),
                         torch.arange(1, n - 19)])
    feats = {"asym_id": asym, "residue_index": residue, "entity_id": entity, "token_index": torch.arange(n),
             "sym_id": sym}
    return z, s_inputs, coords, feats


def checksum(t: torch.Tensor) -> np.ndarray:
    t = t.double()
    return np.array([t.sum().item(), t.abs().sum().item(), (t * t).sum().item()])


# the reference modules' parameters outside the pair steps (single-representation / atom heads)
NON_PAIR_PREFIXES = ("pairformer_stack.", "plddt", "resolved", "input_strunk_ln.", "layernorm_s.",
                     "linear_no_bias_s.", "fourier_embedding.", "layernorm_n.", "linear_no_bias_n.",
                     "transition_s1.", "transition_s2.")


def pair_state_shapes(mod):
    """"name:shape" of a reference module's state_dict entries that belong to its pair steps."""
    return np.array([f"{k}:{'x'.join(str(d) for d in v.shape)}" for k, v in mod.state_dict().items()
                     if not k.startswith(NON_PAIR_PREFIXES)])


def _load(mod, params):
    sd = mod.state_dict()
    for k, v in params.items():
        sd[k].copy_(v)


@torch.no_grad()
def run_distogram():
    import torch.distributed as dist
    from opendde.distributed.foldcp.distogram import distogram_contact_probs_local
    from opendde.distributed.foldcp.pair_sharding import FoldCPPairShardSpec
    from opendde.model.modules.head import DistogramHead
    head = DistogramHead(c_z=C_Z, no_bins=NB_DIST)
    params = seeded_params(distogram_param_shapes(), seed=0, perturb_1d=True)
    _load(head, params)
    z, _, _, _ = heads_inputs()
    logits = head(z)
    if not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29561")
        dist.init_process_group("gloo", rank=0, world_size=1)
    layout = types.SimpleNamespace(shape=(1, 1), numel=1, transpose_rank=lambda coord: 0)
    mesh = types.SimpleNamespace(layout=layout, coord=(0, 0), cp_rank=0, cp_global_ranks=[0],
                                 group_2d=dist.group.WORLD)
    spec = FoldCPPairShardSpec(original_shape=(N, N, C_Z), padded_shape=(N, N, C_Z), pair_dims=(0, 1),
                               row_range=(0, N), col_range=(0, N), mesh_shape=(1, 1), mesh_coord=(0, 0))
    contact = distogram_contact_probs_local(z_pair_local=z, z_pair_spec=spec, mesh=mesh, linear=head.linear,
                                            min_bin=MIN_BIN, max_bin=MAX_BIN, no_bins=NB_DIST, thres=THRES)
    return params, {"logits": logits.numpy().astype(np.float32), "contact": contact.numpy().astype(np.float32),
                    "ref_state": pair_state_shapes(head)}


@torch.no_grad()
def run_confidence():
    from opendde.model.modules.confidence import ConfidenceHead
    head = ConfidenceHead(n_blocks=0, c_s=8, c_z=C_Z, c_s_inputs=C_S_IN, b_pae=B_PAE, b_pde=B_PDE,
                          max_atoms_per_token=2)
    params = seeded_params(confidence_param_shapes(), seed=1, perturb_1d=True)
    _load(head, params)
    z, s_inputs, coords, _ = heads_inputs()
    captured = {}

    def grab(_mod, args, kwargs):
        captured["z"] = (args[1] if len(args) > 1 else kwargs["z"]).clone()

    head.pairformer_stack.register_forward_pre_hook(grab, with_kwargs=True)
    feat = {"distogram_rep_atom_mask": torch.ones(N, dtype=torch.bool),
            "atom_to_token_idx": torch.arange(N), "atom_to_tokatom_idx": torch.zeros(N, dtype=torch.long)}
    _, pae, pde, _ = head(feat, s_inputs, torch.randn(N, 8), z, torch.ones(N, N), coords[None],
                          compute_plddt=False, compute_resolved=False)
    return params, {"z_pair": captured["z"].numpy().astype(np.float32), "pae": pae[0].numpy().astype(np.float32),
                    "pde": pde[0].numpy().astype(np.float32), "ref_state": pair_state_shapes(head)}


@torch.no_grad()
def run_diffusion(c_zd):
    from opendde.model.modules.diffusion import DiffusionConditioning
    from opendde.model.modules.embedders import RelativePositionEncoding
    mod = DiffusionConditioning(c_z=C_Z, c_z_pair_diffusion=c_zd, c_s=8, c_s_inputs=C_S_IN)
    params = seeded_params(diffusion_param_shapes(c_zd=c_zd), seed=2, perturb_1d=True)
    _load(mod, params)
    z, _, _, feats = heads_inputs()
    relp = RelativePositionEncoding(r_max=R_MAX, s_max=S_MAX, c_z=c_zd).generate_relp(dict(feats), lazy=False)["relp"]
    out = mod.prepare_cache(relp, z)
    return params, {"pair_z": out.numpy().astype(np.float32), "ref_state": pair_state_shapes(mod)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path to the OpenDDE source tree")
    args = ap.parse_args()
    sys.path.insert(0, os.path.abspath(args.reference))
    from make_golden import _stub_imports
    _stub_imports()
    z, s_inputs, coords, _ = heads_inputs()
    common = {"chk_z": checksum(z), "chk_s_inputs": checksum(s_inputs), "chk_coords": checksum(coords)}
    os.makedirs(os.path.join(HERE, "heads"), exist_ok=True)
    runs = [("distogram", run_distogram), ("confidence", run_confidence),
            ("diffusion_compress", lambda: run_diffusion(C_ZD)), ("diffusion_plain", lambda: run_diffusion(C_Z))]
    for name, fn in runs:
        params, rec = fn()
        rec["chk_params"] = np.stack([checksum(params[k]) for k in sorted(params)])
        rec["param_names"] = np.array(sorted(params))
        path = os.path.join(HERE, "heads", f"{name}_n{N}.npz")
        np.savez_compressed(path, **common, **rec)
        print("wrote", path, os.path.getsize(path))


if __name__ == "__main__":
    main()
