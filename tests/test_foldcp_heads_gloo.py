"""Fold-CP pair heads and pair conditioning over real torch.distributed process groups (gloo, CPU
ranks): the transposed-rectangle region request of the symmetric heads (distogram, pde), the local
pair input of the confidence head, the local diffusion conditioning and the final gathers, on
square and non-square meshes with padded tiles. The per-tile math is the oracle
(``OracleHeadOps``); the kernels behind the same calls are checked on the GPU
(tests/test_gpu_heads.py)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

C_Z, C_S_IN, NB, B_PAE, B_PDE, C_ZD = 16, 24, 20, 12, 10, 8


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class OracleHeadOps:
    """The HeadKernels calls restated with the oracle (fp32, CPU)."""

    def __init__(self, O, p_dist, p_conf, p_diff, feats, r_max, s_max):
        self.O, self.p_dist, self.p_conf, self.p_diff = O, p_dist, p_conf, p_diff
        self.feats, self.r_max, self.s_max = feats, r_max, s_max

    def distogram(self, head, z, zt, logits, contact, contact_bins):
        O, p = self.O, self.p_dist
        y = O.linear(z, p["linear.weight"], p["linear.bias"]) + O.linear(zt, p["linear.weight"], p["linear.bias"])
        logits.copy_(y)
        contact.copy_(torch.softmax(y, -1)[..., :contact_bins].sum(-1))

    def confidence_logits(self, head, z, zt, pae, pde):
        O, p = self.O, self.p_conf
        if pae is not None:
            pae.copy_(O.linear(O.layer_norm(z, p["pae_ln.weight"], p["pae_ln.bias"]), p["linear_no_bias_pae.weight"]))
        if pde is not None:
            pde.copy_(O.linear(O.layer_norm(z + zt, p["pde_ln.weight"], p["pde_ln.bias"]),
                               p["linear_no_bias_pde.weight"]))

    def confidence_embed(self, head, s_inputs, coords, z_tile, row0, col0):
        r, c = z_tile.shape[:2]
        z_tile.copy_(self.O.confidence_pair_init(z_tile.clone(), s_inputs, coords, self.p_conf,
                                                 rows=slice(row0, row0 + r), cols=slice(col0, col0 + c)))

    def diffusion(self, module, relp_feature, z_tile, out, row0, col0):
        r, c = z_tile.shape[:2]
        out.copy_(self.O.diffusion_pair_conditioning(z_tile, self.feats, self.p_diff, self.r_max, self.s_max,
                                                     rows=slice(row0, row0 + r), cols=slice(col0, col0 + c)))


def _worker(rank, world, port, shape, n):
    import sys
    sys.path.insert(0, os.path.dirname(__file__))
    sys.path.insert(0, os.path.dirname(os.path.dirname(__file__)))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    try:
        from oracle import pairformer_oracle as O
        from opendde_b200.distributed.foldcp import (FoldCPConfig, FoldCPProcessMesh, clear_mesh_cache,
                                                      confidence_pair_input_local, diffusion_prepare_cache_local,
                                                      distributed_confidence_pair_logits,
                                                      distributed_distogram_contact_probs, shard_pair_tensor)
        from opendde_b200.model import ConfidencePairHead, DiffusionPairConditioning, DistogramHead
        from opendde_b200.model.trunk_init import LazyRelativePositionEncodingFeatures
        from opendde_b200.utils import seeded_params

        cfg = FoldCPConfig.from_runtime_args(mode="distributed", size_cp=world, mesh=f"{shape[0]}x{shape[1]}")
        mesh = FoldCPProcessMesh.create(cfg)
        g = torch.Generator().manual_seed(3)
        z = torch.randn((n, n, C_Z), generator=g)
        s_inputs = torch.randn((n, C_S_IN), generator=g)
        coords = torch.randn((n, 3), generator=g) * 12.0
        feats = {"asym_id": torch.tensor([0] * (n // 2) + [1] * (n - n // 2)), "residue_index": torch.arange(n),
                 "entity_id": torch.zeros(n, dtype=torch.long), "token_index": torch.arange(n),
                 "sym_id": torch.tensor([0] * (n // 2) + [1] * (n - n // 2))}
        dh = DistogramHead(c_z=C_Z, no_bins=NB)
        ch = ConfidencePairHead(c_z=C_Z, c_s_inputs=C_S_IN, b_pae=B_PAE, b_pde=B_PDE)
        dc = DiffusionPairConditioning(c_z=C_Z, c_z_pair_diffusion=C_ZD)
        ps = []
        for i, m in enumerate((dh, ch, dc)):
            named = [(k, tuple(v.shape)) for k, v in m.named_parameters() if v.requires_grad]
            p = seeded_params(named, seed=i, perturb_1d=True)
            p.update({k: v.detach().clone() for k, v in m.named_parameters() if not v.requires_grad})
            ps.append(p)
        ops = OracleHeadOps(O, ps[0], ps[1], ps[2], feats, 32, 2)
        local, spec = shard_pair_tensor(z, mesh, pair_dims=(0, 1))

        # distogram contact probabilities (symmetric: the transposed rectangle crosses ranks)
        want = O.contact_probs(O.distogram_logits(z, ps[0]), 2.25, 25.75, NB, 8.0)
        got = distributed_distogram_contact_probs(z_pair_local=local, z_pair_spec=spec, mesh=mesh, head=dh,
                                                  min_bin=2.25, max_bin=25.75, no_bins=NB, ops=ops)
        assert got.shape == (n, n) and (got - want).abs().max().item() <= 1e-5
        got0 = distributed_distogram_contact_probs(z_pair_local=local, z_pair_spec=spec, mesh=mesh, head=dh,
                                                   min_bin=2.25, max_bin=25.75, no_bins=NB, ops=ops,
                                                   gather_to_rank0_only=True)
        assert (got0 is None) == (rank != 0)
        if got0 is not None:
            assert torch.equal(got0, got)

        # confidence pae / pde
        pae_w, pde_w = O.confidence_pair_logits(z, ps[1])
        pae, pde = distributed_confidence_pair_logits(head=ch, z_pair_local=local, z_pair_spec=spec, mesh=mesh,
                                                      ops=ops)
        assert (pae - pae_w).abs().max().item() <= 1e-4 and (pde - pde_w).abs().max().item() <= 1e-4
        none, pde_only = distributed_confidence_pair_logits(head=ch, z_pair_local=local, z_pair_spec=spec,
                                                            mesh=mesh, compute_pae=False, ops=ops)
        assert none is None and torch.equal(pde_only, pde)

        # confidence pair input on the tile (in place; padding untouched)
        want_in, _ = shard_pair_tensor(O.confidence_pair_init(z, s_inputs, coords, ps[1]), mesh, pair_dims=(0, 1))
        loc = local.clone()
        confidence_pair_input_local(head=ch, s_inputs=s_inputs, x_pred_rep_coords=coords, z_trunk_local=loc,
                                    z_spec=spec, ops=ops)
        assert (loc - want_in).abs().max().item() <= 1e-4

        # diffusion conditioning on the tile
        relp = LazyRelativePositionEncodingFeatures(*[feats[k] for k in ("asym_id", "residue_index", "entity_id",
                                                                          "token_index", "sym_id")], 32, 2)
        want_d, want_spec = shard_pair_tensor(O.diffusion_pair_conditioning(z, feats, ps[2]), mesh, pair_dims=(0, 1))
        out, out_spec = diffusion_prepare_cache_local(dc, relp, local, spec, mesh, ops=ops)
        assert out_spec == want_spec and (out - want_d).abs().max().item() <= 1e-4
        clear_mesh_cache()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("shape,n", [((1, 2), 13), ((2, 2), 10), ((2, 1), 9)])
def test_foldcp_heads_gloo_match_serial(shape, n):
    world = shape[0] * shape[1]
    mp.spawn(_worker, args=(world, _free_port(), shape, n), nprocs=world, join=True)
