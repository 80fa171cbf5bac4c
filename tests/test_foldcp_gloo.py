"""Fold-CP over real torch.distributed process groups (gloo, CPU ranks).

Exercises the process-group plumbing the GPU path uses with NCCL: the cached R x C mesh
(2D, row and column groups), the point-to-point band exchanges, the all-gathers of bias
tiles and single rows, and the final pair gather; local band math is the oracle.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

C_Z, C_S, HEADS = 16, 32, 4


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, shape, n):
    import sys
    sys.path.insert(0, os.path.dirname(__file__))
    sys.path.insert(0, os.path.dirname(os.path.dirname(__file__)))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    try:
        from foldcp_support import OracleBandOps
        from oracle import pairformer_oracle as O
        from opendde_b200.distributed.foldcp import (FoldCPConfig, FoldCPProcessMesh, clear_mesh_cache,
                                                      distributed_pairformer_stack_single_bridge_update,
                                                      gather_pair_tensor, shard_pair_tensor)
        from opendde_b200.model import PairformerStack
        from opendde_b200.utils import ragged_pair_mask, seeded_params

        cfg = FoldCPConfig.from_runtime_args(mode="distributed", size_cp=world, mesh=f"{shape[0]}x{shape[1]}")
        mesh = FoldCPProcessMesh.create(cfg)
        assert FoldCPProcessMesh.create(cfg) is mesh          # cached, no new groups
        assert mesh.coord == divmod(rank, shape[1])

        st = PairformerStack(n_blocks=2, n_heads=HEADS, c_z=C_Z, c_s=C_S)
        p = seeded_params([(k, tuple(v.shape)) for k, v in st.named_parameters()], seed=0, perturb_1d=True)
        with torch.no_grad():
            for k, v in st.named_parameters():
                v.copy_(p[k])
        g = torch.Generator().manual_seed(1)
        z = torch.randn((n, n, C_Z), generator=g)
        s = torch.randn((n, C_S), generator=g)
        mask = ragged_pair_mask(n, seed=3, drop=0.2, full_rows=[1])
        with torch.no_grad():
            s_ref, z_ref = O.pairformer_stack(s, z, mask, p, 2, no_heads_pair=4, n_heads=HEADS, c_s=C_S)
            s_out, z_out = distributed_pairformer_stack_single_bridge_update(st, s.clone(), z, mesh, pair_mask=mask,
                                                                             ops=OracleBandOps())
        assert (z_out - z_ref).abs().max().item() <= 1e-4
        assert (s_out - s_ref).abs().max().item() <= 1e-4
        # shard -> gather round trip of a pair tensor
        local, spec = shard_pair_tensor(z, mesh, pair_dims=(0, 1))
        assert torch.equal(gather_pair_tensor(local, spec, mesh.group_2d), z)
        clear_mesh_cache()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("shape,n", [((1, 2), 13), ((2, 2), 10), ((2, 4), 13)])
def test_foldcp_gloo_stack_matches_serial(shape, n):
    world = shape[0] * shape[1]
    mp.spawn(_worker, args=(world, _free_port(), shape, n), nprocs=world, join=True)
