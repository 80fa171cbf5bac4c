"""Entry from the modules' forward under ``OPENDDE_FOLDCP_MODE=distributed`` (the reference's
PairformerStack / PairformerBlock Fold-CP hooks, opendde/model/modules/pairformer.py:116-155
and :402-437): take the full (replicated) inputs, run the stack on this rank's tile, return
the full outputs."""

from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist

from ... import _abi
from .config import FoldCPConfig
from .mesh import FoldCPProcessMesh
from .pair_sharding import shard_pair_tensor
from .real_pairformer import (
    distributed_pairformer_block_pair_update,
    distributed_pairformer_stack_pair_update,
    distributed_pairformer_stack_single_bridge_update,
    gather_full,
    make_context,
)


def current_mesh() -> FoldCPProcessMesh:
    """The (cached) mesh of the launch configuration in ``OPENDDE_FOLDCP_*``."""
    return FoldCPProcessMesh.create(FoldCPConfig.from_env(dist.get_world_size()))


def _check(z: torch.Tensor) -> None:
    if z.dim() != 3:
        raise ValueError("Fold-CP takes an unbatched [N, N, c_z] pair tensor")
    if not z.is_cuda:
        raise RuntimeError("opendde_b200 Fold-CP needs CUDA tensors; there is no CPU fallback")


def stack_forward(stack, s: Optional[torch.Tensor], z: torch.Tensor, pair_mask: Optional[torch.Tensor],
                  extra_attn_bias: Optional[torch.Tensor] = None, chunk_size: Optional[int] = None):
    _check(z)
    mesh = current_mesh()
    if s is not None and stack.blocks and getattr(stack.blocks[0], "c_s", 0) > 0:
        out = distributed_pairformer_stack_single_bridge_update(
            stack, s, z, mesh, pair_mask=pair_mask, extra_attn_bias=extra_attn_bias)
        _abi.status_checkpoint(z.device)
        return out
    z_local, spec = shard_pair_tensor(z, mesh, pair_dims=(-3, -2))
    ctx = make_context(mesh, z_local, spec, mask_full=pair_mask)
    z_local = distributed_pairformer_stack_pair_update(stack, z_local, mesh, context=ctx)
    out = s, gather_full(z_local, ctx)
    _abi.status_checkpoint(z.device)
    return out


def block_pair_only(block, s: Optional[torch.Tensor], z: torch.Tensor, pair_mask: Optional[torch.Tensor],
                    chunk_size: Optional[int] = None):
    _check(z)
    mesh = current_mesh()
    z_local, spec = shard_pair_tensor(z, mesh, pair_dims=(-3, -2))
    ctx = make_context(mesh, z_local, spec, mask_full=pair_mask)
    z_local = distributed_pairformer_block_pair_update(block, z_local, mesh, context=ctx)
    out = s, gather_full(z_local, ctx)
    _abi.status_checkpoint(z.device)
    return out
