"""Fold-CP local construction of the trunk's pair input and its recycling update, drop-in for
opendde/distributed/foldcp/trunk_init.py:90-178 (``build_trunk_z_init_local``,
``apply_trunk_z_cycle_local``): each rank writes only its (padded) tile of z_init, from the
replicated s_init and the per-token ids; the full pair plane is never formed on any rank."""

from __future__ import annotations

from typing import Any, Tuple

import torch

from ...model.trunk_init import trunk_pair_cycle, trunk_pair_init_tile
from .mesh import FoldCPProcessMesh
from .pair_sharding import FoldCPPairShardSpec, make_pair_shard_spec


def build_trunk_z_init_local(*, s_init: torch.Tensor, linear_zinit1: torch.nn.Module,
                             linear_zinit2: torch.nn.Module, relative_position_encoding: torch.nn.Module,
                             linear_token_bond: torch.nn.Module, relp_feature: Any, token_bonds: torch.Tensor,
                             mesh: FoldCPProcessMesh) -> Tuple[torch.Tensor, FoldCPPairShardSpec]:
    """This rank's tile of z_init (zero past N) and its shard spec (pair dims -3, -2)."""
    n_token = int(s_init.shape[-2])
    c_z = int(linear_zinit1.weight.shape[0])
    spec = make_pair_shard_spec((*s_init.shape[:-2], n_token, n_token, c_z), mesh, pair_dims=(-3, -2))
    z_local = torch.zeros(spec.local_shape, device=s_init.device, dtype=s_init.dtype)
    (r0, r1), (c0, c1) = spec.row_range, spec.col_range
    vr, vc = min(r1, n_token) - r0, min(c1, n_token) - c0
    if vr > 0 and vc > 0:
        trunk_pair_init_tile(s_init, linear_zinit1, linear_zinit2, relative_position_encoding, linear_token_bond,
                             relp_feature, token_bonds, z_local[:vr, :vc], row0=r0, col0=c0)
    return z_local, spec


def apply_trunk_z_cycle_local(*, z_init_local: torch.Tensor, z_local: torch.Tensor,
                              layernorm_z_cycle: torch.nn.Module, linear_z_cycle: torch.nn.Module,
                              z_spec: FoldCPPairShardSpec) -> torch.Tensor:
    """z_init_local + linear_z_cycle(layernorm_z_cycle(z_local)) on the tile (a pointwise update:
    no exchange). The padded positions past N carry LN(0)-driven values as in the reference."""
    return trunk_pair_cycle(z_init_local, z_local, layernorm_z_cycle, linear_z_cycle)
