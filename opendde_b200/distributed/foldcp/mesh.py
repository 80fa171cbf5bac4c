"""Fold-CP process mesh (drop-in for opendde/distributed/foldcp/mesh.py:18-104), R x C.

``create`` builds the 2D, row and column process groups once per (world, config) and
caches them: the reference rebuilds them on every module call (pairformer.py:132-139),
which costs 1 + R + C ``new_group`` rendezvous per call.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, Tuple

import torch
import torch.distributed as dist

from .config import FoldCPConfig
from .layout import FoldCP2DLayout

_CACHE: Dict[tuple, "FoldCPProcessMesh"] = {}


@dataclass(frozen=True)
class FoldCPProcessMesh:
    config: FoldCPConfig
    layout: FoldCP2DLayout
    group_2d: "dist.ProcessGroup"
    group_row: "dist.ProcessGroup"
    group_col: "dist.ProcessGroup"
    cp_global_ranks: Tuple[int, ...]
    cp_rank: int
    coord: Tuple[int, int]

    @classmethod
    def create(cls, config: FoldCPConfig) -> "FoldCPProcessMesh":
        if not config.enabled:
            raise ValueError("FoldCPProcessMesh.create requires distributed mode.")
        if not dist.is_available() or not dist.is_initialized():
            raise RuntimeError("torch.distributed must be initialized first.")
        world_size = dist.get_world_size()
        if world_size != config.size_dp * config.size_cp:
            raise ValueError("WORLD_SIZE must equal foldcp_size_dp * foldcp_size_cp; "
                             f"got {world_size} vs {config.size_dp} * {config.size_cp}.")
        key = (id(dist.group.WORLD), world_size, config.size_dp, config.size_cp, config.cp_mesh_shape)
        hit = _CACHE.get(key)
        if hit is not None:
            return hit

        rows, cols = config.cp_mesh_shape
        layout = FoldCP2DLayout((rows, cols))
        world_rank = dist.get_rank()
        dp_index = world_rank // config.size_cp
        cp_offset = dp_index * config.size_cp
        cp_rank = world_rank - cp_offset
        coord = layout.to_coord(cp_rank)
        sel_2d = sel_row = sel_col = None
        # every rank creates every group in the same order
        for dp in range(config.size_dp):
            off = dp * config.size_cp
            g = dist.new_group(list(range(off, off + config.size_cp)))
            if dp == dp_index:
                sel_2d = g
            for r in range(rows):
                g = dist.new_group([off + layout.to_linear((r, c)) for c in range(cols)])
                if dp == dp_index and r == coord[0]:
                    sel_row = g
            for c in range(cols):
                g = dist.new_group([off + layout.to_linear((r, c)) for r in range(rows)])
                if dp == dp_index and c == coord[1]:
                    sel_col = g
        if sel_2d is None or sel_row is None or sel_col is None:
            raise RuntimeError("failed to create Fold-CP row/column groups.")
        mesh = cls(config=config, layout=layout, group_2d=sel_2d, group_row=sel_row, group_col=sel_col,
                   cp_global_ranks=tuple(range(cp_offset, cp_offset + config.size_cp)), cp_rank=cp_rank,
                   coord=coord)
        mesh._warm_up()
        _CACHE[key] = mesh
        return mesh

    def _warm_up(self) -> None:
        """One collective per group so that point-to-point batches later start on a live
        communicator (all ranks of the group take part)."""
        dev = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend(self.group_2d) == "nccl" \
            else torch.device("cpu")
        t = torch.zeros(1, device=dev)
        for g in (self.group_2d, self.group_row, self.group_col):
            dist.all_reduce(t, group=g)

    def global_rank(self, cp_rank: int) -> int:
        return self.cp_global_ranks[cp_rank]

    @property
    def shape(self) -> Tuple[int, int]:
        return self.layout.shape


def clear_mesh_cache() -> None:
    """Release the peer windows (collective) and forget cached meshes (call on every rank
    before ``destroy_process_group``)."""
    from .peer import release_windows
    release_windows()
    _CACHE.clear()
