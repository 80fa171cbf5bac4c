"""Fold-CP OuterProductMean: the pair tile a rank owns, computed from the replicated MSA
representation (drop-in for MSABlock._foldcp_outer_product_mean_local_update /
_outer_product_mean_tile_update, opendde/model/modules/pairformer.py:979-1059).

The reference computes the projections of every residue on every rank and then the einsum of
its tile; here ``pf_opm_fwd`` takes the tile's row / column offsets and forms only the tile's
outer products (the projections of the tile's rows and columns, one contraction over the
sequences, W_out). No exchange is needed: m is replicated on the mesh.
"""

from __future__ import annotations

from typing import Optional

import torch

from .mesh import FoldCPProcessMesh


def outer_product_mean_local_update(opm, m: torch.Tensor, mesh: FoldCPProcessMesh,
                                    mask: Optional[torch.Tensor] = None,
                                    chunk_size: Optional[int] = None) -> torch.Tensor:
    """This rank's [ceil(N/R), ceil(N/C), c_z] tile of the OuterProductMean update (zero past N).
    ``opm`` is an ``opendde_b200.model.OuterProductMean``; ``chunk_size`` is accepted for the
    reference's signature (nothing is chunked)."""
    return opm.tile_update(m, mesh.layout.shape, mesh.coord, mask=mask)
