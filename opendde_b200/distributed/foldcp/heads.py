"""Fold-CP pair heads and pair conditioning on the local tiles, drop-in for

* ``distributed_distogram_contact_probs`` / ``distogram_contact_probs_local``
  (opendde/distributed/foldcp/distogram.py:133-200),
* ``distributed_confidence_pair_logits`` (opendde/distributed/foldcp/confidence.py:329-394),
* the confidence head's local pair input: ``ConfidenceHead._build_confidence_z_init_local``
  (opendde/model/modules/confidence.py:177-202) and ``add_confidence_distance_embedding_local``
  (foldcp/confidence.py:81-148), one kernel pass here,
* ``DiffusionConditioning.prepare_cache_foldcp_local`` (opendde/model/modules/diffusion.py:906-1017).

The symmetric forms (distogram, pde) need z^T at the tile's positions. The reference sends the
transposed tile between transpose ranks (a square mesh; distogram.py:22-50 broadcasts every tile);
here it is one region request for the rectangle (rows = this tile's columns, columns = its rows),
which the mesh's transport serves on any R x C grid (peer memory over NVLink on NCCL meshes,
point-to-point otherwise). The distogram and pde logits are then formed from z and z^T in one
kernel pass; no logits cross ranks until the final gather. The local pair input and the diffusion
conditioning are pointwise in the pair plane: no exchange.

``ops`` carries the kernel calls (``HeadKernels``); the CPU tests pass an object with the same
methods to run the exchange logic on gloo ranks.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch

from ...model.heads import contact_bin_count
from .mesh import FoldCPProcessMesh
from .pair_sharding import FoldCPPairShardSpec, gather_pair_tensor_like, gather_pair_tensor_like_to_rank
from .real_pairformer import default_exchange


class HeadKernels:
    """The library's kernels behind the drivers below."""

    def distogram(self, head, z, zt, logits, contact, contact_bins: int) -> None:
        head.logits_tile(z, zt, logits, contact, contact_bins)

    def confidence_logits(self, head, z, zt, pae, pde) -> None:
        head.pair_logits_tile(z, zt, pae, pde)

    def confidence_embed(self, head, s_inputs, coords, z_tile, row0: int, col0: int) -> None:
        head.embed_pair_tile(s_inputs, coords, z_tile, z_tile, row0, col0)

    def diffusion(self, module, relp_feature, z_tile, out, row0: int, col0: int) -> None:
        module.prepare_cache_tile(relp_feature, z_tile, out, row0, col0)


def _valid(spec: FoldCPPairShardSpec) -> Tuple[int, int]:
    n = spec.n_token
    (r0, r1), (c0, c1) = spec.row_range, spec.col_range
    return max(0, min(r1, n) - r0), max(0, min(c1, n) - c0)


def transposed_tile(ex, z_local: torch.Tensor, spec: FoldCPPairShardSpec) -> torch.Tensor:
    """[Tr, Tc, ...] view of z^T at this tile's positions: the rectangle (rows = this tile's
    column range, columns = its row range) of the padded plane, fetched by one region request
    and viewed transposed. Every rank of the mesh must call it (it is a collective step)."""
    region = ex.region(z_local, spec, lambda c: (spec.col_range_of(c[1]), spec.row_range_of(c[0])))
    return region.transpose(0, 1)


def _gather(local: torch.Tensor, spec: FoldCPPairShardSpec, mesh, rank0_only: bool) -> Optional[torch.Tensor]:
    if rank0_only:
        return gather_pair_tensor_like_to_rank(local, spec, mesh.group_2d, 0)
    return gather_pair_tensor_like(local, spec, mesh.group_2d)


def distogram_contact_probs_local(*, z_pair_local: torch.Tensor, z_pair_spec: FoldCPPairShardSpec,
                                  mesh: FoldCPProcessMesh, head, min_bin: float, max_bin: float, no_bins: int,
                                  thres: float = 8.0, exchange=None, ops=None) -> torch.Tensor:
    """[Tr, Tc] fp32 contact probabilities of this rank's tile (zero past N)."""
    ex = exchange if exchange is not None else default_exchange(mesh)
    ops = ops if ops is not None else HeadKernels()
    zt = transposed_tile(ex, z_pair_local, z_pair_spec)
    vr, vc = _valid(z_pair_spec)
    contact = torch.zeros(z_pair_local.shape[:2], device=z_pair_local.device, dtype=torch.float32)
    if vr and vc:
        logits = torch.empty((vr, vc, no_bins), device=z_pair_local.device, dtype=z_pair_local.dtype)
        ops.distogram(head, z_pair_local[:vr, :vc], zt[:vr, :vc], logits, contact[:vr, :vc],
                      contact_bin_count(min_bin, max_bin, no_bins, thres, z_pair_local.dtype))
    return contact


def distributed_distogram_contact_probs(*, z_pair_local: torch.Tensor, z_pair_spec: FoldCPPairShardSpec,
                                        mesh: FoldCPProcessMesh, head, min_bin: float, max_bin: float, no_bins: int,
                                        thres: float = 8.0, gather_to_rank0_only: bool = False, exchange=None,
                                        ops=None) -> Optional[torch.Tensor]:
    """The [N, N] contact probabilities gathered on every rank (or on rank 0 only)."""
    local = distogram_contact_probs_local(z_pair_local=z_pair_local, z_pair_spec=z_pair_spec, mesh=mesh, head=head,
                                          min_bin=min_bin, max_bin=max_bin, no_bins=no_bins, thres=thres,
                                          exchange=exchange, ops=ops)
    full = _gather(local.unsqueeze(-1), z_pair_spec, mesh, gather_to_rank0_only)
    return None if full is None else full.squeeze(-1)


def confidence_pair_logits_local(*, head, z_pair_local: torch.Tensor, z_pair_spec: FoldCPPairShardSpec,
                                 mesh: FoldCPProcessMesh, compute_pae: bool = True, compute_pde: bool = True,
                                 exchange=None, ops=None) -> Tuple[Optional[torch.Tensor], Optional[torch.Tensor]]:
    """This tile's fp32 pae / pde logits [Tr, Tc, bins] (zero past N). ``head``: a
    ``ConfidencePairHead`` (pae_ln, pde_ln, linear_no_bias_pae, linear_no_bias_pde)."""
    ex = exchange if exchange is not None else default_exchange(mesh)
    ops = ops if ops is not None else HeadKernels()
    zt = transposed_tile(ex, z_pair_local, z_pair_spec) if compute_pde else None
    vr, vc = _valid(z_pair_spec)
    shape, dev = z_pair_local.shape[:2], z_pair_local.device
    pae = torch.zeros(shape + (head.b_pae,), device=dev, dtype=torch.float32) if compute_pae else None
    pde = torch.zeros(shape + (head.b_pde,), device=dev, dtype=torch.float32) if compute_pde else None
    if vr and vc and (compute_pae or compute_pde):
        ops.confidence_logits(head, z_pair_local[:vr, :vc], zt[:vr, :vc] if zt is not None else None,
                              pae[:vr, :vc] if pae is not None else None, pde[:vr, :vc] if pde is not None else None)
    return pae, pde


def distributed_confidence_pair_logits(*, head, z_pair_local: torch.Tensor, z_pair_spec: FoldCPPairShardSpec,
                                       mesh: FoldCPProcessMesh, compute_pae: bool = True, compute_pde: bool = True,
                                       gather_to_rank0_only: bool = False, exchange=None, ops=None):
    """The [N, N, bins] pae / pde logits gathered on every rank (or on rank 0 only; the others
    get None for each)."""
    pae, pde = confidence_pair_logits_local(head=head, z_pair_local=z_pair_local, z_pair_spec=z_pair_spec, mesh=mesh,
                                            compute_pae=compute_pae, compute_pde=compute_pde, exchange=exchange,
                                            ops=ops)
    out = [None if t is None else _gather(t, z_pair_spec, mesh, gather_to_rank0_only) for t in (pae, pde)]
    return out[0], out[1]


def confidence_pair_input_local(*, head, s_inputs: torch.Tensor, x_pred_rep_coords: torch.Tensor,
                                z_trunk_local: torch.Tensor, z_spec: FoldCPPairShardSpec, ops=None) -> torch.Tensor:
    """z_trunk_local + the s_inputs projections + the distance embedding on this tile's valid
    positions, in place (padded positions keep z_trunk_local)."""
    ops = ops if ops is not None else HeadKernels()
    vr, vc = _valid(z_spec)
    if vr and vc:
        ops.confidence_embed(head, s_inputs, x_pred_rep_coords, z_trunk_local[:vr, :vc], z_spec.row_range[0],
                             z_spec.col_range[0])
    return z_trunk_local


def diffusion_prepare_cache_local(module, relp_feature, z_trunk_local: torch.Tensor, z_spec: FoldCPPairShardSpec,
                                  mesh: Optional[FoldCPProcessMesh] = None,
                                  ops=None) -> Tuple[torch.Tensor, FoldCPPairShardSpec]:
    """This rank's tile of the conditioned pair [Tr, Tc, c_zd] (zero past N) and its spec."""
    del mesh
    ops = ops if ops is not None else HeadKernels()
    c_zd = module.c_z_pair_diffusion
    out = torch.zeros(z_trunk_local.shape[:2] + (c_zd,), device=z_trunk_local.device, dtype=z_trunk_local.dtype)
    spec = FoldCPPairShardSpec(original_shape=z_spec.original_shape[:-1] + (c_zd,),
                               padded_shape=z_spec.padded_shape[:-1] + (c_zd,), pair_dims=z_spec.pair_dims,
                               row_range=z_spec.row_range, col_range=z_spec.col_range, mesh_shape=z_spec.mesh_shape,
                               mesh_coord=z_spec.mesh_coord)
    vr, vc = _valid(z_spec)
    if vr and vc:
        ops.diffusion(module, relp_feature, z_trunk_local[:vr, :vc], out[:vr, :vc], z_spec.row_range[0],
                      z_spec.col_range[0])
    return out, spec


__all__ = ["HeadKernels", "transposed_tile", "distogram_contact_probs_local", "distributed_distogram_contact_probs",
           "confidence_pair_logits_local", "distributed_confidence_pair_logits", "confidence_pair_input_local",
           "diffusion_prepare_cache_local"]
