"""Fold-CP pair-stack drivers on an R x C mesh (drop-in for the entry points of
opendde/distributed/foldcp/real_pairformer.py: distributed_triangle_multiplication_update
:1226, distributed_pair_transition_update :1405, distributed_attention_pair_bias_update :1714,
distributed_triangle_attention_update :2633, distributed_pairformer_block_pair_update :2757,
distributed_pairformer_stack_pair_update :2818, distributed_pairformer_stack_single_bridge_update
:2841; same arguments and return values).

Rank (r, c) holds the pair tile rows R_r = [r*Tr, (r+1)*Tr) x columns C_c = [c*Tc, (c+1)*Tc)
of the zero-padded [Np, Np] plane. Per op it exchanges the bands the op reads and runs one
library call on strided views, accumulating into its tile in place:

  triangle mult. outgoing   x_ij = sum_k a_ik b_jk   rows R_r of z (a), rows C_c of z (b)
  triangle mult. incoming   x_ij = sum_k a_ki b_kj   columns R_r of z (a), columns C_c (b)
  triangle attn. starting   rows R_r of z (keys = all columns), queries C_c
  triangle attn. ending     columns C_c of z read transposed (keys = all rows), queries R_r
  pair transition           local
  pair bias (attn. bias)    local tiles, all-gathered: H x Np x Np values, f16 in bf16 mode

The ending / incoming ops never transpose z across ranks (the reference's
``comm_2d_trans.exchange`` round trip, real_pairformer.py:2718-2744, needs a square mesh):
they read a column band through a transposed view. The pair mask is kept whole on every
rank ([Np, Np] fp32) since every op reads a band of it.

The single representation s is replicated; each rank runs the AttentionPairBias rows of a
1/(R*C) share of the tokens (its tile row's bias rows are gathered over the mesh row: 16
bias channels instead of the 128 z channels the reference gathers, real_pairformer.py:1747),
then the rows are all-gathered.
"""

from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Optional, Tuple

import torch
import torch.distributed as dist

from .exchange import DistExchange, gather_bands
from .layout import FoldCP2DLayout
from .mesh import FoldCPProcessMesh
from .ops import KernelOps
from .pair_sharding import FoldCPPairShardSpec, _spec_for, gather_pair_tensor, shard_pair_tensor

_DEFAULT_OPS = None


def _ops(ops):
    global _DEFAULT_OPS
    if ops is not None:
        return ops
    if _DEFAULT_OPS is None:
        _DEFAULT_OPS = KernelOps()
    return _DEFAULT_OPS


# ------------------------------------------------------------------------------ context

@dataclass
class FoldCPPairContext:
    """Geometry of this rank's tile, the whole padded pair mask and the transport; built
    once per stack call."""

    exchange: object  # DistExchange (or any object with .layout, .coord, .region, .all_gather)
    spec: FoldCPPairShardSpec
    mask: torch.Tensor  # [Np, Np] float32, zero outside the valid N x N block

    @property
    def layout(self) -> FoldCP2DLayout:
        return self.exchange.layout

    @property
    def coord(self) -> Tuple[int, int]:
        return self.exchange.coord

    @property
    def n(self) -> int:
        return self.spec.n_token

    @property
    def n_pad(self) -> int:
        return self.spec.n_padded

    @property
    def rows(self) -> Tuple[int, int]:
        return self.spec.row_range

    @property
    def cols(self) -> Tuple[int, int]:
        return self.spec.col_range


def _spec_from_local(z_local: torch.Tensor, layout: FoldCP2DLayout, coord) -> FoldCPPairShardSpec:
    """Geometry of an unpadded tiling when the caller gives no spec."""
    R, C = layout.shape
    n_pad = z_local.shape[0] * R
    if z_local.shape[1] * C != n_pad:
        raise ValueError(f"local tile {tuple(z_local.shape[:2])} does not tile a square plane on a {R}x{C} mesh")
    shape = (n_pad, n_pad) + tuple(z_local.shape[2:])
    return _spec_for(shape, layout.shape, coord, (0, 1))


def _full_mask(ex, spec, mask_full: Optional[torch.Tensor], mask_local: Optional[torch.Tensor],
               device) -> torch.Tensor:
    n, n_pad = spec.n_token, spec.n_padded
    out = torch.zeros((n_pad, n_pad), device=device, dtype=torch.float32)
    if mask_full is not None:
        out[:n, :n] = mask_full.to(device=device, dtype=torch.float32)
        return out
    if mask_local is None:
        out[:n, :n] = 1.0
        return out
    tiles = ex.all_gather(mask_local.to(device=device, dtype=torch.float32), "2d")
    R, C = ex.layout.shape
    tr, tc = spec.tile_rows, spec.tile_cols
    out.view(R, tr, C, tc).copy_(tiles.view(R, C, tr, tc).permute(0, 2, 1, 3))
    out[n:, :] = 0.0
    out[:, n:] = 0.0
    return out


def default_exchange(mesh: FoldCPProcessMesh):
    """Peer-memory transport on NCCL meshes (unless OPENDDE_B200_FOLDCP_TRANSPORT=nccl), the
    torch.distributed transport otherwise."""
    from .peer import PeerExchange, transport_choice
    if transport_choice(dist.get_backend(mesh.group_2d)) == "peer":
        return PeerExchange(mesh)
    return DistExchange(mesh)


def make_context(mesh: FoldCPProcessMesh, z_local: torch.Tensor, z_spec: Optional[FoldCPPairShardSpec] = None,
                 mask_local: Optional[torch.Tensor] = None, mask_full: Optional[torch.Tensor] = None,
                 exchange=None) -> FoldCPPairContext:
    """Context over ``mesh`` (or over a given transport ``exchange``)."""
    ex = exchange if exchange is not None else default_exchange(mesh)
    spec = z_spec if z_spec is not None else _spec_from_local(z_local, ex.layout, ex.coord)
    return FoldCPPairContext(ex, spec, _full_mask(ex, spec, mask_full, mask_local, z_local.device))


# ------------------------------------------------------------------------------ bias planes

def _round8(x: int) -> int:
    return (x + 7) // 8 * 8


def _triatt_bias_plane(module, z_local: torch.Tensor, ctx: FoldCPPairContext, ending: bool, ops) -> torch.Tensor:
    """[H, Np, ld] bias plane of the (transposed, for the ending node) pair tensor.

    Starting: plane[h, a, b] = bias of z(a, b). Ending (attention over x = z^T):
    plane[h, a, b] = bias of x(a, b) = bias of z(b, a). Each rank computes its tile, the
    tiles are all-gathered over the 2D group and placed; ld rounds Np up to 8 elements so
    every bias row starts 16-byte aligned (the tensor-core path loads it by TMA).
    """
    spec = ctx.spec
    R, C = ctx.layout.shape
    tr, tc, n_pad = spec.tile_rows, spec.tile_cols, spec.n_padded
    H = module.no_heads
    bdt = ops.bias_dtype(z_local.dtype)
    view = z_local.transpose(0, 1) if ending else z_local
    tile = torch.empty((H, view.shape[0], view.shape[1]), device=z_local.device, dtype=bdt)
    ops.triatt_bias(module, view, tile)
    tiles = ctx.exchange.all_gather(tile, "2d")
    ld = _round8(n_pad)
    plane = torch.empty((H, n_pad, ld), device=z_local.device, dtype=bdt)
    body = plane[:, :, :n_pad]
    if ending:
        body.view(H, C, tc, R, tr).copy_(tiles.view(R, C, H, tc, tr).permute(2, 1, 3, 0, 4))
    else:
        body.view(H, R, tr, C, tc).copy_(tiles.view(R, C, H, tr, tc).permute(2, 0, 3, 1, 4))
    return plane


# ------------------------------------------------------------------------------ per-op drivers

OVERLAP_KEY = "OPENDDE_B200_FOLDCP_OVERLAP"


def overlap_chunks() -> int:
    """Row chunks of the overlapped band exchanges of triangle attention and the triangle update
    (``OPENDDE_B200_FOLDCP_OVERLAP``; 0 or 1: one band per op, the default). The overlap is real
    with the copy-engine transport (``OPENDDE_B200_FOLDCP_COPY=dma``); band-copy kernels wait
    for the persistent kernels' SMs."""
    v = os.environ.get(OVERLAP_KEY, "").strip()
    if not v:
        return 0
    n = int(v)
    if n < 0:
        raise ValueError(f"{OVERLAP_KEY} must be a chunk count >= 0, got {v!r}")
    return n


def _row_of(spec):
    return lambda coord: spec.row_range_of(coord[0])


def _col_of(spec):
    return lambda coord: spec.col_range_of(coord[1])


def _trimul(module, z_local, ctx: FoldCPPairContext, ops) -> None:
    spec, ex, m = ctx.spec, ctx.exchange, ctx.mask
    (r0, r1), (c0, c1) = ctx.rows, ctx.cols
    if hasattr(ex, "trimul_bands") and hasattr(ops, "trimul_project"):
        # Exchange the projections (the reference's ring moves a_local / b_local too,
        # real_pairformer.py:1308-1384): each rank projects only its own tile. Incoming works
        # on x = z^T: a(i, k) = a(z(k, i)), so the tile is projected through a transposed view.
        mt = m[r0:r1, c0:c1]
        zt, mt = (z_local, mt) if module._outgoing else (z_local.transpose(0, 1), mt.t())
        chunks = overlap_chunks()
        if chunks > 1 and hasattr(ex, "trimul_chunks"):
            # the a band (output rows) in chunks: chunk i's copy on a side stream overlaps the
            # contraction and epilogue of chunk i-1 (every output row needs the whole b band)
            step = -(-(r1 - r0) // chunks)
            parts = [(a_, min(a_ + step, r1)) for a_ in range(r0, r1, step)]

            def consume(i, a_i, b_full, n_k):
                lo, hi = parts[i]
                rows = z_local[lo - r0:hi - r0]
                ops.trimul_combine(module, a_i, b_full, n_k, rows, rows)

            ex.trimul_chunks(z_local, spec, transposed=not module._outgoing, c_h=module.c_hidden,
                             project=lambda pa, pb, ld: ops.trimul_project(module, zt, mt, pa, pb, ld),
                             parts=parts, rows_b=(c0, c1), consume=consume)
            return
        a, b, n_k = ex.trimul_bands(
            z_local, spec, transposed=not module._outgoing, c_h=module.c_hidden,
            project=lambda pa, pb, ld: ops.trimul_project(module, zt, mt, pa, pb, ld),
            rows_a=(r0, r1), rows_b=(c0, c1))
        ops.trimul_combine(module, a, b, n_k, z_local, z_local)
        return
    if module._outgoing:
        # z rows R_r [Tr, Np, C] and z rows C_c [Tc, Np, C]
        za, zb = gather_bands(ex, z_local, spec, [("own_rows",), ("rows", _col_of(spec))])
        ma, mb = m[r0:r1], m[c0:c1]
    else:
        # z columns R_r and C_c, read transposed: (i, k) = z(k, i)
        za, zb = gather_bands(ex, z_local, spec, [("cols", _row_of(spec)), ("own_cols",)])
        za, zb = za.transpose(0, 1), zb.transpose(0, 1)
        ma, mb = m[:, r0:r1].t(), m[:, c0:c1].t()
    ops.trimul(module, za, zb, ma, mb, z_local, z_local)


def _triatt(module, z_local, ctx: FoldCPPairContext, ending: bool, ops) -> None:
    spec, ex, m = ctx.spec, ctx.exchange, ctx.mask
    (r0, r1), (c0, c1) = ctx.rows, ctx.cols
    n_pad = ctx.n_pad
    if hasattr(ex, "attention_bands"):
        # one snapshot of the tile and of its bias tile, one barrier, one copy launch: the z band
        # and only the bias rows of this rank's queries
        view = z_local.transpose(0, 1) if ending else z_local
        tile = torch.empty((module.no_heads, view.shape[0], view.shape[1]), device=z_local.device,
                           dtype=ops.bias_dtype(z_local.dtype))
        ops.triatt_bias(module, view, tile)
        full = (0, n_pad)
        chunks = overlap_chunks()
        if chunks > 1 and hasattr(ex, "attention_chunks"):
            # the attention rows (z rows R_r, or z columns C_c for the ending node) in chunks:
            # chunk i's band copy on a side stream overlaps chunk i-1's attention
            lo, hi = (c0, c1) if ending else (r0, r1)
            step = -(-(hi - lo) // chunks)
            parts = [(a, min(a + step, hi)) for a in range(lo, hi, step)]
            if not ending:
                needs = [lambda c, a=a, b=b: ((a, b), full) for a, b in parts]

                def consume(i, zs, bias):
                    a, b = parts[i]
                    ops.triatt(module, zs, m[a:b], bias[:, :, :n_pad], z_local[a - r0:b - r0], q_col0=c0,
                               n_q=c1 - c0, n_valid=ctx.n)
            else:
                needs = [lambda c, a=a, b=b: (full, (a, b)) for a, b in parts]

                def consume(i, zs, bias):
                    a, b = parts[i]
                    ops.triatt(module, zs.transpose(0, 1), m[:, a:b].t(), bias[:, :, :n_pad],
                               z_local[:, a - c0:b - c0].transpose(0, 1), q_col0=r0, n_q=r1 - r0, n_valid=ctx.n)
            ex.attention_chunks(z_local, spec, needs, tile, transposed=ending,
                                bias_rows=(r0, r1) if ending else (c0, c1), consume=consume)
            return
        if not ending:
            zs, bias = ex.attention_bands(z_local, spec, lambda c: (spec.row_range_of(c[0]), full), tile,
                                          transposed=False, bias_rows=(c0, c1))
            ops.triatt(module, zs, m[r0:r1], bias[:, :, :n_pad], z_local, q_col0=c0, n_q=c1 - c0, n_valid=ctx.n)
        else:
            zs, bias = ex.attention_bands(z_local, spec, lambda c: (full, spec.col_range_of(c[1])), tile,
                                          transposed=True, bias_rows=(r0, r1))
            ops.triatt(module, zs.transpose(0, 1), m[:, c0:c1].t(), bias[:, :, :n_pad], z_local.transpose(0, 1),
                       q_col0=r0, n_q=r1 - r0, n_valid=ctx.n)
        return
    plane = _triatt_bias_plane(module, z_local, ctx, ending, ops)
    if not ending:
        zs, = gather_bands(ex, z_local, spec, [("own_rows",)])   # rows R_r, keys = all columns
        ops.triatt(module, zs, m[r0:r1], plane[:, c0:c1, :n_pad], z_local, q_col0=c0, n_q=c1 - c0, n_valid=ctx.n)
    else:
        zs, = gather_bands(ex, z_local, spec, [("own_cols",)])
        zs = zs.transpose(0, 1)                                 # x rows C_c, keys = all rows of z
        ops.triatt(module, zs, m[:, c0:c1].t(), plane[:, r0:r1, :n_pad], z_local.transpose(0, 1),
                   q_col0=r0, n_q=r1 - r0, n_valid=ctx.n)


def _check_tile(z_local: torch.Tensor) -> None:
    if z_local.dim() != 3 or not z_local.is_contiguous():
        raise ValueError("Fold-CP pair ops take a contiguous [Tr, Tc, C] local tile")


def _in_place(z_local: torch.Tensor, residual_local: Optional[torch.Tensor]) -> bool:
    return residual_local is not None and (residual_local is z_local or (
        residual_local.data_ptr() == z_local.data_ptr() and residual_local.shape == z_local.shape and
        residual_local.stride() == z_local.stride()))


def _prepare(z_local, residual_local):
    """The tile the kernels accumulate into (the kernels add the update to it) and the input
    it started from when that is not the result: the update is fused into z_local itself when
    residual_local is z_local (the block's usage); otherwise a copy takes the update."""
    _check_tile(z_local)
    if _in_place(z_local, residual_local):
        return z_local, None
    return z_local.clone(), z_local


def _finish(work: torch.Tensor, residual_local: Optional[torch.Tensor], before: Optional[torch.Tensor]):
    """The reference returns residual + update when a residual is given, else the update."""
    if before is None:
        return work
    update = work - before
    return update if residual_local is None else residual_local + update


def distributed_triangle_multiplication_update(module, z_local: torch.Tensor, mesh: FoldCPProcessMesh,
                                               mask_local: Optional[torch.Tensor] = None,
                                               residual_local: Optional[torch.Tensor] = None,
                                               z_spec: Optional[FoldCPPairShardSpec] = None, *,
                                               ops=None, context: Optional[FoldCPPairContext] = None):
    """z_local + TriMul(z) on this rank's tile (update only when no residual is given)."""
    ops = _ops(ops)
    ctx = context or make_context(mesh, z_local, z_spec, mask_local)
    work, before = _prepare(z_local, residual_local)
    _trimul(module, work, ctx, ops)
    return _finish(work, residual_local, before)


def distributed_triangle_attention_update(module, z_local: torch.Tensor, mesh: FoldCPProcessMesh,
                                          mask_local: Optional[torch.Tensor] = None,
                                          residual_local: Optional[torch.Tensor] = None,
                                          z_spec: Optional[FoldCPPairShardSpec] = None,
                                          chunk_size: Optional[int] = None, *, ops=None,
                                          context: Optional[FoldCPPairContext] = None):
    """z_local + TriangleAttention(z) on this rank's tile; the module's ``starting`` flag picks
    the starting or ending node (the ending node without the reference's transposes)."""
    ops = _ops(ops)
    ctx = context or make_context(mesh, z_local, z_spec, mask_local)
    work, before = _prepare(z_local, residual_local)
    _triatt(module, work, ctx, not module.starting, ops)
    return _finish(work, residual_local, before)


def distributed_pair_transition_update(module, z_local: torch.Tensor, mesh: FoldCPProcessMesh,
                                       residual_local: Optional[torch.Tensor] = None,
                                       z_spec: Optional[FoldCPPairShardSpec] = None, *, ops=None):
    """z_local + Transition(z_local): pointwise, no communication."""
    ops = _ops(ops)
    work, before = _prepare(z_local, residual_local)
    ops.transition(module, work.view(-1, work.shape[-1]))
    return _finish(work, residual_local, before)


def _single_rows(ctx: FoldCPPairContext) -> Tuple[int, int, int]:
    """(first global query row, number of valid rows, rows per rank) of this rank's share of
    the single-attention queries: the tile's rows split over the mesh row's C ranks."""
    C = ctx.layout.shape[1]
    r0, r1 = ctx.rows
    per = -(-(r1 - r0) // C)
    q0 = r0 + ctx.coord[1] * per
    q1 = min(q0 + per, r1, ctx.n)
    return q0, max(0, q1 - q0), per


def distributed_attention_pair_bias_update(attention_pair_bias, a: torch.Tensor, z_local: torch.Tensor,
                                           mesh: FoldCPProcessMesh, z_spec: Optional[FoldCPPairShardSpec] = None,
                                           extra_attn_bias_local: Optional[torch.Tensor] = None, *,
                                           ops=None, context: Optional[FoldCPPairContext] = None,
                                           single_transition=None, extra_attn_bias_full: Optional[torch.Tensor] = None
                                           ) -> torch.Tensor:
    """The AttentionPairBias update of s (replicated [N, c_s]) from the pair tiles.

    Returns the update, like the reference; with ``single_transition`` given it returns the
    new s = s + APB + Transition(s + APB) instead (one gather per block instead of two).
    """
    if getattr(attention_pair_bias, "has_s", False):
        raise ValueError("Fold-CP AttentionPairBias currently supports has_s=False.")
    if a.ndim != 2 or z_local.ndim != 3:
        raise ValueError("Fold-CP AttentionPairBias expects a=[N,C] and z_local=[T,T,C].")
    ops = _ops(ops)
    ctx = context or make_context(mesh, z_local, z_spec)
    spec, layout = ctx.spec, ctx.layout
    R, C = layout.shape
    H = attention_pair_bias.n_heads
    n = a.shape[0]
    if n != ctx.n:
        raise ValueError(f"single representation has {n} tokens, the pair tiles {ctx.n}")
    tr, tc = spec.tile_rows, spec.tile_cols
    tile = torch.empty((H, tr, tc), device=z_local.device, dtype=torch.float32)
    ops.apb_pair_bias(attention_pair_bias, z_local, tile)
    if extra_attn_bias_full is None and extra_attn_bias_local is not None:
        # this rank's tile of the extra bias ([H or 1, Tr, Tc]) rides in the same row gather
        e = extra_attn_bias_local.to(device=tile.device, dtype=torch.float32)
        tile = tile + (e if e.dim() == 3 else e[None])[..., :tr, :tc]
    row_tiles = ctx.exchange.all_gather(tile, "row")                      # [C, H, Tr, Tc]
    q0, nq, per = _single_rows(ctx)
    lo = q0 - ctx.rows[0]
    a = a.contiguous()
    rows = a[q0:q0 + nq].clone() if single_transition is not None else torch.zeros_like(a[q0:q0 + nq])
    if nq > 0:
        bias_rows = row_tiles[:, :, lo:lo + nq, :].permute(1, 2, 0, 3).reshape(H, nq, C * tc)[:, :, :n]
        if extra_attn_bias_full is not None:
            e = extra_attn_bias_full.to(device=bias_rows.device, dtype=torch.float32)
            e = e if e.dim() == 3 else e[None]
            bias_rows = bias_rows + e[:, q0:q0 + nq, :n]
        bias_rows = bias_rows.contiguous()
        ops.apb_rows(attention_pair_bias, a, rows, bias_rows, q0)
        if single_transition is not None:
            ops.single_transition(single_transition, rows)
    # every rank's rows, padded to `per`, gathered over the whole CP group
    send = a.new_zeros((per, a.shape[1]))
    send[:nq] = rows
    allrows = ctx.exchange.all_gather(send, "2d")                          # [R*C, per, c_s]
    out = a.new_empty(a.shape) if single_transition is not None else torch.zeros_like(a)
    for rank in range(layout.numel):
        rr, cc = layout.to_coord(rank)
        g0 = spec.row_range_of(rr)[0] + cc * per
        g1 = min(g0 + per, spec.row_range_of(rr)[1], n)
        if g1 > g0:
            out[g0:g1] = allrows[rank, :g1 - g0]
    return out


# ------------------------------------------------------------------------------ block / stack

def _block_pair_ops(block, z_local: torch.Tensor, ctx: FoldCPPairContext, ops) -> torch.Tensor:
    _trimul(block.tri_mul_out, z_local, ctx, ops)
    _trimul(block.tri_mul_in, z_local, ctx, ops)
    _triatt(block.tri_att_start, z_local, ctx, False, ops)
    _triatt(block.tri_att_end, z_local, ctx, True, ops)
    ops.transition(block.pair_transition, z_local.view(-1, z_local.shape[-1]))
    return z_local


def distributed_pairformer_block_pair_update(block, z_local: torch.Tensor, mesh: FoldCPProcessMesh,
                                             pair_mask_local: Optional[torch.Tensor] = None,
                                             z_spec: Optional[FoldCPPairShardSpec] = None,
                                             chunk_size: Optional[int] = None, *, ops=None,
                                             context: Optional[FoldCPPairContext] = None) -> torch.Tensor:
    """The pair-only part of a PairformerBlock on a Fold-CP tile (updated in place)."""
    if getattr(block, "c_s", 0) != 0:
        raise ValueError("distributed_pairformer_block_pair_update currently requires c_s=0.")
    _check_tile(z_local)
    ctx = context or make_context(mesh, z_local, z_spec, pair_mask_local)
    return _block_pair_ops(block, z_local, ctx, _ops(ops))


def distributed_pairformer_stack_pair_update(stack, z_local: torch.Tensor, mesh: FoldCPProcessMesh,
                                             pair_mask_local: Optional[torch.Tensor] = None,
                                             z_spec: Optional[FoldCPPairShardSpec] = None,
                                             chunk_size: Optional[int] = None, *, ops=None,
                                             context: Optional[FoldCPPairContext] = None) -> torch.Tensor:
    """A c_s = 0 PairformerStack with the pair activations kept sharded."""
    z_local = z_local.contiguous()
    ctx = context or make_context(mesh, z_local, z_spec, pair_mask_local)
    ops = _ops(ops)
    for block in stack.blocks:
        if getattr(block, "c_s", 0) != 0:
            raise ValueError("distributed_pairformer_stack_pair_update currently requires c_s=0.")
        _block_pair_ops(block, z_local, ctx, ops)
    return z_local


def distributed_pairformer_stack_single_bridge_update(stack, s: torch.Tensor, z: torch.Tensor,
                                                      mesh: FoldCPProcessMesh,
                                                      pair_mask: Optional[torch.Tensor] = None,
                                                      extra_attn_bias: Optional[torch.Tensor] = None,
                                                      extra_attn_bias_is_local: bool = False,
                                                      return_local_pair: bool = False,
                                                      z_spec: Optional[FoldCPPairShardSpec] = None,
                                                      chunk_size: Optional[int] = None, *, ops=None,
                                                      context: Optional[FoldCPPairContext] = None):
    """A c_s > 0 PairformerStack: pair ops on Fold-CP tiles, single update from bias rows.

    ``z`` is the full pair tensor (or, with ``z_spec``, this rank's tile) and ``pair_mask``
    the full [N, N] mask. Returns (s, z) with z gathered, or (s, z_local, z_spec) when
    ``return_local_pair``.
    """
    if not stack.blocks:
        return (s, z, z_spec) if return_local_pair else (s, z)
    if getattr(stack.blocks[0], "c_s", 0) <= 0:
        raise ValueError("single bridge requires a PairformerStack with c_s > 0.")
    ops = _ops(ops)
    if z_spec is None:
        z_local, z_spec = shard_pair_tensor(z, mesh, pair_dims=(-3, -2))
        mask_full, mask_local = pair_mask, None
    else:
        z_local = z.contiguous()
        mask_full, mask_local = None, pair_mask
    ctx = context or make_context(mesh, z_local, z_spec, mask_local=mask_local, mask_full=mask_full)
    extra_full = None
    if extra_attn_bias is not None:
        if extra_attn_bias_is_local:
            from .pair_sharding import gather_pair_tensor_like
            dims = (extra_attn_bias.dim() - 2, extra_attn_bias.dim() - 1)
            espec = FoldCPPairShardSpec(
                original_shape=tuple(extra_attn_bias.shape[:-2]) + (ctx.n, ctx.n),
                padded_shape=tuple(extra_attn_bias.shape[:-2]) + (ctx.n_pad, ctx.n_pad), pair_dims=dims,
                row_range=z_spec.row_range, col_range=z_spec.col_range, mesh_shape=z_spec.mesh_shape,
                mesh_coord=z_spec.mesh_coord)
            extra_full = gather_pair_tensor_like(extra_attn_bias.contiguous(), espec, ctx.exchange.mesh.group_2d)
        else:
            extra_full = extra_attn_bias
    for block in stack.blocks:
        _block_pair_ops(block, z_local, ctx, ops)
        s = distributed_attention_pair_bias_update(block.attention_pair_bias, s, z_local, mesh, z_spec,
                                                   ops=ops, context=ctx, single_transition=block.single_transition,
                                                   extra_attn_bias_full=extra_full)
    if return_local_pair:
        return s, z_local, z_spec
    return s, gather_full(z_local, ctx)


def gather_full(z_local: torch.Tensor, ctx: FoldCPPairContext) -> torch.Tensor:
    """The full (cropped) pair tensor from every rank's tile."""
    spec = ctx.spec
    R, C = ctx.layout.shape
    tiles = ctx.exchange.all_gather(z_local, "2d")                      # [R*C, Tr, Tc, ...]
    tr, tc, n = spec.tile_rows, spec.tile_cols, spec.n_token
    rest = tuple(z_local.shape[2:])
    full = tiles.view((R, C, tr, tc) + rest).transpose(1, 2).reshape((R * tr, C * tc) + rest)
    return full[:n, :n].contiguous()


__all__ = [
    "FoldCPPairContext", "make_context", "gather_full",
    "distributed_triangle_multiplication_update", "distributed_triangle_attention_update",
    "distributed_pair_transition_update", "distributed_attention_pair_bias_update",
    "distributed_pairformer_block_pair_update", "distributed_pairformer_stack_pair_update",
    "distributed_pairformer_stack_single_bridge_update",
]
