"""Band exchanges between the R x C tiles of a Fold-CP pair tensor.

Every rank asks for one rectangle of the padded pair plane (a band of rows over all
columns, or a band of columns over all rows); each owner sends its tile's intersection
with that rectangle, point to point, in one grouped batch. This replaces the reference's
ring and transpose exchanges (opendde/distributed/foldcp/comm.py:26-184), which need a
square mesh: a band request works for any R x C grid, and the ending-node / incoming ops
read column bands through transposed views instead of transposing z across ranks.

An exchange object carries the transport: ``DistExchange`` runs over torch.distributed
(NCCL on GPUs, gloo on CPU): the band of a rank's own mesh row (or column) is an all-gather
over the row (column) group, the other bands are point-to-point batches. ``PeerExchange``
(``peer.py``, the default on NCCL meshes) serves the same requests from the peers' memory over
NVLink. The drivers ask for bands through ``gather_bands`` (and the peer transport's
projection / attention variants) and for collectives through ``all_gather``.
"""

from __future__ import annotations

from typing import Callable, List, Optional, Tuple

import torch
import torch.distributed as dist

from .layout import FoldCP2DLayout
from .pair_sharding import FoldCPPairShardSpec

Range = Tuple[int, int]
Region = Tuple[Range, Range]
Need = Callable[[Tuple[int, int]], Region]


def intersect(a: Range, b: Range) -> Optional[Range]:
    lo, hi = max(a[0], b[0]), min(a[1], b[1])
    return (lo, hi) if lo < hi else None


def tile_region(spec: FoldCPPairShardSpec, coord: Tuple[int, int]) -> Region:
    return spec.row_range_of(coord[0]), spec.col_range_of(coord[1])


def copy_intersection(out: torch.Tensor, out_region: Region, src: torch.Tensor, src_region: Region) -> None:
    """out[overlap] = src[overlap] for two rectangles of the pair plane."""
    ir = intersect(out_region[0], src_region[0])
    ic = intersect(out_region[1], src_region[1])
    if ir is None or ic is None:
        return
    (o_r, o_c), (s_r, s_c) = (out_region[0][0], out_region[1][0]), (src_region[0][0], src_region[1][0])
    out[ir[0] - o_r:ir[1] - o_r, ic[0] - o_c:ic[1] - o_c] = src[ir[0] - s_r:ir[1] - s_r, ic[0] - s_c:ic[1] - s_c]


class DistExchange:
    """Transport over torch.distributed process groups of a FoldCPProcessMesh."""

    def __init__(self, mesh) -> None:
        self.mesh = mesh
        self.layout: FoldCP2DLayout = mesh.layout
        self.coord = mesh.coord

    def _group(self, axis: str):
        return {"2d": self.mesh.group_2d, "row": self.mesh.group_row, "col": self.mesh.group_col}[axis]

    def _size(self, axis: str) -> int:
        R, C = self.layout.shape
        return {"2d": R * C, "row": C, "col": R}[axis]

    def region(self, local: torch.Tensor, spec: FoldCPPairShardSpec, need: Need) -> torch.Tensor:
        """The rectangle ``need(coord)`` of the padded pair plane, assembled on this rank.

        ``local`` is this rank's tile [Tr, Tc, ...]; ``need`` gives every rank's request
        (each rank evaluates it for every peer, so no request travels).
        """
        mesh, layout = self.mesh, self.layout
        me = mesh.cp_rank
        mine = tile_region(spec, self.coord)
        want = need(self.coord)
        (nr0, nr1), (nc0, nc1) = want
        out = local.new_empty((nr1 - nr0, nc1 - nc0) + tuple(local.shape[2:]))
        ops: List[dist.P2POp] = []
        keep: List[torch.Tensor] = []
        recvs = []
        for q in range(layout.numel):
            qc = layout.to_coord(q)
            theirs = tile_region(spec, qc)
            if q == me:
                copy_intersection(out, want, local, mine)
                continue
            peer = mesh.global_rank(q)
            q_want = need(qc)
            sr, sc = intersect(mine[0], q_want[0]), intersect(mine[1], q_want[1])
            if sr and sc:
                piece = local[sr[0] - mine[0][0]:sr[1] - mine[0][0], sc[0] - mine[1][0]:sc[1] - mine[1][0]].contiguous()
                keep.append(piece)
                ops.append(dist.P2POp(dist.isend, piece, peer, mesh.group_2d))
            rr, rc = intersect(theirs[0], want[0]), intersect(theirs[1], want[1])
            if rr and rc:
                buf = local.new_empty((rr[1] - rr[0], rc[1] - rc[0]) + tuple(local.shape[2:]))
                ops.append(dist.P2POp(dist.irecv, buf, peer, mesh.group_2d))
                recvs.append((buf, (rr, rc)))
        if ops:
            for w in dist.batch_isend_irecv(ops):
                w.wait()
        for buf, reg in recvs:
            copy_intersection(out, want, buf, reg)
        del keep
        return out

    def all_gather(self, t: torch.Tensor, axis: str) -> torch.Tensor:
        """[n, *t.shape] stack of ``t`` from every rank of the 2D group ("2d", row-major rank
        order), of this rank's mesh row ("row", by column) or mesh column ("col", by row)."""
        group, n = self._group(axis), self._size(axis)
        t = t.contiguous()
        if dist.get_backend(group) == "nccl":
            flat = t.new_empty((n,) + tuple(t.shape))
            dist.all_gather_into_tensor(flat, t, group=group)
            return flat
        parts = [torch.empty_like(t) for _ in range(n)]
        dist.all_gather(parts, t, group=group)
        return torch.stack(parts, 0)


def own_row_band(ex, local: torch.Tensor) -> torch.Tensor:
    """This rank's mesh-row band (rows R_r x all padded columns), gathered over the row group
    (one all-gather of the tiles, then one reorder into row-major)."""
    t = ex.all_gather(local, "row")                     # [C, Tr, Tc, ...] by mesh column
    rest = tuple(range(3, t.dim()))
    return t.permute(1, 0, 2, *rest).reshape((t.shape[1], t.shape[0] * t.shape[2]) + tuple(t.shape[3:]))


def own_col_band(ex, local: torch.Tensor) -> torch.Tensor:
    """This rank's mesh-column band (all padded rows x columns C_c): the column group's tiles
    stacked by mesh row are already that band, so the all-gather output is used as is."""
    t = ex.all_gather(local, "col")                     # [R, Tr, Tc, ...] by mesh row
    return t.reshape((t.shape[0] * t.shape[1],) + tuple(t.shape[2:]))


def gather_bands(ex, local: torch.Tensor, spec: FoldCPPairShardSpec, requests) -> List[torch.Tensor]:
    """The bands of ``requests`` from one state of ``local``, each request one of
    ("own_rows",), ("own_cols",) (this rank's mesh row / column band), ("rows", rows_of) or
    ("cols", cols_of). Transports with a ``bands`` method serve them all from one snapshot;
    otherwise own bands are all-gathers over the row / column group and the others
    point-to-point regions."""
    full = (0, spec.n_padded)

    def need_of(req):
        kind = req[0]
        if kind == "own_rows":
            return lambda c: (spec.row_range_of(c[0]), full)
        if kind == "own_cols":
            return lambda c: (full, spec.col_range_of(c[1]))
        if kind == "rows":
            return lambda c, f=req[1]: (f(c), full)
        if kind == "cols":
            return lambda c, f=req[1]: (full, f(c))
        raise ValueError(f"unknown band request {kind!r}")

    if hasattr(ex, "bands"):
        return ex.bands(local, spec, [need_of(r) for r in requests])
    out = []
    for req in requests:
        if req[0] == "own_rows":
            out.append(own_row_band(ex, local))
        elif req[0] == "own_cols":
            out.append(own_col_band(ex, local))
        else:
            out.append(ex.region(local, spec, need_of(req)))
    return out
