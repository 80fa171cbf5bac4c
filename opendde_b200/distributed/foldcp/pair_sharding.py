"""2D pair-tensor sharding over an R x C Fold-CP mesh (drop-in for
opendde/distributed/foldcp/pair_sharding.py:19-356).

The pair plane [N, N] is zero-padded to Np = ceil(N / L) * L with L = lcm(R, C) and cut
into R x C tiles of Tr = Np / R rows and Tc = Np / C columns; rank (r, c) holds rows
[r*Tr, (r+1)*Tr) and columns [c*Tc, (c+1)*Tc). For a square mesh this is the reference's
layout (tile = ceil(N / s), pair_sharding.py:150-160).
"""

from __future__ import annotations

import math
from dataclasses import asdict, dataclass
from typing import Dict, List, Optional, Tuple

import torch
import torch.distributed as dist

from .layout import FoldCP2DLayout
from .mesh import FoldCPProcessMesh

Range = Tuple[int, int]


@dataclass(frozen=True)
class FoldCPPairShardSpec:
    """Metadata needed to gather a local 2D pair shard back to serial layout."""

    original_shape: Tuple[int, ...]
    padded_shape: Tuple[int, ...]
    pair_dims: Tuple[int, int]
    row_range: Range
    col_range: Range
    mesh_shape: Tuple[int, int]
    mesh_coord: Tuple[int, int]

    @property
    def local_shape(self) -> Tuple[int, ...]:
        shape = list(self.padded_shape)
        shape[self.pair_dims[0]] = self.row_range[1] - self.row_range[0]
        shape[self.pair_dims[1]] = self.col_range[1] - self.col_range[0]
        return tuple(shape)

    @property
    def n_token(self) -> int:
        return self.original_shape[self.pair_dims[0]]

    @property
    def n_padded(self) -> int:
        return self.padded_shape[self.pair_dims[0]]

    @property
    def tile_rows(self) -> int:
        return self.n_padded // self.mesh_shape[0]

    @property
    def tile_cols(self) -> int:
        return self.n_padded // self.mesh_shape[1]

    def row_range_of(self, mesh_row: int) -> Range:
        t = self.tile_rows
        return (mesh_row * t, (mesh_row + 1) * t)

    def col_range_of(self, mesh_col: int) -> Range:
        t = self.tile_cols
        return (mesh_col * t, (mesh_col + 1) * t)

    def to_dict(self) -> Dict[str, object]:
        return asdict(self)


def _resolve_pair_dims(ndim: int, pair_dims: Tuple[int, int]) -> Tuple[int, int]:
    """Absolute (row, column) dims of the token-pair plane; negative dims count from the end."""
    dims = []
    for d in pair_dims:
        a = d + ndim if d < 0 else d
        if not 0 <= a < ndim:
            raise ValueError(f"pair dim {d} does not exist in a {ndim}-d tensor (pair_dims={pair_dims})")
        dims.append(a)
    if dims[0] == dims[1]:
        raise ValueError(f"pair_dims {pair_dims} name the same dimension twice")
    return dims[0], dims[1]


def infer_pair_dims(tensor: torch.Tensor, n_token: int) -> Optional[Tuple[int, int]]:
    """Token-pair dims of common OpenDDE tensors: [..., N, N] (masks, biases) or
    [..., N, N, C] (pair representations); None when neither layout matches."""
    shape = tuple(tensor.shape)
    for lead in (2, 3):  # the pair dims end the shape, or sit just before a channel dim
        if len(shape) >= lead:
            a = len(shape) - lead
            if shape[a] == n_token and shape[a + 1] == n_token:
                return a, a + 1
    return None


def padded_pair_size(n_pair: int, mesh_shape: Tuple[int, int]) -> int:
    r, c = mesh_shape
    step = r * c // math.gcd(r, c)
    return int(math.ceil(n_pair / step) * step)


def _pair_index(ndim: int, pair_dims: Tuple[int, int], rows: Range, cols: Range):
    """Index tuple selecting rows x cols of the pair plane and everything of the other dims."""
    return tuple(slice(*rows) if d == pair_dims[0] else slice(*cols) if d == pair_dims[1] else slice(None)
                 for d in range(ndim))


def _spec_for(original_shape, mesh_shape, coord, pair_dims) -> FoldCPPairShardSpec:
    row_dim, col_dim = pair_dims
    n_row, n_col = original_shape[row_dim], original_shape[col_dim]
    if n_row != n_col:
        raise ValueError(f"pair tensor must be square, got {n_row} x {n_col}.")
    n_pad = padded_pair_size(n_row, mesh_shape)
    padded = list(original_shape)
    padded[row_dim] = padded[col_dim] = n_pad
    tr, tc = n_pad // mesh_shape[0], n_pad // mesh_shape[1]
    return FoldCPPairShardSpec(
        original_shape=tuple(original_shape), padded_shape=tuple(padded), pair_dims=pair_dims,
        row_range=(coord[0] * tr, (coord[0] + 1) * tr), col_range=(coord[1] * tc, (coord[1] + 1) * tc),
        mesh_shape=tuple(mesh_shape), mesh_coord=tuple(coord))


def make_pair_shard_spec(original_shape: Tuple[int, ...], mesh: FoldCPProcessMesh,
                         pair_dims: Tuple[int, int]) -> FoldCPPairShardSpec:
    """Pair-shard metadata without materialising the full pair tensor."""
    pair_dims = _resolve_pair_dims(len(original_shape), pair_dims)
    return _spec_for(tuple(original_shape), mesh.layout.shape, mesh.coord, pair_dims)


def shard_pair_tensor(tensor: torch.Tensor, mesh: FoldCPProcessMesh, pair_dims: Tuple[int, int],
                      pad_value: float = 0.0) -> Tuple[torch.Tensor, FoldCPPairShardSpec]:
    """This rank's (padded) tile of a full pair tensor."""
    pair_dims = _resolve_pair_dims(tensor.ndim, pair_dims)
    spec = _spec_for(tuple(tensor.shape), mesh.layout.shape, mesh.coord, pair_dims)
    return shard_with_spec(tensor, spec, pad_value), spec


def shard_with_spec(tensor: torch.Tensor, spec: FoldCPPairShardSpec, pad_value: float = 0.0) -> torch.Tensor:
    local = tensor.new_full(spec.local_shape, pad_value)
    n = spec.n_token
    (r0, r1), (c0, c1) = spec.row_range, spec.col_range
    vr, vc = min(r1, n), min(c1, n)
    if r0 < vr and c0 < vc:
        local[_pair_index(tensor.ndim, spec.pair_dims, (0, vr - r0), (0, vc - c0))] = \
            tensor[_pair_index(tensor.ndim, spec.pair_dims, (r0, vr), (c0, vc))]
    return local


def _all_gather_list(t: torch.Tensor, group, world: int) -> List[torch.Tensor]:
    t = t.contiguous()
    if dist.get_backend(group) == "nccl":
        flat = t.new_empty((world,) + tuple(t.shape))
        dist.all_gather_into_tensor(flat, t, group=group)
        return list(flat.unbind(0))
    out = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(out, t, group=group)
    return out


def _assemble(shards: List[torch.Tensor], layout: FoldCP2DLayout, pair_dims, out_shape) -> torch.Tensor:
    full = shards[0].new_empty(out_shape)
    rd, cd = pair_dims
    n_r, n_c = out_shape[rd], out_shape[cd]
    for cp_rank, shard in enumerate(shards):
        row, col = layout.to_coord(cp_rank)
        tr, tc = shard.shape[rd], shard.shape[cd]
        r0, c0 = row * tr, col * tc
        r1, c1 = min(r0 + tr, n_r), min(c0 + tc, n_c)
        if r0 >= r1 or c0 >= c1:
            continue
        full[_pair_index(full.ndim, pair_dims, (r0, r1), (c0, c1))] = \
            shard[_pair_index(shard.ndim, pair_dims, (0, r1 - r0), (0, c1 - c0))]
    return full


def gather_pair_tensor(local_tensor: torch.Tensor, spec: FoldCPPairShardSpec, group) -> torch.Tensor:
    """All CP tiles gathered on every rank and cropped to the original shape."""
    if not dist.is_initialized():
        raise RuntimeError("torch.distributed must be initialized before gather.")
    layout = FoldCP2DLayout(spec.mesh_shape)
    shards = _all_gather_list(local_tensor, group, layout.numel)
    return _assemble(shards, layout, spec.pair_dims, spec.original_shape)


def _like_shape(local_tensor: torch.Tensor, spec: FoldCPPairShardSpec) -> Tuple[int, ...]:
    shape = list(local_tensor.shape)
    shape[spec.pair_dims[0]] = spec.original_shape[spec.pair_dims[0]]
    shape[spec.pair_dims[1]] = spec.original_shape[spec.pair_dims[1]]
    return tuple(shape)


def gather_pair_tensor_like(local_tensor: torch.Tensor, spec: FoldCPPairShardSpec, group) -> torch.Tensor:
    """Gather a pair-like shard whose non-pair dimensions differ from ``spec`` (same tiling)."""
    if not dist.is_initialized():
        raise RuntimeError("torch.distributed must be initialized before gather.")
    if local_tensor.ndim != len(spec.original_shape):
        raise ValueError("local pair-like tensor must keep the same rank as the source pair tensor.")
    layout = FoldCP2DLayout(spec.mesh_shape)
    shards = _all_gather_list(local_tensor, group, layout.numel)
    return _assemble(shards, layout, spec.pair_dims, _like_shape(local_tensor, spec))


def gather_pair_tensor_like_to_rank(local_tensor: torch.Tensor, spec: FoldCPPairShardSpec, group,
                                    dst_group_rank: int = 0) -> Optional[torch.Tensor]:
    """Gather a pair-like shard on one group rank only (others return None)."""
    if not dist.is_initialized():
        raise RuntimeError("torch.distributed must be initialized before gather.")
    if local_tensor.ndim != len(spec.original_shape):
        raise ValueError("local pair-like tensor must keep the same rank as the source pair tensor.")
    layout = FoldCP2DLayout(spec.mesh_shape)
    me = dist.get_rank(group)
    dst = dist.get_global_rank(group, dst_group_rank)
    local_tensor = local_tensor.contiguous()
    if me != dst_group_rank:
        dist.send(local_tensor, dst=dst, group=group)
        return None
    shards = []
    for cp_rank in range(layout.numel):
        if cp_rank == dst_group_rank:
            shards.append(local_tensor)
        else:
            buf = torch.empty_like(local_tensor)
            dist.recv(buf, src=dist.get_global_rank(group, cp_rank), group=group)
            shards.append(buf)
    return _assemble(shards, layout, spec.pair_dims, _like_shape(local_tensor, spec))


def shard_pair_feature_dict(feature_dict: Dict[str, object], mesh: FoldCPProcessMesh, n_token: int):
    """Shard every tensor of a feature dict that has token-pair dimensions."""
    sharded: Dict[str, object] = {}
    specs: Dict[str, FoldCPPairShardSpec] = {}
    for key, value in feature_dict.items():
        if isinstance(value, torch.Tensor):
            pd = infer_pair_dims(value, n_token)
            if pd is not None:
                sharded[key], specs[key] = shard_pair_tensor(value, mesh, pair_dims=pd)
                continue
        sharded[key] = value
    return sharded, specs
