"""Fold-CP configuration, R x C layout and tile geometry (host logic, no process group)."""
import pytest
import torch

from opendde_b200.distributed.foldcp import FoldCP2DLayout, FoldCPConfig
from opendde_b200.distributed.foldcp.pair_sharding import _spec_for, padded_pair_size, shard_with_spec


def test_default_meshes():
    cfg = lambda cp, mesh="": FoldCPConfig.from_runtime_args(mode="distributed", size_cp=cp, mesh=mesh)  # noqa: E731
    assert cfg(4).cp_mesh_shape == (2, 2)
    assert cfg(9).cp_mesh_shape == (3, 3)
    assert cfg(2).cp_mesh_shape == (1, 2)
    assert cfg(8).cp_mesh_shape == (2, 4)
    assert cfg(8, "4x2").cp_mesh_shape == (4, 2)


def test_validation_messages_match_reference():
    with pytest.raises(ValueError, match="foldcp_mode must be 'single' or 'distributed'"):
        FoldCPConfig.from_runtime_args(mode="x")
    with pytest.raises(ValueError, match="requires foldcp_size_cp=1"):
        FoldCPConfig.from_runtime_args(mode="single", size_cp=2)
    with pytest.raises(ValueError, match="requires foldcp_size_cp > 1"):
        FoldCPConfig.from_runtime_args(mode="distributed", size_cp=1)
    with pytest.raises(ValueError, match="does not hold"):
        FoldCPConfig.from_runtime_args(mode="distributed", size_cp=8, mesh="3x3")


def test_env_config(monkeypatch):
    monkeypatch.setenv("OPENDDE_FOLDCP_MODE", "distributed")
    monkeypatch.setenv("OPENDDE_FOLDCP_SIZE_CP", "8")
    monkeypatch.setenv("OPENDDE_FOLDCP_MESH", "2x4")
    cfg = FoldCPConfig.from_env(8)
    assert cfg.enabled and cfg.cp_mesh_shape == (2, 4)
    assert "OPENDDE_FOLDCP_MESH=2x4" in cfg.launch_hint()


def test_layout_rank_maps():
    lay = FoldCP2DLayout((2, 4))
    assert [lay.to_coord(r) for r in range(8)] == [(r, c) for r in range(2) for c in range(4)]
    assert lay.shifted_rank((1, 3), 1, 1) == lay.to_linear((1, 0))
    with pytest.raises(ValueError):
        lay.transpose_rank((0, 1))
    assert FoldCP2DLayout((2, 2)).transpose_rank((0, 1)) == 2


@pytest.mark.parametrize("shape", [(1, 2), (2, 2), (2, 4), (4, 2), (3, 3)])
@pytest.mark.parametrize("n", [1, 7, 13, 1536])
def test_tiles_cover_the_plane_once(shape, n):
    n_pad = padded_pair_size(n, shape)
    assert n_pad >= n and n_pad % shape[0] == 0 and n_pad % shape[1] == 0
    z = torch.arange(n * n, dtype=torch.float32).view(n, n, 1) if n <= 13 else None
    cover = torch.zeros((n_pad, n_pad), dtype=torch.int32)
    for r in range(shape[0]):
        for c in range(shape[1]):
            spec = _spec_for((n, n, 1), shape, (r, c), (0, 1))
            (r0, r1), (c0, c1) = spec.row_range, spec.col_range
            cover[r0:r1, c0:c1] += 1
            if z is not None:
                loc = shard_with_spec(z, spec)
                vr, vc = max(0, min(r1, n) - r0), max(0, min(c1, n) - c0)
                assert torch.equal(loc[:vr, :vc], z[r0:r0 + vr, c0:c0 + vc])
                assert loc[vr:].abs().sum() == 0 and loc[:, vc:].abs().sum() == 0
    assert torch.all(cover == 1)
