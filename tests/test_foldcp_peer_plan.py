"""Host logic of the peer-memory band exchange: the copy plans assemble every band request of
every rank of R x C meshes exactly (applied with host memmoves on CPU tiles)."""
import ctypes

import numpy as np
import pytest

from opendde_b200 import _abi
from opendde_b200.distributed.foldcp.layout import FoldCP2DLayout
from opendde_b200.distributed.foldcp.pair_sharding import _spec_for
from opendde_b200.distributed.foldcp.peer import band_copy_plan, transport_choice


def _apply(plan):
    for src, dst, planes, rows, row_bytes, sp, dp, spp, dpp in plan:
        for c in range(planes):
            for r in range(rows):
                ctypes.memmove(dst + c * dpp + r * dp, src + c * spp + r * sp, row_bytes)


@pytest.mark.parametrize("shape", [(1, 2), (2, 1), (2, 2), (2, 4), (4, 2), (1, 3), (3, 3)])
@pytest.mark.parametrize("n", [13, 16, 37])
def test_band_plans_assemble_every_request(shape, n):
    layout = FoldCP2DLayout(shape)
    ch = 3
    spec0 = _spec_for((n, n, ch), shape, (0, 0), (0, 1))
    n_pad = spec0.n_padded
    rng = np.random.default_rng(n * 10 + shape[0] * 3 + shape[1])
    plane = rng.standard_normal((n_pad, n_pad, ch)).astype(np.float32)
    tiles = []
    for q in range(layout.numel):
        sp = _spec_for((n, n, ch), shape, layout.to_coord(q), (0, 1))
        (r0, r1), (c0, c1) = sp.row_range, sp.col_range
        tiles.append(np.ascontiguousarray(plane[r0:r1, c0:c1]))
    ptrs = [t.ctypes.data for t in tiles]
    full = (0, n_pad)
    for q in range(layout.numel):
        coord = layout.to_coord(q)
        spec = _spec_for((n, n, ch), shape, coord, (0, 1))
        wants = [(spec.row_range, full), (full, spec.col_range),
                 (spec.col_range, full), (full, spec.row_range)]
        plans = []
        for want in wants:
            (r0, r1), (c0, c1) = want
            out = np.full((r1 - r0, c1 - c0, ch), np.nan, dtype=np.float32)
            plan = band_copy_plan(spec, layout, want, ptrs, out.ctypes.data, ch * 4)
            plans.append(plan)
            _apply(plan)
            np.testing.assert_array_equal(out, plane[r0:r1, c0:c1])
        # the two bands of one op fit one kernel launch
        assert len(plans[0]) + len(plans[2]) <= _abi.PF_MAX_COPY_REGIONS


def test_transport_choice(monkeypatch):
    monkeypatch.delenv("OPENDDE_B200_FOLDCP_TRANSPORT", raising=False)
    assert transport_choice("nccl") == "peer"
    assert transport_choice("gloo") == "dist"
    monkeypatch.setenv("OPENDDE_B200_FOLDCP_TRANSPORT", "nccl")
    assert transport_choice("nccl") == "nccl"
    monkeypatch.setenv("OPENDDE_B200_FOLDCP_TRANSPORT", "shm")
    with pytest.raises(ValueError):
        transport_choice("nccl")


@pytest.mark.parametrize("shape", [(1, 2), (2, 1), (2, 2), (2, 4), (4, 2), (1, 3)])
@pytest.mark.parametrize("n", [13, 37])
@pytest.mark.parametrize("transposed", [False, True])
def test_projection_plans_assemble_operand_bands(shape, n, transposed):
    """Channel-major projection bands P[ch][i in I][k < Np] from per-rank tile projections in the
    plain (i, k) = z(i, k) or transposed (i, k) = z(k, i) orientation."""
    from opendde_b200.distributed.foldcp.peer import projection_copy_plan, projection_geometry
    layout = FoldCP2DLayout(shape)
    planes, elem = 3, 4
    spec0 = _spec_for((n, n, 1), shape, (0, 0), (0, 1))
    n_pad = spec0.n_padded
    rng = np.random.default_rng(n + 100 * shape[0] + 10 * shape[1] + int(transposed))
    plane = rng.standard_normal((planes, n_pad, n_pad)).astype(np.float32)   # P[ch][i][k]
    ld_t = (max(spec0.tile_rows, spec0.tile_cols) + 7) // 8 * 8 + 8         # padded pitch
    slots = []
    for q in range(layout.numel):
        sp = _spec_for((n, n, 1), shape, layout.to_coord(q), (0, 1))
        xr, yr = projection_geometry(sp, layout.to_coord(q), transposed)
        t = np.full((planes, xr[1] - xr[0], ld_t), np.nan, dtype=np.float32)
        t[:, :, :yr[1] - yr[0]] = plane[:, xr[0]:xr[1], yr[0]:yr[1]]
        slots.append(t)
    ptrs = [t.ctypes.data for t in slots]
    ld_b = (n_pad + 7) // 8 * 8
    for q in range(layout.numel):
        coord = layout.to_coord(q)
        spec = _spec_for((n, n, 1), shape, coord, (0, 1))
        for rows in (spec.row_range, spec.col_range):
            out = np.full((planes, rows[1] - rows[0], ld_b), np.nan, dtype=np.float32)
            plan = projection_copy_plan(spec, layout, rows, transposed, ptrs, 0, planes, elem, ld_t,
                                        out.ctypes.data, ld_b)
            assert len(plan) <= layout.numel
            _apply(plan)
            np.testing.assert_array_equal(out[:, :, :n_pad], plane[:, rows[0]:rows[1], :])
