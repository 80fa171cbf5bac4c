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
    for src, dst, rows, row_bytes, sp, dp in plan:
        for r in range(rows):
            ctypes.memmove(dst + r * dp, src + r * sp, row_bytes)


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
