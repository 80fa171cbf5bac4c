"""The reference's closed-form Fold-CP mini-oracles: restated in the oracle, pinned to golden
vectors produced by the reference (tests/golden/make_mini_golden.py), and used the way the
reference's own Fold-CP tests use them: the band exchanges of the drivers, followed by the
closed-form local contraction / attention, reproduce the serial result on every rank."""
import os
import sys

import numpy as np
import pytest
import torch

from foldcp_support import ThreadMesh
from oracle import pairformer_oracle as O
from opendde_b200.distributed.foldcp.exchange import gather_bands
from opendde_b200.distributed.foldcp.pair_sharding import _spec_for, shard_with_spec

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))
from make_mini_golden import OUT, SPLITS, block_state, checksum, mini_inputs  # noqa: E402


def test_mini_oracles_match_reference_goldens():
    rec = dict(np.load(OUT))
    a, b, z, q, k, v = mini_inputs()
    for name, t in zip("abzqkv", (a, b, z, q, k, v)):
        np.testing.assert_allclose(checksum(t), rec[f"chk_{name}"], rtol=1e-12)
    np.testing.assert_allclose(O.serial_triangle_multiplication(a, b, True).numpy(), rec["tm_out"], atol=1e-12)
    np.testing.assert_allclose(O.serial_triangle_multiplication(a, b, False).numpy(), rec["tm_in"], atol=1e-12)
    np.testing.assert_allclose(O.serial_triangle_attention_starting(z).numpy(), rec["ta_start"], atol=1e-12)
    np.testing.assert_allclose(O.serial_triangle_attention_ending(z).numpy(), rec["ta_end"], atol=1e-12)
    out = lse = amax = None
    for lo, hi in SPLITS:
        out, lse, amax = O.online_softmax_update(*block_state(q, k, v, lo, hi), out, lse, amax)
    np.testing.assert_allclose(out.numpy(), rec["os_out"], atol=1e-12)
    np.testing.assert_allclose(lse.numpy(), rec["os_lse"], atol=1e-12)
    np.testing.assert_allclose(amax.numpy(), rec["os_amax"], atol=1e-12)


def test_online_softmax_merge_equals_full_softmax():
    """Merging key blocks in any split reproduces softmax attention over all keys."""
    _, _, _, q, k, v = mini_inputs()
    full = torch.softmax(q @ k.transpose(-1, -2), -1) @ v
    for splits in (SPLITS, ((0, 1), (1, 9)), ((0, 8), (8, 9)), tuple((i, i + 1) for i in range(9))):
        out = lse = amax = None
        for lo, hi in splits:
            out, lse, amax = O.online_softmax_update(*block_state(q, k, v, lo, hi), out, lse, amax)
        torch.testing.assert_close(out, full, atol=1e-12, rtol=0)
        torch.testing.assert_close(lse + amax, torch.logsumexp(q @ k.transpose(-1, -2), -1), atol=1e-12, rtol=0)


def _run(shape, tensors, fn, transport):
    mesh = ThreadMesh(shape, transport=transport)

    def rank_fn(ex, rank):
        n = tensors[0].shape[0]
        spec = _spec_for(tuple(tensors[0].shape), shape, ex.coord, (0, 1))
        locs = [shard_with_spec(t, spec) for t in tensors]
        return spec, fn(ex, spec, locs)

    with torch.no_grad():
        return mesh.run(rank_fn)


@pytest.mark.parametrize("transport", ["copy", "peer"])
@pytest.mark.parametrize("shape", [(1, 2), (2, 2), (2, 4), (4, 2), (1, 3)])
@pytest.mark.parametrize("outgoing", [True, False])
def test_band_exchange_reproduces_serial_triangle_multiplication(shape, outgoing, transport):
    n, c = 13, 3
    g = torch.Generator().manual_seed(5)
    a = torch.randn((n, n, c), generator=g)
    b = torch.randn((n, n, c), generator=g)
    want = O.serial_triangle_multiplication(a[None], b[None], outgoing)[0]

    def fn(ex, spec, locs):
        (r0, r1), (c0, c1) = spec.row_range, spec.col_range
        a_loc, b_loc = locs
        if outgoing:   # x_ij = sum_k a_ik b_jk: a rows R_r, b rows C_c
            a_band, = gather_bands(ex, a_loc, spec, [("own_rows",)])
            b_band, = gather_bands(ex, b_loc, spec, [("rows", lambda co: spec.col_range_of(co[1]))])
            return torch.einsum("ikc,jkc->ijc", a_band, b_band)
        # x_ij = sum_k a_ki b_kj: a columns R_r, b columns C_c
        a_band, = gather_bands(ex, a_loc, spec, [("cols", lambda co: spec.row_range_of(co[0]))])
        b_band, = gather_bands(ex, b_loc, spec, [("own_cols",)])
        return torch.einsum("kic,kjc->ijc", a_band, b_band)

    for spec, tile in _run(shape, (a, b), fn, transport):
        (r0, r1), (c0, c1) = spec.row_range, spec.col_range
        vr, vc = max(0, min(r1, n) - r0), max(0, min(c1, n) - c0)
        torch.testing.assert_close(tile[:vr, :vc], want[r0:r0 + vr, c0:c0 + vc], atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize("transport", ["copy", "peer"])
@pytest.mark.parametrize("shape", [(1, 2), (2, 2), (2, 4), (4, 2)])
@pytest.mark.parametrize("starting", [True, False])
def test_band_exchange_reproduces_serial_triangle_attention(shape, starting, transport):
    n, c = 16, 4      # a multiple of every mesh side: no padded keys
    g = torch.Generator().manual_seed(6)
    z = 0.5 * torch.randn((n, n, c), generator=g)
    want = (O.serial_triangle_attention_starting if starting else O.serial_triangle_attention_ending)(z[None])[0]

    def fn(ex, spec, locs):
        (r0, r1), (c0, c1) = spec.row_range, spec.col_range
        z_loc, = locs
        if starting:   # rows R_r, all keys; queries C_c
            band, = gather_bands(ex, z_loc, spec, [("own_rows",)])
            qz = band[:, c0:c1]
            w = torch.softmax(qz @ band.transpose(-1, -2), -1)
            return w @ band
        band, = gather_bands(ex, z_loc, spec, [("own_cols",)])   # all rows, columns C_c
        x = band.transpose(0, 1)                                  # x = z^T rows C_c
        qx = x[:, r0:r1]
        return (torch.softmax(qx @ x.transpose(-1, -2), -1) @ x).transpose(0, 1)

    for spec, tile in _run(shape, (z,), fn, transport):
        (r0, r1), (c0, c1) = spec.row_range, spec.col_range
        torch.testing.assert_close(tile, want[r0:r1, c0:c1], atol=1e-5, rtol=1e-5)
