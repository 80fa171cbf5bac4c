"""Fold-CP on one B200: every rank of an R x C mesh emulated as a thread on cuda:0, running
the real drivers and the real kernels (bands, bias planes, query offsets, transposed views).

bf16: the CP stack equals the single-device stack (same kernels, same full-K contractions
and full-key softmax per output) up to bf16 rounding of the exchanged tiles; fp32: equals
the CPU oracle at the fp32 bar.
"""
import pytest
import torch

from foldcp_support import ThreadMesh
from gpu_helpers import max_abs, rel_l2
from oracle import pairformer_oracle as O
from opendde_b200 import _abi
from opendde_b200.distributed.foldcp import real_pairformer as RP
from opendde_b200.distributed.foldcp.ops import KernelOps
from opendde_b200.distributed.foldcp.pair_sharding import _spec_for, shard_with_spec
from opendde_b200.model import PairformerStack
from opendde_b200.utils import ragged_pair_mask, seeded_params

pytestmark = pytest.mark.gpu


def _stack(n_blocks, dev, **kw):
    st = PairformerStack(n_blocks=n_blocks, **kw)
    p = seeded_params([(k, tuple(v.shape)) for k, v in st.named_parameters()], seed=0, perturb_1d=True)
    with torch.no_grad():
        for k, v in st.named_parameters():
            v.copy_(p[k])
    return st.to(dev), p


def _cp(shape, stack, s, z, mask, transport="copy"):
    mesh = ThreadMesh(shape, transport=transport)

    def rank_fn(ex, rank):
        spec = _spec_for(tuple(z.shape), shape, ex.coord, (0, 1))
        z_local = shard_with_spec(z, spec)
        ctx = RP.make_context(None, z_local, spec, mask_full=mask, exchange=ex)
        return RP.distributed_pairformer_stack_single_bridge_update(
            stack, s.clone(), z_local, None, z_spec=spec, ops=KernelOps(), context=ctx)

    with torch.no_grad():
        out = mesh.run(rank_fn)
    torch.cuda.synchronize()
    return out


@pytest.mark.parametrize("transport", ["copy", "peer"])
@pytest.mark.parametrize("shape", [(1, 2), (2, 2), (2, 4)])
def test_cp_bf16_matches_single_device(shape, transport, cuda_device):
    n = 300   # not a multiple of the tiles: exercises padding and partial MMA tiles
    stack, _ = _stack(1, cuda_device)
    g = torch.Generator().manual_seed(1)
    z = torch.randn((n, n, 128), generator=g).to(cuda_device, torch.bfloat16)
    s = torch.randn((n, 384), generator=g).to(cuda_device, torch.bfloat16)
    mask = ragged_pair_mask(n, seed=3, drop=0.2, full_rows=[5]).to(cuda_device)
    with torch.no_grad():
        s1, z1 = stack(s, z, mask)
    outs = _cp(shape, stack, s, z, mask, transport)
    assert _abi.device_status(clear=True) == 0
    for s2, z2 in outs:
        assert rel_l2(z2, z1) <= 5e-3
        assert rel_l2(s2, s1) <= 5e-3


@pytest.mark.parametrize("transport", ["copy", "peer"])
@pytest.mark.parametrize("shape", [(1, 2), (2, 4)])
def test_cp_fp32_matches_oracle(shape, transport, cuda_device):
    n = 37
    stack, p = _stack(1, cuda_device, n_heads=16, c_z=128, c_s=384)
    g = torch.Generator().manual_seed(2)
    z = torch.randn((n, n, 128), generator=g)
    s = torch.randn((n, 384), generator=g)
    mask = ragged_pair_mask(n, seed=4, drop=0.2, full_rows=[0])
    torch.set_num_threads(8)
    with torch.no_grad():
        s_ref, z_ref = O.pairformer_stack(s, z, mask, p, 1)
    outs = _cp(shape, stack, s.to(cuda_device), z.to(cuda_device), mask.to(cuda_device), transport)
    for s2, z2 in outs:
        assert max_abs(z2, z_ref) <= 1e-4
        assert max_abs(s2, s_ref) <= 1e-4


@pytest.mark.parametrize("dma", [False, True])
@pytest.mark.parametrize("unit", [16, 8, 4, 1])
def test_copy_regions_every_vector_width(unit, dma, cuda_device):
    """pf_copy_regions moves 2D rectangles at the widest common alignment (16/8/4/1 bytes);
    pf_copy_regions_dma moves the same boxes by the copy engines (one 2-D copy for evenly spaced
    planes, a 3-D copy for plane pitches that are whole numbers of rows, else a copy per plane)."""
    from opendde_b200 import kernels
    size = 8 << 20
    g = torch.Generator().manual_seed(7)
    src = torch.randint(0, 255, (size,), generator=g, dtype=torch.uint8).to(cuda_device)
    dst = torch.zeros_like(src)
    u = unit
    #  offset  planes rows row_bytes  src_pitch  dst_pitch src_plane dst_plane (odd multiples of u)
    boxes = [(u, 1, 100, 37 * u, 103 * u, 70 * u, 0, 0),
             (64 * u, 1, 3, 4097 * u, 4099 * u, 4098 * u, 0, 0),
             (2 * u, 1, 1, 25000 * u, 25000 * u, 25000 * u, 0, 0),
             (3 * u, 5, 7, 11 * u, 13 * u, 12 * u, 97 * u, 89 * u),
             (5 * u, 3, 4, 10 * u, 12 * u, 16 * u, 72 * u, 80 * u),     # plane pitches: whole rows
             (7 * u, 2, 3, 8 * u, 9 * u, 10 * u, 27 * u, 30 * u)]        # planes evenly spaced
    regions, want = [], dst.clone()
    for i, (off, planes, rows, row_bytes, sp, dp, spp, dpp) in enumerate(boxes):
        s_off, d_off = off, off + (1 << 20) * i
        assert s_off + (planes - 1) * spp + (rows - 1) * sp + row_bytes <= size      # every access in bounds
        assert d_off + (planes - 1) * dpp + (rows - 1) * dp + row_bytes <= size
        regions.append((src.data_ptr() + s_off, dst.data_ptr() + d_off, planes, rows, row_bytes, sp, dp, spp, dpp))
        for c in range(planes):
            for r in range(rows):
                so, do = s_off + c * spp + r * sp, d_off + c * dpp + r * dp
                want[do:do + row_bytes] = src[so:so + row_bytes]
    kernels.copy_regions(regions, dma=dma)
    torch.cuda.synchronize()
    assert torch.equal(dst, want)


@pytest.mark.parametrize("overlap", ["0", "2"])
def test_cp_bf16_copy_engine_transport(overlap, cuda_device, monkeypatch):
    """The peer transport with the bands moved by the copy engines (and, overlap 2, the attention
    band in two chunks on the side stream) matches the single-device stack."""
    monkeypatch.setenv("OPENDDE_B200_FOLDCP_COPY", "dma")
    monkeypatch.setenv("OPENDDE_B200_FOLDCP_OVERLAP", overlap)
    n = 300
    stack, _ = _stack(1, cuda_device)
    g = torch.Generator().manual_seed(1)
    z = torch.randn((n, n, 128), generator=g).to(cuda_device, torch.bfloat16)
    s = torch.randn((n, 384), generator=g).to(cuda_device, torch.bfloat16)
    mask = ragged_pair_mask(n, seed=3, drop=0.2, full_rows=[5]).to(cuda_device)
    with torch.no_grad():
        s1, z1 = stack(s, z, mask)
    outs = _cp((2, 4), stack, s, z, mask, "peer")
    assert _abi.device_status(clear=True) == 0
    for s2, z2 in outs:
        assert rel_l2(z2, z1) <= 5e-3
        assert rel_l2(s2, s1) <= 5e-3


def test_cp_bf16_sm_reserve_overlap(cuda_device, monkeypatch):
    """The overlapped band exchange with SMs reserved for the copy kernel (persistent grids of
    148 - 16 CTAs while a chunk computes): the same z and s as the same overlap without the
    reserve, bit for bit (the grid size changes which CTA computes a tile, not the tile), and the
    single-device stack's within tolerance."""
    n = 300
    stack, _ = _stack(1, cuda_device)
    g = torch.Generator().manual_seed(2)
    z = torch.randn((n, n, 128), generator=g).to(cuda_device, torch.bfloat16)
    s = torch.randn((n, 384), generator=g).to(cuda_device, torch.bfloat16)
    mask = ragged_pair_mask(n, seed=3, drop=0.2, full_rows=[5]).to(cuda_device)
    with torch.no_grad():
        s1, z1 = stack(s, z, mask)
    monkeypatch.setenv("OPENDDE_B200_FOLDCP_OVERLAP", "3")
    base = _cp((2, 4), stack, s, z, mask, "peer")
    monkeypatch.setenv("OPENDDE_B200_FOLDCP_RESERVE_SMS", "16")
    outs = _cp((2, 4), stack, s, z, mask, "peer")
    assert _abi.device_status(clear=True) == 0
    for (s2, z2), (sb, zb) in zip(outs, base):
        assert torch.equal(z2, zb) and torch.equal(s2, sb)
        assert rel_l2(z2, z1) <= 5e-3 and rel_l2(s2, s1) <= 5e-3
