"""Fold-CP drivers on emulated R x C meshes (threads, CPU) vs the serial CPU oracle.

Every rank runs the real drivers (band exchanges, bias planes, query splits, gathers); the
local band computations are the oracle restatement (foldcp_support.OracleBandOps).
"""
import pytest
import torch

from foldcp_support import OracleBandOps, ThreadMesh
from oracle import pairformer_oracle as O
from opendde_b200.distributed.foldcp import real_pairformer as RP
from opendde_b200.distributed.foldcp.pair_sharding import _spec_for, shard_with_spec
from opendde_b200.model import PairformerStack
from opendde_b200.utils import ragged_pair_mask, seeded_params

C_Z, C_S, HEADS = 16, 32, 4
TOL = 1e-4


def _stack(n_blocks):
    st = PairformerStack(n_blocks=n_blocks, n_heads=HEADS, c_z=C_Z, c_s=C_S)
    p = seeded_params([(k, tuple(v.shape)) for k, v in st.named_parameters()], seed=0, perturb_1d=True)
    with torch.no_grad():
        for k, v in st.named_parameters():
            v.copy_(p[k])
    return st, p


def _inputs(n, seed=1):
    g = torch.Generator().manual_seed(seed)
    z = torch.randn((n, n, C_Z), generator=g)
    s = torch.randn((n, C_S), generator=g)
    mask = ragged_pair_mask(n, seed=3, drop=0.2, full_rows=[1])
    return s, z, mask


def _run_cp(shape, stack, s, z, mask, transport="copy"):
    mesh = ThreadMesh(shape, transport=transport)

    def rank_fn(ex, rank):
        spec = _spec_for(tuple(z.shape), shape, ex.coord, (0, 1))
        z_local = shard_with_spec(z, spec)
        ctx = RP.make_context(None, z_local, spec, mask_full=mask, exchange=ex)
        return RP.distributed_pairformer_stack_single_bridge_update(
            stack, s.clone(), z_local, None, z_spec=spec, ops=OracleBandOps(), context=ctx)

    return mesh.run(rank_fn)


@pytest.mark.parametrize("transport", ["copy", "peer"])
@pytest.mark.parametrize("shape", [(1, 2), (2, 2), (2, 4), (4, 2), (1, 3)])
@pytest.mark.parametrize("n", [13, 16])
def test_cp_stack_matches_serial_oracle(shape, n, transport):
    """"peer": the peer-memory transport's snapshot / projection-exchange logic with host
    windows (copy plans applied by memmove), including the trimul projection exchange."""
    torch.manual_seed(0)
    stack, p = _stack(2)
    s, z, mask = _inputs(n)
    with torch.no_grad():
        s_ref, z_ref = O.pairformer_stack(s, z, mask, p, 2, no_heads_pair=4, n_heads=HEADS, c_s=C_S)
        outs = _run_cp(shape, stack, s, z, mask, transport)
    for s_out, z_out in outs:     # every rank returns the full, identical result
        assert (z_out - z_ref).abs().max().item() <= TOL
        assert (s_out - s_ref).abs().max().item() <= TOL


@pytest.mark.parametrize("shape", [(1, 2), (2, 4)])
def test_cp_single_ops_reference_return_convention(shape):
    """Per-op entry points: with residual_local the tile is updated in place and returned;
    without it the update alone is returned (the reference's convention)."""
    n = 11
    stack, p = _stack(1)
    blk = stack.blocks[0]
    blk.tri_att_end.starting = False   # a stand-alone ending-node module (the block transposes itself)
    s, z, mask = _inputs(n, seed=5)
    sub = lambda pre: {k[len(pre) + 1:]: v for k, v in p.items() if k.startswith(pre + ".")}  # noqa: E731
    with torch.no_grad():
        want = {
            "tmo": O.triangle_multiplication(z, mask, sub("blocks.0.tri_mul_out"), outgoing=True),
            "tmi": O.triangle_multiplication(z, mask, sub("blocks.0.tri_mul_in"), outgoing=False),
            "tas": O.triangle_attention(z, mask, sub("blocks.0.tri_att_start"), 4, starting=True),
            "tae": O.triangle_attention(z, mask, sub("blocks.0.tri_att_end"), 4, starting=False),
            "tr": O.transition(z, sub("blocks.0.pair_transition")),
        }
    mesh = ThreadMesh(shape)

    def rank_fn(ex, rank):
        spec = _spec_for(tuple(z.shape), shape, ex.coord, (0, 1))
        z_local = shard_with_spec(z, spec)
        ctx = RP.make_context(None, z_local, spec, mask_full=mask, exchange=ex)
        ops = OracleBandOps()
        got = {
            "tmo": RP.distributed_triangle_multiplication_update(blk.tri_mul_out, z_local, None, ops=ops, context=ctx),
            "tmi": RP.distributed_triangle_multiplication_update(blk.tri_mul_in, z_local, None, ops=ops, context=ctx),
            "tas": RP.distributed_triangle_attention_update(blk.tri_att_start, z_local, None, ops=ops, context=ctx),
            "tae": RP.distributed_triangle_attention_update(blk.tri_att_end, z_local, None, ops=ops, context=ctx),
            "tr": RP.distributed_pair_transition_update(blk.pair_transition, z_local, None, ops=ops),
        }
        # the in-place form returns the same tile object, updated
        before = z_local.clone()
        out = RP.distributed_pair_transition_update(blk.pair_transition, z_local, None, residual_local=z_local, ops=ops)
        assert out is z_local
        torch.testing.assert_close(out - before, got["tr"], atol=1e-5, rtol=0)
        return spec, {k: RP.gather_full(v.contiguous(), ctx) for k, v in got.items()}

    with torch.no_grad():
        res = mesh.run(rank_fn)
    for _, got in res:
        for k in want:
            assert (got[k] - want[k]).abs().max().item() <= TOL, k


@pytest.mark.parametrize("shape", [(1, 2), (2, 2), (2, 4)])
@pytest.mark.parametrize("chunks", [2, 3])
def test_cp_stack_overlapped_attention_chunks(shape, chunks, monkeypatch):
    """The chunked band exchanges (side-stream overlap on GPUs) compute the same stack: every
    chunk of attention rows gets its own band and the shared bias rows, and every chunk of the
    triangle update's output rows its own a band next to the whole b band."""
    monkeypatch.setenv("OPENDDE_B200_FOLDCP_OVERLAP", str(chunks))
    torch.manual_seed(0)
    stack, p = _stack(1)
    s, z, mask = _inputs(13)
    with torch.no_grad():
        s_ref, z_ref = O.pairformer_stack(s, z, mask, p, 1, no_heads_pair=4, n_heads=HEADS, c_s=C_S)
        outs = _run_cp(shape, stack, s, z, mask, "peer")
    for s_out, z_out in outs:
        assert (z_out - z_ref).abs().max().item() <= TOL
        assert (s_out - s_ref).abs().max().item() <= TOL


@pytest.mark.parametrize("shape", [(1, 2), (2, 2)])
def test_cp_single_ops_with_a_separate_residual(shape):
    """residual_local that is not the tile itself: the result is residual + update, and the
    tile is left as it was (reference real_pairformer.py:1226 semantics)."""
    n = 11
    stack, p = _stack(1)
    blk = stack.blocks[0]
    s, z, mask = _inputs(n, seed=6)
    g = torch.Generator().manual_seed(9)
    resid = torch.randn(z.shape, generator=g)
    sub = lambda pre: {k[len(pre) + 1:]: v for k, v in p.items() if k.startswith(pre + ".")}  # noqa: E731
    with torch.no_grad():
        upd = {"tmo": O.triangle_multiplication(z, mask, sub("blocks.0.tri_mul_out"), outgoing=True),
               "tas": O.triangle_attention(z, mask, sub("blocks.0.tri_att_start"), 4, starting=True),
               "tr": O.transition(z, sub("blocks.0.pair_transition"))}
    mesh = ThreadMesh(shape)

    def rank_fn(ex, rank):
        spec = _spec_for(tuple(z.shape), shape, ex.coord, (0, 1))
        z_local = shard_with_spec(z, spec)
        r_local = shard_with_spec(resid, spec)
        keep = z_local.clone()
        ctx = RP.make_context(None, z_local, spec, mask_full=mask, exchange=ex)
        ops = OracleBandOps()
        got = {
            "tmo": RP.distributed_triangle_multiplication_update(blk.tri_mul_out, z_local, None, residual_local=r_local,
                                                                 ops=ops, context=ctx),
            "tas": RP.distributed_triangle_attention_update(blk.tri_att_start, z_local, None, residual_local=r_local,
                                                            ops=ops, context=ctx),
            "tr": RP.distributed_pair_transition_update(blk.pair_transition, z_local, None, residual_local=r_local,
                                                        ops=ops),
        }
        assert torch.equal(z_local, keep)
        return {k: RP.gather_full(v.contiguous(), ctx) for k, v in got.items()}

    with torch.no_grad():
        res = mesh.run(rank_fn)
    for got in res:
        for k in upd:
            assert (got[k] - (resid + upd[k])).abs().max().item() <= TOL, k


@pytest.mark.parametrize("shape", [(2, 2), (2, 4)])
def test_cp_attention_pair_bias_with_a_local_extra_bias(shape):
    """extra_attn_bias_local (each rank's tile of an extra [H, N, N] bias) on an R x C mesh
    equals passing the whole bias."""
    n = 13
    stack, p = _stack(1)
    blk = stack.blocks[0]
    s, z, mask = _inputs(n, seed=7)
    g = torch.Generator().manual_seed(11)
    extra = torch.randn((HEADS, n, n), generator=g)
    mesh = ThreadMesh(shape)

    def rank_fn(ex, rank):
        spec = _spec_for(tuple(z.shape), shape, ex.coord, (0, 1))
        z_local = shard_with_spec(z, spec)
        espec = _spec_for((HEADS, n, n), shape, ex.coord, (1, 2))
        e_local = shard_with_spec(extra, espec)
        ctx = RP.make_context(None, z_local, spec, mask_full=mask, exchange=ex)
        ops = OracleBandOps()
        a = RP.distributed_attention_pair_bias_update(blk.attention_pair_bias, s, z_local, None, spec,
                                                      extra_attn_bias_local=e_local, ops=ops, context=ctx)
        b = RP.distributed_attention_pair_bias_update(blk.attention_pair_bias, s, z_local, None, spec, ops=ops,
                                                      context=ctx, extra_attn_bias_full=extra)
        return a, b

    with torch.no_grad():
        res = mesh.run(rank_fn)
    for a, b in res:
        assert (a - b).abs().max().item() <= 1e-5
