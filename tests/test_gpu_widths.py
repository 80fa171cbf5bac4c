"""The general-width tensor-core path (csrc/pf_tc_rows.cu) at the reference's real-model
Pairformer widths, against the fp32 oracle run on the GPU (TF32 off).

The fused kernels cover c_z = c_h = 128 with 4 heads of 32; every other bf16 width runs on
tcgen05 GEMMs with LayerNorm passes between them, the per-channel contraction and the
attention core (dispatch path "tc.rows"). The widths are those of the Pairformer's callers
(opendde/config/model_base.py:20,30; opendde/model/modules/pairformer.py:91-93,804-808,
1678-1685): the template stack (c_z = 64, c_h = 128, 4 heads, transition x2, no single path)
and the structural refiner (c_z = c_h = 384, 12 heads, transition x2, AttentionPairBias with
c_z = 384), plus small odd widths.

* each op alone, both directions, on odd sizes with ragged masks (fully masked rows included);
* the Fold-CP split stages (project, then combine) bit-identical to the one-call update;
* PairformerStack in the template and refiner configurations, block by block against the
  oracle applied to the same bf16 input (the contract of the trunk's drift test).

Tolerance: bf16 relative-L2 <= 2e-2 against the fp32 oracle.
"""
import contextlib

import pytest
import torch

from gpu_helpers import cuda_module, rel_l2
from oracle import pairformer_oracle as O
from opendde_b200 import _abi, kernels
from opendde_b200.model import (AttentionPairBias, PairformerStack, Transition, TriangleAttention,
                                TriangleMultiplicationIncoming, TriangleMultiplicationOutgoing)
from opendde_b200.utils import make_inputs, ragged_pair_mask, seeded_init_, seeded_params

pytestmark = pytest.mark.gpu

BF16_TOL = 2e-2


@contextlib.contextmanager
def exact_fp32():
    old = (torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32)
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    try:
        yield
    finally:
        torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32 = old


def _params(mod, seed=0):
    return seeded_params([(k, tuple(p.shape)) for k, p in mod.named_parameters()], seed=seed, perturb_1d=True)


def _dev(params, device, dtype=torch.float32):
    return {k: v.to(device=device, dtype=dtype) for k, v in params.items()}


def _pair(n, c, seed, device):
    g = torch.Generator().manual_seed(seed)
    return torch.randn((n, n, c), generator=g).to(device, torch.bfloat16)


def _mask(n, device):
    return ragged_pair_mask(n, seed=3, drop=0.2, full_rows=[5]).to(device)


@pytest.mark.parametrize("c_z,c_h", [(64, 128), (384, 384), (40, 64), (288, 64)])
@pytest.mark.parametrize("outgoing", [True, False])
def test_trimul_general_width(c_z, c_h, outgoing, cuda_device):
    n = 97
    mod = (TriangleMultiplicationOutgoing if outgoing else TriangleMultiplicationIncoming)(c_z=c_z, c_hidden=c_h)
    params = _params(mod)
    z, m = _pair(n, c_z, 1, cuda_device), _mask(n, cuda_device)
    with torch.no_grad():
        got = cuda_module(mod, params, cuda_device)(z, mask=m)
        assert _abi.last_path() == "tc.rows"
        with exact_fp32():
            want = O.triangle_multiplication(z.float(), m, _dev(params, cuda_device), outgoing=outgoing)
    assert _abi.device_status(clear=True) == 0
    err = rel_l2(got, want)
    print(f"trimul {'out' if outgoing else 'in'} c_z={c_z} c_h={c_h} N={n}: rel-L2 {err:.3e}")
    assert err <= BF16_TOL


@pytest.mark.parametrize("c,heads", [(64, 4), (384, 12), (56, 8)])
@pytest.mark.parametrize("starting", [True, False])
def test_triangle_attention_general_width(c, heads, starting, cuda_device):
    n = 130  # two key tiles, the second partial
    mod = TriangleAttention(c_in=c, c_hidden=32, no_heads=heads, starting=starting)
    params = _params(mod)
    _, z, mask = make_inputs(n, c_z=c, seed=2, pad_frac=0.1, with_s=False)
    zb, md = z.to(cuda_device, torch.bfloat16), mask.to(cuda_device)
    with torch.no_grad():
        got = cuda_module(mod, params, cuda_device)(zb, mask=md)
        assert _abi.last_path() == "tc.rows"
        with exact_fp32():
            want = O.triangle_attention(zb.float(), md, _dev(params, cuda_device), heads, starting=starting)
    assert _abi.device_status(clear=True) == 0
    err = rel_l2(got, want)
    print(f"triatt {'start' if starting else 'end'} c={c} H={heads} N={n}: rel-L2 {err:.3e}")
    assert err <= BF16_TOL


def test_triangle_attention_general_width_ragged(cuda_device):
    """Random holes and a fully masked row (the uniform-row rule of the core)."""
    n, c, heads = 77, 384, 12
    mod = TriangleAttention(c_in=c, c_hidden=32, no_heads=heads, starting=True)
    params = _params(mod, seed=4)
    z, m = _pair(n, c, 5, cuda_device), _mask(n, cuda_device)
    with torch.no_grad():
        got = cuda_module(mod, params, cuda_device)(z, mask=m)
        with exact_fp32():
            want = O.triangle_attention(z.float(), m, _dev(params, cuda_device), heads, starting=True)
    assert _abi.device_status(clear=True) == 0
    assert rel_l2(got, want) <= BF16_TOL


@pytest.mark.parametrize("c,n_mult", [(64, 2), (384, 2), (384, 4), (128, 2)])
def test_transition_general_width(c, n_mult, cuda_device):
    mod = Transition(c_in=c, n=n_mult)
    params = _params(mod)
    x = _pair(45, c, 6, cuda_device)
    with torch.no_grad():
        got = cuda_module(mod, params, cuda_device)(x)
        assert _abi.last_path() == "tc.rows"
        with exact_fp32():
            want = O.transition(x.float(), _dev(params, cuda_device))
    assert _abi.device_status(clear=True) == 0
    err = rel_l2(got, want)
    print(f"transition c={c} n={n_mult}: rel-L2 {err:.3e}")
    assert err <= BF16_TOL


def test_pair_bias_general_width(cuda_device):
    """AttentionPairBias of the refiner: 16 heads over c_z = 384 (the pair bias on tcgen05)."""
    n, c_s, c_z = 96, 384, 384
    mod = AttentionPairBias(has_s=False, create_offset_ln_z=True, n_heads=16, c_a=c_s, c_z=c_z)
    params = _params(mod)
    g = torch.Generator().manual_seed(7)
    s = torch.randn((n, c_s), generator=g).to(cuda_device, torch.bfloat16)
    z = _pair(n, c_z, 8, cuda_device)
    with torch.no_grad():
        got = cuda_module(mod, params, cuda_device)(a=s, s=None, z=z)
        assert _abi.last_path() == "tc+simt"
        with exact_fp32():
            want = O.attention_pair_bias(s.float(), z.float(), _dev(params, cuda_device), 16)
    assert _abi.device_status(clear=True) == 0
    err = rel_l2(got, want)
    print(f"attention pair bias c_z={c_z}: rel-L2 {err:.3e}")
    assert err <= BF16_TOL


@pytest.mark.parametrize("c_z,c_h", [(64, 128), (384, 384)])
def test_trimul_split_stages_match_one_call(c_z, c_h, cuda_device):
    """pf_trimul_project + pf_trimul_combine (the Fold-CP exchange points) == pf_trimul_fwd."""
    n = 70
    mod = TriangleMultiplicationOutgoing(c_z=c_z, c_hidden=c_h)
    seeded_init_(mod, seed=1, perturb_1d=True)
    mod = mod.to(cuda_device)
    pack = mod.weight_pack(torch.bfloat16, cuda_device)
    z, m = _pair(n, c_z, 9, cuda_device), _mask(n, cuda_device)
    want = torch.empty_like(z)
    kernels.trimul(pack, z, z, m, m, z, want, c_h, accumulate=False)
    ld = (n + 7) // 8 * 8
    a = torch.zeros((c_h, n, ld), device=cuda_device, dtype=torch.bfloat16)
    b = torch.zeros_like(a)
    kernels.trimul_project(pack, z, m, c_h, a.data_ptr(), b.data_ptr(), ld)
    assert _abi.last_path() == "tc.rows"
    got = torch.empty_like(z)
    kernels.trimul_combine(pack, a, b, n, z, got, accumulate=False)
    torch.cuda.synchronize()
    assert _abi.device_status(clear=True) == 0
    assert torch.equal(got, want)


def _sub(p, prefix):
    k0 = prefix + "."
    return {k[len(k0):]: v for k, v in p.items() if k.startswith(k0)}


STACKS = {
    # the template embedder's stack: c_z = 64, no single representation, transition x2
    "template": dict(kw=dict(n_blocks=2, c_z=64, c_s=0, num_intermediate_factor=2), heads_pair=4),
    # the structural refiner: c_z = c_h = 384, 12 pair heads, transition x2, c_s = 384
    "refiner": dict(kw=dict(n_blocks=2, n_heads=16, c_z=384, c_s=384, hidden_scale_up=True,
                            num_intermediate_factor=2), heads_pair=12),
}


@pytest.mark.parametrize("name", sorted(STACKS))
def test_stack_real_model_configuration(name, cuda_device):
    cfg = STACKS[name]
    kw = cfg["kw"]
    stack = PairformerStack(**kw)
    params = seeded_init_(stack, seed=0)
    stack = stack.to(cuda_device)
    n, c_z, c_s = 72, kw["c_z"], kw["c_s"]
    s, z, mask = make_inputs(n, c_z=c_z, c_s=max(c_s, 1), seed=1, pad_frac=0.1)
    md = mask.to(cuda_device)
    pd = _dev(params, cuda_device)
    zb = z.to(cuda_device, torch.bfloat16)
    sb = s.to(cuda_device, torch.bfloat16) if c_s > 0 else None
    with torch.no_grad():
        s_full, z_full = stack(sb, zb, md)
        for bi, blk in enumerate(stack.blocks):
            with exact_fp32():
                sc, zc = O.pairformer_block(sb.float() if sb is not None else None, zb.float(), md,
                                            _sub(pd, f"blocks.{bi}"), no_heads_pair=cfg["heads_pair"], n_heads=16,
                                            c_s=c_s)
            sb, zb = blk(sb, zb, md)
            ez = rel_l2(zb, zc)
            es = rel_l2(sb, sc) if c_s > 0 else 0.0
            print(f"{name} block {bi + 1}: z {ez:.3e} s {es:.3e}")
            assert ez <= BF16_TOL and es <= BF16_TOL
    assert _abi.device_status(clear=True) == 0
    assert torch.equal(z_full, zb)
