"""Parity at the stated configurations, against the fp32 oracle run on the GPU.

The oracle (the reference's algorithm restated in torch) runs here on CUDA tensors in fp32 with
TF32 off, so that problems of the benchmark configurations' sizes finish in seconds:

* C1: standalone triangle attention, starting and ending node, N = 384 and 768 with the last
  10 % of tokens padded, and rows of the N = 1536 problem (a row subset of the oracle);
* C2: standalone triangle multiplicative update, outgoing and incoming, N = 1024;
* drift of the bf16 trunk over many blocks (8 blocks at N = 256, all 48 blocks at N = 128),
  block by block against the fp32 oracle, and (context only) the same algorithm run in torch
  bf16 against the same oracle;
* large triangle-attention logits (q and k weights scaled up) against the oracle, and a logit
  past the f16 range reported through the status word instead of a silent NaN;
* the standalone LayerNorm entry point in both dtypes.

Tolerances: bf16 relative-L2 <= 2e-2 against the fp32 oracle; fp32 max-abs <= 1e-4.
"""
import contextlib
import math

import pytest
import torch

from golden_cases import module_for
from gpu_helpers import cuda_module, max_abs, rel_l2
from oracle import pairformer_oracle as O
from opendde_b200 import _abi, kernels
from opendde_b200.model import PairformerStack
from opendde_b200.utils import make_inputs, seeded_init_, seeded_params

pytestmark = pytest.mark.gpu

BF16_TOL = 2e-2
FP32_TOL = 1e-4


@contextlib.contextmanager
def exact_fp32():
    """fp32 matmuls without TF32 for the oracle on the GPU."""
    old = (torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32)
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    try:
        yield
    finally:
        torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32 = old


def _dev(params, device, dtype=torch.float32):
    return {k: v.to(device=device, dtype=dtype) for k, v in params.items()}


def _weights(kind, seed=0):
    mod = module_for(kind)
    params = seeded_params([(k, tuple(p.shape)) for k, p in mod.named_parameters()], seed=seed, perturb_1d=True)
    return mod, params


# ------------------------------------------------------------------------------ C1
@pytest.mark.parametrize("n", [384, 768])
@pytest.mark.parametrize("starting", [True, False])
def test_c1_triangle_attention(n, starting, cuda_device):
    kind = "triatt_start" if starting else "triatt_end"
    mod, params = _weights(kind)
    _, z, mask = make_inputs(n, seed=1, pad_frac=0.1, with_s=False)
    zb = z.to(cuda_device, torch.bfloat16)
    md = mask.to(cuda_device)
    with torch.no_grad():
        got = cuda_module(mod, params, cuda_device)(zb, mask=md)
        assert _abi.last_path() == "tc"
        with exact_fp32():
            want = O.triangle_attention(zb.float(), md, _dev(params, cuda_device), 4, starting=starting)
    assert _abi.device_status(clear=True) == 0
    err = rel_l2(got, want)
    print(f"C1 N={n} {'start' if starting else 'end'}: rel-L2 {err:.3e}")
    assert err <= BF16_TOL


@pytest.mark.parametrize("starting", [True, False])
@pytest.mark.parametrize("rows", [(0, 48), (1392, 1440), (1488, 1536)])
def test_c1_triangle_attention_n1536_row_subset(starting, rows, cuda_device):
    """N = 1536, 10 % padding: the whole op on the GPU, checked on row bands (valid rows, rows
    straddling the padding boundary at 1382, and padded rows) against the oracle."""
    n = 1536
    kind = "triatt_start" if starting else "triatt_end"
    mod, params = _weights(kind)
    _, z, mask = make_inputs(n, seed=1, pad_frac=0.1, with_s=False)
    zb = z.to(cuda_device, torch.bfloat16)
    md = mask.to(cuda_device)
    sl = slice(*rows)
    with torch.no_grad():
        got = cuda_module(mod, params, cuda_device)(zb, mask=md)
        with exact_fp32():
            want = O.triangle_attention(zb.float(), md, _dev(params, cuda_device), 4, starting=starting,
                                        rows=sl, row_chunk=16)
    got_rows = got[sl] if starting else got[:, sl]
    err = rel_l2(got_rows, want)
    print(f"C1 N=1536 {'start' if starting else 'end'} rows {rows}: rel-L2 {err:.3e}")
    assert err <= BF16_TOL


# ------------------------------------------------------------------------------ C2
@pytest.mark.parametrize("outgoing", [True, False])
def test_c2_triangle_multiplication_n1024(outgoing, cuda_device):
    n = 1024
    mod, params = _weights("trimul_out" if outgoing else "trimul_in")
    _, z, mask = make_inputs(n, seed=1, with_s=False)
    zb = z.to(cuda_device, torch.bfloat16)
    md = mask.to(cuda_device)
    with torch.no_grad():
        got = cuda_module(mod, params, cuda_device)(zb, mask=md)
        assert _abi.last_path() == "tc"
        with exact_fp32():
            want = O.triangle_multiplication(zb.float(), md, _dev(params, cuda_device), outgoing=outgoing)
    assert _abi.device_status(clear=True) == 0
    err = rel_l2(got, want)
    print(f"C2 N=1024 {'out' if outgoing else 'in'}: rel-L2 {err:.3e}")
    assert err <= BF16_TOL


# ------------------------------------------------------------------------------ drift
def _sub(p, prefix):
    k0 = prefix + "."
    return {k[len(k0):]: v for k, v in p.items() if k.startswith(k0)}


@pytest.mark.parametrize("n,blocks,pad", [(256, 8, 0.1), (128, 48, 0.0)])
def test_bf16_trunk_against_fp32_oracle(n, blocks, pad, cuda_device):
    """The bf16 trunk, block by block, against the fp32 oracle.

    * Per-block chain: every block's bf16 output against the fp32 oracle applied to that block's
      (bf16) input must be within the bf16 tolerance, for all blocks of the trunk.
    * Accumulated drift: the bf16 trunk run end to end from the shared input drifts from the
      fp32 trunk as bf16 rounding of the stored pair tensor compounds over the blocks; it must
      stay below the drift of the same algorithm evaluated with torch bf16 arithmetic (the
      reference modules' bf16 semantics: bf16 storage, bf16 GEMM outputs). Both are printed.
    """
    stack = PairformerStack(n_blocks=blocks, n_heads=16, c_z=128, c_s=384)
    params = seeded_init_(stack, seed=0)
    stack = stack.to(cuda_device)
    s, z, mask = make_inputs(n, seed=1, pad_frac=pad)
    md = mask.to(cuda_device)
    pd = _dev(params, cuda_device)
    pt = _dev(params, cuda_device, torch.bfloat16)
    zb, sb = z.to(cuda_device, torch.bfloat16), s.to(cuda_device, torch.bfloat16)
    zr, sr = zb.float(), sb.float()          # fp32 oracle trunk
    zt, st = zb.clone(), sb.clone()          # torch-bf16 trunk (context)
    chain, drift = [], []
    with torch.no_grad():
        # the whole stack through the public forward must equal the block-by-block chain
        s_full, z_full = stack(sb, zb, md)
        for bi, blk in enumerate(stack.blocks):
            p_bi = _sub(pd, f"blocks.{bi}")
            with exact_fp32():
                sc, zc = O.pairformer_block(sb.float(), zb.float(), md, p_bi)   # oracle from our input
                sr, zr = O.pairformer_block(sr, zr, md, p_bi)
            sb, zb = blk(sb, zb, md)
            st, zt = O.pairformer_block(st, zt, md.bfloat16(), _sub(pt, f"blocks.{bi}"))
            chain.append((rel_l2(zb, zc), rel_l2(sb, sc)))
            drift.append((rel_l2(zb, zr), rel_l2(sb, sr), rel_l2(zt, zr), rel_l2(st, sr)))
    assert _abi.device_status(clear=True) == 0
    assert torch.equal(z_full, zb) and torch.equal(s_full, sb)
    for bi, ((cz, cs), (ez, es, tz, ts)) in enumerate(zip(chain, drift)):
        print(f"trunk N={n} block {bi + 1}: per-block z {cz:.3e} s {cs:.3e} | drift z {ez:.3e} s {es:.3e} "
              f"| torch-bf16 drift z {tz:.3e} s {ts:.3e}")
    worst = max(max(c) for c in chain)
    assert worst <= BF16_TOL, f"worst per-block rel-L2 {worst:.3e}"
    ez, es, tz, ts = drift[-1]
    assert ez <= tz and es <= ts, f"drift z {ez:.3e} s {es:.3e} above torch-bf16's z {tz:.3e} s {ts:.3e}"


# ------------------------------------------------------------------------------ large logits
@pytest.mark.parametrize("scale", [2.0, 4.0, 8.0])
@pytest.mark.parametrize("starting", [True, False])
def test_triangle_attention_large_logits(scale, starting, cuda_device):
    """q and k weights scaled by `scale` each: logits grow by scale^2 (the largest reach
    ~ 6 scale^2 in natural units), so softmax rows approach one-hot and small logit errors
    become visible. The bf16 path must stay within the bf16 tolerance up to 4x larger logits
    than the seeded weights give, and beyond that no worse than the same attention evaluated
    with torch bf16 arithmetic (bf16 logits, as the reference's bf16 path computes them)."""
    n = 160
    kind = "triatt_start" if starting else "triatt_end"
    mod, params = _weights(kind)
    params["mha.linear_q.weight"] = params["mha.linear_q.weight"] * scale
    params["mha.linear_k.weight"] = params["mha.linear_k.weight"] * scale
    _, z, mask = make_inputs(n, seed=1, pad_frac=0.1, with_s=False)
    zb = z.to(cuda_device, torch.bfloat16)
    md = mask.to(cuda_device)
    with torch.no_grad():
        got = cuda_module(mod, params, cuda_device)(zb, mask=md)
        with exact_fp32():
            pd = _dev(params, cuda_device)
            want = O.triangle_attention(zb.float(), md, pd, 4, starting=starting)
            x = O.layer_norm(zb.float(), pd["layer_norm.weight"], pd["layer_norm.bias"])
            q = O.linear(x, pd["mha.linear_q.weight"]).view(n, n, 4, 32)
            k = O.linear(x, pd["mha.linear_k.weight"]).view(n, n, 4, 32)
            peak = torch.einsum("ijhd,ikhd->ihjk", q[:16], k[:16]).abs().max().item() / math.sqrt(32)
        tb = O.triangle_attention(zb, md.bfloat16(), _dev(params, cuda_device, torch.bfloat16), 4,
                                  starting=starting)
    assert _abi.device_status(clear=True) == 0
    err, err_t = rel_l2(got, want), rel_l2(tb, want)
    print(f"large logits x{scale}^2 {'start' if starting else 'end'}: max |logit| (rows 0-15) {peak:.1f}, "
          f"rel-L2 {err:.3e} (torch bf16 {err_t:.3e})")
    if scale <= 2.0:
        assert err <= BF16_TOL
    else:
        assert err <= err_t


def test_triangle_attention_logit_overflow_is_reported(cuda_device):
    """A logit past the f16 range (here ~1e5 after the log2(e)/sqrt(d) scaling) cannot be held
    by the bf16 path's f16 logit accumulator; the kernel reports it in the status word (bit 1)
    and the module forward raises at its checkpoint, instead of returning NaN rows silently."""
    n = 64
    mod, params = _weights("triatt_start")
    params["mha.linear_q.weight"] = params["mha.linear_q.weight"] * 300.0
    params["mha.linear_k.weight"] = params["mha.linear_k.weight"] * 300.0
    _, z, mask = make_inputs(n, seed=1, with_s=False)
    zb = z.to(cuda_device, torch.bfloat16)
    md = mask.to(cuda_device)
    assert _abi.device_status(clear=True) == 0
    with torch.no_grad():
        cuda_module(mod, params, cuda_device)(zb, mask=md)
    word = _abi.device_status(clear=True)
    assert word & 2, f"status word {word:#x}"
    assert "f16 range" in _abi.status_message(word)


# ------------------------------------------------------------------------------ LayerNorm
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("c", [128, 384, 64, 24])
def test_standalone_layernorm(dtype, c, cuda_device):
    rows = 3001
    g = torch.Generator().manual_seed(c)
    x = torch.randn((rows, c), generator=g) * 3 + 0.5
    w = 1 + 0.1 * torch.randn(c, generator=g)
    b = 0.1 * torch.randn(c, generator=g)
    xd = x.to(cuda_device, dtype)
    got = kernels.layernorm(xd, w.to(cuda_device), b.to(cuda_device))
    want = O.layer_norm(xd.float().cpu(), w, b)
    if dtype == torch.float32:
        assert max_abs(got, want) <= FP32_TOL
    else:
        assert rel_l2(got, want) <= 1e-2  # one bf16 rounding of the output
    none = kernels.layernorm(xd, None, None)
    assert rel_l2(none, O.layer_norm(xd.float().cpu(), None, None)) <= 1e-2
