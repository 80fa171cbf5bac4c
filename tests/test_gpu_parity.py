"""CUDA path vs the reference's golden vectors and vs the CPU oracle (parity tests proper).

Tolerances (the parity contract of this path): fp32 mode max-abs <= 1e-4; bf16 mode relative-L2 <= 2e-2
against the fp32 oracle on the same seeded inputs and weights.
"""
import pytest
import torch

from golden_cases import CASE_FILES, load_case, module_for
from gpu_helpers import cuda_module, cuda_op, max_abs, oracle_op, rel_l2
from oracle import pairformer_oracle as O
from opendde_b200 import _abi
from opendde_b200.utils import make_inputs, ragged_pair_mask, seeded_params

pytestmark = pytest.mark.gpu

FP32_TOL = 1e-4
BF16_TOL = 2e-2
OPS = ["trimul_out", "trimul_in", "triatt_start", "triatt_end", "transition", "apb"]


@pytest.mark.parametrize("fname", CASE_FILES)
def test_fp32_matches_reference_golden(fname, cuda_device):
    kind, n, s, z, mask, params, rec, mod = load_case(fname)
    mod = cuda_module(mod, params, cuda_device)
    if kind.startswith("block"):
        with torch.no_grad():
            s_out, z_out = mod(s.to(cuda_device), z.to(cuda_device), mask.to(cuda_device))
        assert max_abs(z_out, torch.from_numpy(rec["z_out"])) <= FP32_TOL
        assert max_abs(s_out, torch.from_numpy(rec["s_out"])) <= FP32_TOL
    else:
        got = cuda_op(kind, mod, s, z, mask, cuda_device, torch.float32)
        err = max_abs(got, torch.from_numpy(rec["out"]))
        assert err <= FP32_TOL, f"{fname}: max-abs {err:.3e}"


def _case(kind, n, pad_frac=0.0, ragged=False, seed_w=0, full_rows=()):
    mod = module_for(kind)
    params = seeded_params([(k, tuple(p.shape)) for k, p in mod.named_parameters()], seed=seed_w,
                           perturb_1d=True)
    s, z, mask = make_inputs(n, seed=1, pad_frac=pad_frac)
    if ragged:
        mask = ragged_pair_mask(n, seed=3, drop=0.2, full_rows=full_rows)
    return mod, params, s, z, mask


@pytest.mark.parametrize("kind", OPS)
@pytest.mark.parametrize("n", [1, 2, 33, 70])
def test_fp32_edge_sizes_vs_oracle(kind, n, cuda_device):
    mod, params, s, z, mask = _case(kind, n, ragged=True, full_rows=[0] if n > 1 else [])
    want = oracle_op(kind, s, z, mask, params)
    got = cuda_op(kind, cuda_module(mod, params, cuda_device), s, z, mask, cuda_device, torch.float32)
    assert max_abs(got, want) <= FP32_TOL


def test_c0_block_fp32_n128(cuda_device):
    """Config C0: one block, fp32, N=128, all-ones mask, seed-0 weights."""
    mod = module_for("block")
    params = seeded_params([(k, tuple(p.shape)) for k, p in mod.named_parameters()], seed=0)
    s, z, mask = make_inputs(128, seed=1)
    torch.set_num_threads(8)
    with torch.no_grad():
        s_ref, z_ref = O.pairformer_block(s, z, mask, params)
        s_out, z_out = cuda_module(mod, params, cuda_device)(s.to(cuda_device), z.to(cuda_device),
                                                              mask.to(cuda_device))
    assert max_abs(z_out, z_ref) <= FP32_TOL
    assert max_abs(s_out, s_ref) <= FP32_TOL


@pytest.mark.parametrize("kind", OPS)
@pytest.mark.parametrize("n", [48, 160])
@pytest.mark.parametrize("path", ["dispatch", "simt"])
def test_bf16_vs_fp32_oracle(kind, n, path, cuda_device):
    mod, params, s, z, mask = _case(kind, n, pad_frac=0.1)
    want = oracle_op(kind, s.bfloat16().float(), z.bfloat16().float(), mask, params)
    _abi.set_force_simt(path == "simt")
    try:
        got = cuda_op(kind, cuda_module(mod, params, cuda_device), s, z, mask, cuda_device, torch.bfloat16)
    finally:
        _abi.set_force_simt(False)
    err = rel_l2(got, want)
    assert err <= BF16_TOL, f"{kind} n={n} {path}: rel-L2 {err:.3e}"


def test_block_bf16_vs_fp32_oracle(cuda_device):
    mod = module_for("block")
    params = seeded_params([(k, tuple(p.shape)) for k, p in mod.named_parameters()], seed=0)
    s, z, mask = make_inputs(96, seed=1, pad_frac=0.1)
    with torch.no_grad():
        s_ref, z_ref = O.pairformer_block(s.bfloat16().float(), z.bfloat16().float(), mask, params)
        s_out, z_out = cuda_module(mod, params, cuda_device)(
            s.to(cuda_device, torch.bfloat16), z.to(cuda_device, torch.bfloat16), mask.to(cuda_device))
    assert rel_l2(z_out, z_ref) <= BF16_TOL
    assert rel_l2(s_out, s_ref) <= BF16_TOL


@pytest.mark.parametrize("kind", ["trimul_out", "trimul_in", "triatt_start", "triatt_end", "transition", "apb"])
@pytest.mark.parametrize("n", [300])
def test_bf16_tensor_core_path_vs_simt_path(kind, n, cuda_device):
    """The tcgen05 kernels and the SIMT kernels agree on one bf16 problem with partial tiles."""
    mod, params, s, z, mask = _case(kind, n, ragged=True, full_rows=[5])
    mod = cuda_module(mod, params, cuda_device)
    got_tc = cuda_op(kind, mod, s, z, mask, cuda_device, torch.bfloat16)
    path = _abi.last_path()
    _abi.set_force_simt(True)
    try:
        got_simt = cuda_op(kind, mod, s, z, mask, cuda_device, torch.bfloat16)
    finally:
        _abi.set_force_simt(False)
    # apb: the pair bias runs on the tensor cores, the N-token single attention on SIMT.
    assert path == ("tc+simt" if kind == "apb" else "tc"), f"{kind} dispatched to {path}"
    assert _abi.device_status(clear=True) == 0
    err = rel_l2(got_tc, got_simt)
    assert err <= 1e-2, f"{kind}: tc vs simt rel-L2 {err:.3e}"


@pytest.mark.parametrize("reserve", [0, 64])
def test_bf16_transition_persistent_pairs(reserve, cuda_device):
    """The persistent transition walks several 256-row pairs per CTA (299^2 rows = 349 pairs +
    57 rows: ~2.4 pairs per CTA on 148 SMs, ~4.2 with 64 SMs reserved) and ends on a one-tile
    pair: bit-identical to the run on every SM, and within the bf16 bar of the SIMT path."""
    mod, params, s, z, mask = _case("transition", 299)
    mod = cuda_module(mod, params, cuda_device)
    base = cuda_op("transition", mod, s, z, mask, cuda_device, torch.bfloat16)
    _abi.set_sm_reserve(reserve)
    try:
        got = cuda_op("transition", mod, s, z, mask, cuda_device, torch.bfloat16)
        assert _abi.last_path() == "tc"
    finally:
        _abi.set_sm_reserve(0)
    assert _abi.device_status(clear=True) == 0
    assert torch.equal(got, base)
    _abi.set_force_simt(True)
    try:
        want = cuda_op("transition", mod, s, z, mask, cuda_device, torch.bfloat16)
    finally:
        _abi.set_force_simt(False)
    err = rel_l2(got, want)
    assert err <= 1e-2, f"transition tc vs simt rel-L2 {err:.3e}"
