"""Pair heads and the diffusion pair conditioning on the GPU (pf_pair_head_fwd,
pf_confidence_pair_init_fwd, pf_diffusion_pair_cond_fwd):

* fp32 (SIMT) against the reference's own outputs (tests/golden/heads, N = 23): max-abs <= 1e-4
  relative to the output's magnitude;
* bf16 (tcgen05 row GEMM with the bias and softmax in its epilogue) against the fp32 oracle at the
  released widths (c_z = 128 / 384, 64 / 96 bins, c_z_pair_diffusion = 128): rel-L2 <= 2e-2, contact
  probabilities max-abs <= 2e-2;
* tiles (row / column offsets, strided outputs) bit-identical to the same positions of the full
  plane, and the transposed-partner form used by Fold-CP.
"""
import os
import sys

import numpy as np
import pytest
import torch

from gpu_helpers import rel_l2
from oracle import pairformer_oracle as O
from opendde_b200 import _abi
from opendde_b200.model import ConfidencePairHead, DiffusionPairConditioning, DistogramHead
from opendde_b200.model.heads import contact_bin_count
from opendde_b200.model.trunk_init import LazyRelativePositionEncodingFeatures
from opendde_b200.utils import seeded_params

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
import make_heads_golden as G  # noqa: E402

pytestmark = pytest.mark.gpu
BF16_TOL = 2e-2
ID_KEYS = ("asym_id", "residue_index", "entity_id", "token_index", "sym_id")


def load(name):
    return dict(np.load(os.path.join(HERE, "golden", "heads", f"{name}_n{G.N}.npz")))


def fp32_err(got, want):
    want = torch.as_tensor(want).double()
    return (got.double().cpu() - want).abs().max().item() / max(1.0, want.abs().max().item())


def set_params(mod, params, device):
    with torch.no_grad():
        for k, v in mod.named_parameters():
            if k in params:
                v.copy_(params[k])
    return mod.to(device)


def lazy(feats, device, r_max=32, s_max=2):
    return LazyRelativePositionEncodingFeatures(*[feats[k].to(device) for k in ID_KEYS], r_max=r_max, s_max=s_max)


def inputs(n, c_z, c_s_in, seed, device, dtype):
    g = torch.Generator().manual_seed(seed)
    z = torch.randn((n, n, c_z), generator=g)
    s_in = torch.randn((n, c_s_in), generator=g)
    coords = torch.randn((n, 3), generator=g) * 15.0
    chains = torch.arange(n) * 4 // n
    feats = {"asym_id": chains, "residue_index": torch.arange(n) - chains * 7, "entity_id": chains % 2,
             "token_index": torch.arange(n), "sym_id": chains // 2}
    return z, z.to(device, dtype), s_in, coords, feats


# ------------------------------------------------------------------ fp32 vs the reference's outputs
def test_distogram_fp32_matches_reference_outputs(cuda_device):
    rec = load("distogram")
    p = seeded_params(G.distogram_param_shapes(), seed=0, perturb_1d=True)
    head = set_params(DistogramHead(c_z=G.C_Z, no_bins=G.NB_DIST), p, cuda_device)
    z = G.heads_inputs()[0].to(cuda_device)
    with torch.no_grad():
        logits = head(z)
        assert _abi.last_path() == "simt"
        contact = head.contact_probs(z, G.MIN_BIN, G.MAX_BIN, G.NB_DIST, G.THRES)
    assert _abi.device_status(clear=True) == 0
    e1, e2 = fp32_err(logits, rec["logits"]), fp32_err(contact, rec["contact"])
    print(f"distogram fp32: logits {e1:.2e} contact {e2:.2e}")
    assert e1 <= 1e-4 and e2 <= 1e-4


def test_confidence_fp32_matches_reference_outputs(cuda_device):
    rec = load("confidence")
    p = seeded_params(G.confidence_param_shapes(), seed=1, perturb_1d=True)
    head = set_params(ConfidencePairHead(c_z=G.C_Z, c_s_inputs=G.C_S_IN, b_pae=G.B_PAE, b_pde=G.B_PDE), p,
                      cuda_device)
    z, s_in, coords, _ = G.heads_inputs()
    with torch.no_grad():
        zp = head.embed_pair(s_in.to(cuda_device), z.to(cuda_device), coords.to(cuda_device))
        pae, pde = head.pair_logits(zp)
    assert _abi.device_status(clear=True) == 0
    errs = [fp32_err(zp, rec["z_pair"]), fp32_err(pae, rec["pae"]), fp32_err(pde, rec["pde"])]
    print("confidence fp32: z_pair {:.2e} pae {:.2e} pde {:.2e}".format(*errs))
    assert max(errs) <= 1e-4


@pytest.mark.parametrize("name,c_zd", [("diffusion_compress", G.C_ZD), ("diffusion_plain", G.C_Z)])
def test_diffusion_fp32_matches_reference_outputs(name, c_zd, cuda_device):
    rec = load(name)
    p = seeded_params(G.diffusion_param_shapes(c_zd=c_zd), seed=2, perturb_1d=True)
    mod = set_params(DiffusionPairConditioning(c_z=G.C_Z, c_z_pair_diffusion=c_zd), p, cuda_device)
    z, _, _, feats = G.heads_inputs()
    with torch.no_grad():
        out = mod.prepare_cache(lazy(feats, cuda_device), z.to(cuda_device))
    assert _abi.device_status(clear=True) == 0
    e = fp32_err(out, rec["pair_z"])
    print(f"{name} fp32: {e:.2e}")
    assert e <= 1e-4


# ------------------------------------------------------------------ bf16 (tensor cores) vs the oracle
@pytest.mark.parametrize("n,c_z,bins", [(200, 128, 64), (131, 384, 96), (77, 40, 24)])
def test_distogram_bf16_against_oracle(n, c_z, bins, cuda_device):
    p = seeded_params(G.distogram_param_shapes(c_z, bins), seed=3, perturb_1d=True)
    head = set_params(DistogramHead(c_z=c_z, no_bins=bins), p, cuda_device)
    _, zb, _, _, _ = inputs(n, c_z, 8, 4, cuda_device, torch.bfloat16)
    with torch.no_grad():
        logits = head(zb)
        assert _abi.last_path() == "tc.rows" and logits.dtype == torch.bfloat16
        contact = head.contact_probs(zb, 2.25, 25.75, bins, 8.0)
    assert _abi.device_status(clear=True) == 0
    want = O.distogram_logits(zb.float().cpu(), p)
    want_c = O.contact_probs(want, 2.25, 25.75, bins, 8.0)
    e1, e2 = rel_l2(logits, want), (contact.cpu() - want_c).abs().max().item()
    print(f"distogram bf16 N={n} c_z={c_z} bins={bins}: logits rel-L2 {e1:.2e}, contact max-abs {e2:.2e}")
    assert e1 <= BF16_TOL and e2 <= BF16_TOL
    assert torch.equal(logits, logits.transpose(0, 1))


@pytest.mark.parametrize("n,c_z,c_s_in", [(160, 128, 449), (96, 384, 449), (45, 32, 40)])
def test_confidence_bf16_against_oracle(n, c_z, c_s_in, cuda_device):
    p = seeded_params(G.confidence_param_shapes(c_z, c_s_in, 64, 64), seed=5, perturb_1d=True)
    p["lower_bins"], p["upper_bins"] = G.distance_bins()
    head = set_params(ConfidencePairHead(c_z=c_z, c_s_inputs=c_s_in), p, cuda_device)
    _, zb, s_in, coords, _ = inputs(n, c_z, c_s_in, 6, cuda_device, torch.bfloat16)
    with torch.no_grad():
        zp = head.embed_pair(s_in.to(cuda_device, torch.bfloat16), zb, coords.to(cuda_device))
        pae, pde = head.pair_logits(zp)
        assert _abi.last_path() == "tc.rows" and pae.dtype == torch.float32
    assert _abi.device_status(clear=True) == 0
    pb = {k: (v.to(torch.bfloat16).float() if v.dim() == 2 else v) for k, v in p.items()}
    want = O.confidence_pair_init(zb.float().cpu(), s_in.to(torch.bfloat16).float(), coords, pb)
    e0 = rel_l2(zp, want)
    pae_w, pde_w = O.confidence_pair_logits(zp.float().cpu(), p)
    e1, e2 = rel_l2(pae, pae_w), rel_l2(pde, pde_w)
    print(f"confidence bf16 N={n} c_z={c_z}: z_pair {e0:.2e} pae {e1:.2e} pde {e2:.2e}")
    assert max(e0, e1, e2) <= BF16_TOL
    assert torch.allclose(pde, pde.transpose(0, 1), atol=1e-5, rtol=0)


@pytest.mark.parametrize("n,c_z,c_zd", [(128, 384, 128), (96, 128, 128), (50, 64, 32)])
def test_diffusion_bf16_against_oracle(n, c_z, c_zd, cuda_device):
    p = seeded_params(G.diffusion_param_shapes(c_z, c_zd), seed=7, perturb_1d=True)
    mod = set_params(DiffusionPairConditioning(c_z=c_z, c_z_pair_diffusion=c_zd), p, cuda_device)
    _, zb, _, _, feats = inputs(n, c_z, 8, 8, cuda_device, torch.bfloat16)
    with torch.no_grad():
        out = mod.prepare_cache(lazy(feats, cuda_device), zb)
        assert _abi.last_path() == "tc.rows"
    assert _abi.device_status(clear=True) == 0
    e = rel_l2(out, O.diffusion_pair_conditioning(zb.float().cpu(), feats, p))
    print(f"diffusion bf16 N={n} c_z={c_z} c_zd={c_zd}: rel-L2 {e:.2e}")
    assert e <= BF16_TOL


# ------------------------------------------------------------------ tiles and the transposed partner
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_tiles_equal_the_full_plane(dtype, cuda_device):
    """Each kernel on a tile (row / column offsets, strided output views) writes exactly the full
    plane's values there; the heads on a tile with its transposed partner (the Fold-CP form)
    equal the full plane's."""
    n, c_z, c_s_in = 90, 128, 64
    _, z, s_in, coords, feats = inputs(n, c_z, c_s_in, 9, cuda_device, dtype)
    s_in, coords = s_in.to(cuda_device, dtype), coords.to(cuda_device)
    dh = set_params(DistogramHead(c_z, 64), seeded_params(G.distogram_param_shapes(c_z, 64), seed=1,
                                                          perturb_1d=True), cuda_device)
    ch = set_params(ConfidencePairHead(c_z=c_z, c_s_inputs=c_s_in),
                    seeded_params(G.confidence_param_shapes(c_z, c_s_in, 64, 64), seed=2, perturb_1d=True),
                    cuda_device)
    dc = set_params(DiffusionPairConditioning(c_z, 64), seeded_params(G.diffusion_param_shapes(c_z, 64), seed=3,
                                                                      perturb_1d=True), cuda_device)
    relp = lazy(feats, cuda_device)
    r0, r1, c0, c1 = 17, 61, 40, 90
    n_c = contact_bin_count(2.25, 25.75, 64, 8.0, dtype)
    with torch.no_grad():
        logits = dh(z)
        contact = dh.contact_probs(z, 2.25, 25.75, 64, 8.0)
        zp = ch.embed_pair(s_in, z, coords)
        pae, pde = ch.pair_logits(zp)
        dz = dc.prepare_cache(relp, z)
        zt = z.transpose(0, 1)
        lt = torch.zeros((r1 - r0, c1 - c0, 64), device=cuda_device, dtype=dtype)
        ct = torch.zeros((r1 - r0, c1 - c0 + 5), device=cuda_device)[:, :c1 - c0]    # strided contact view
        dh.logits_tile(z[r0:r1, c0:c1], zt[r0:r1, c0:c1], lt, ct, n_c)
        zpt = z[r0:r1, c0:c1].clone()
        ch.embed_pair_tile(s_in, coords, zpt, zpt, r0, c0)
        pt = torch.zeros((r1 - r0, c1 - c0, 64), device=cuda_device)
        qt = torch.zeros((r1 - r0, c1 - c0, 64), device=cuda_device)
        ch.pair_logits_tile(zp[r0:r1, c0:c1], zp.transpose(0, 1)[r0:r1, c0:c1], pt, qt)
        big = torch.zeros((n + 5, n + 7, 64), device=cuda_device, dtype=dtype)   # strided output view
        dc.prepare_cache_tile(relp, z[r0:r1, c0:c1], big[r0:r1, c0:c1], r0, c0)
    assert _abi.device_status(clear=True) == 0
    assert torch.equal(lt, logits[r0:r1, c0:c1])
    assert torch.equal(ct, contact[r0:r1, c0:c1])
    assert torch.equal(zpt, zp[r0:r1, c0:c1])
    assert torch.equal(pt, pae[r0:r1, c0:c1]) and torch.equal(qt, pde[r0:r1, c0:c1])
    assert torch.equal(big[r0:r1, c0:c1], dz[r0:r1, c0:c1])
    assert big[:r0].abs().sum().item() == 0 and big[r1:].abs().sum().item() == 0


def test_head_rejects_bad_arguments(cuda_device):
    head = DistogramHead(32, 16).to(cuda_device)
    z = torch.zeros((8, 8, 32), device=cuda_device)
    with pytest.raises(_abi.PFError, match="fp32 input needs fp32 logits"):
        head.logits_tile(z, z.transpose(0, 1), torch.zeros((8, 8, 16), device=cuda_device, dtype=torch.bfloat16))
    with pytest.raises(_abi.PFError, match="contact_bins"):
        head.logits_tile(z, z.transpose(0, 1), torch.zeros((8, 8, 16), device=cuda_device),
                         torch.zeros((8, 8), device=cuda_device), 17)
