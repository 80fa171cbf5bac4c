"""The oracle's restatement of the pair heads and the diffusion pair conditioning against the
reference's own outputs (tests/golden/heads, made by tests/golden/make_heads_golden.py from
DistogramHead, the Fold-CP contact helper, ConfidenceHead and DiffusionConditioning), and the tile
forms against the full plane."""
import os
import sys

import numpy as np
import pytest
import torch

from oracle import pairformer_oracle as O
from opendde_b200.utils import seeded_params

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
import make_heads_golden as G  # noqa: E402

TOL = 2e-5


def load(name):
    return dict(np.load(os.path.join(HERE, "golden", "heads", f"{name}_n{G.N}.npz")))


def close(got, want, tol=TOL):
    want = torch.as_tensor(want)
    err = (got - want).abs().max().item() / max(1.0, want.abs().max().item())
    assert err <= tol, err


def check_fixture(rec, params):
    z, s_inputs, coords, _ = G.heads_inputs()
    assert np.allclose(G.checksum(z), rec["chk_z"]) and np.allclose(G.checksum(coords), rec["chk_coords"])
    assert np.allclose(G.checksum(s_inputs), rec["chk_s_inputs"])
    assert list(rec["param_names"]) == sorted(params)
    assert np.allclose(np.stack([G.checksum(params[k]) for k in sorted(params)]), rec["chk_params"])


def test_distogram_logits_and_contact_probs():
    rec = load("distogram")
    p = seeded_params(G.distogram_param_shapes(), seed=0, perturb_1d=True)
    check_fixture(rec, p)
    z = G.heads_inputs()[0]
    logits = O.distogram_logits(z, p)
    close(logits, rec["logits"])
    close(O.contact_probs(logits, G.MIN_BIN, G.MAX_BIN, G.NB_DIST, G.THRES), rec["contact"])
    assert torch.equal(logits, logits.transpose(0, 1))


def test_confidence_pair_input_and_logits():
    rec = load("confidence")
    p = seeded_params(G.confidence_param_shapes(), seed=1, perturb_1d=True)
    check_fixture(rec, p)
    p["lower_bins"], p["upper_bins"] = G.distance_bins()
    z, s_inputs, coords, _ = G.heads_inputs()
    close(O.confidence_pair_init(z, s_inputs, coords, p), rec["z_pair"])
    pae, pde = O.confidence_pair_logits(torch.from_numpy(rec["z_pair"]), p)
    close(pae, rec["pae"])
    close(pde, rec["pde"])


@pytest.mark.parametrize("name,c_zd", [("diffusion_compress", G.C_ZD), ("diffusion_plain", G.C_Z)])
def test_diffusion_pair_conditioning(name, c_zd):
    rec = load(name)
    p = seeded_params(G.diffusion_param_shapes(c_zd=c_zd), seed=2, perturb_1d=True)
    check_fixture(rec, p)
    z, _, _, feats = G.heads_inputs()
    close(O.diffusion_pair_conditioning(z, feats, p, G.R_MAX, G.S_MAX), rec["pair_z"])


def test_tile_forms_are_slices_of_the_plane():
    z, s_inputs, coords, feats = G.heads_inputs()
    pc = seeded_params(G.confidence_param_shapes(), seed=1, perturb_1d=True)
    pc["lower_bins"], pc["upper_bins"] = G.distance_bins()
    pd = seeded_params(G.diffusion_param_shapes(), seed=2, perturb_1d=True)
    rows, cols = slice(3, 17), slice(9, 23)
    close(O.confidence_pair_init(z[rows, cols], s_inputs, coords, pc, rows, cols),
          O.confidence_pair_init(z, s_inputs, coords, pc)[rows, cols], 1e-6)
    close(O.diffusion_pair_conditioning(z[rows, cols], feats, pd, rows=rows, cols=cols),
          O.diffusion_pair_conditioning(z, feats, pd)[rows, cols], 1e-6)


def test_distances_direct_form_matches_cdist_below_the_matrix_product_switch():
    """N <= 25: torch.cdist's default mode is the direct form, so the two agree exactly."""
    coords = G.heads_inputs()[2]
    assert torch.equal(O.pair_distances(coords), torch.cdist(coords, coords))
