"""Module API of the pair heads and the diffusion pair conditioning (CPU): parameter names and
shapes against the reference modules' pair steps (recorded in tests/golden/heads by
tests/golden/make_heads_golden.py), no CPU fallback, and the contact-bin selection."""
import os
import sys

import numpy as np
import pytest
import torch

from opendde_b200.model import ConfidencePairHead, DiffusionPairConditioning, DistogramHead
from opendde_b200.model.heads import bin_tops, contact_bin_count
from oracle import pairformer_oracle as O

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
import make_heads_golden as G  # noqa: E402


def ref_state(name):
    rec = np.load(os.path.join(HERE, "golden", "heads", f"{name}_n{G.N}.npz"))
    return [str(x) for x in rec["ref_state"]]


def state(mod):
    return [f"{k}:{'x'.join(str(d) for d in v.shape)}" for k, v in mod.state_dict().items()]


def test_distogram_head_state_matches_reference():
    assert state(DistogramHead(c_z=G.C_Z, no_bins=G.NB_DIST)) == ref_state("distogram")


def test_confidence_pair_head_state_matches_reference_pair_steps():
    head = ConfidencePairHead(c_z=G.C_Z, c_s_inputs=G.C_S_IN, b_pae=G.B_PAE, b_pde=G.B_PDE)
    assert sorted(state(head)) == sorted(ref_state("confidence"))
    lower, upper = G.distance_bins()
    assert torch.equal(head.lower_bins.data, lower) and torch.equal(head.upper_bins.data, upper)


@pytest.mark.parametrize("name,c_zd", [("diffusion_compress", G.C_ZD), ("diffusion_plain", G.C_Z)])
def test_diffusion_pair_conditioning_state_matches_reference(name, c_zd):
    mod = DiffusionPairConditioning(c_z=G.C_Z, c_z_pair_diffusion=c_zd)
    assert state(mod) == ref_state(name)
    assert mod.compress_pair_z == (c_zd != G.C_Z)


def test_cpu_tensors_are_rejected_no_fallback():
    z = torch.zeros(5, 5, G.C_Z)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        DistogramHead(c_z=G.C_Z, no_bins=G.NB_DIST)(z)
    head = ConfidencePairHead(c_z=G.C_Z, c_s_inputs=G.C_S_IN, b_pae=G.B_PAE, b_pde=G.B_PDE)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        head.pair_logits(z)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        head.embed_pair(torch.zeros(5, G.C_S_IN), z, torch.zeros(5, 3))
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        DiffusionPairConditioning(c_z=G.C_Z).prepare_cache(None, z)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("min_bin,max_bin,no_bins,thres", [(2.25, 25.75, 96, 8.0), (2.25, 25.75, 24, 8.0),
                                                           (0.0, 32.0, 64, 8.0), (2.25, 25.75, 96, 1.0)])
def test_contact_bins_are_the_oracle_selection(dtype, min_bin, max_bin, no_bins, thres):
    """The kernel sums the first contact_bin_count bins; that prefix is exactly the reference's
    boolean selection tops <= thres, computed in the logits' dtype."""
    n = contact_bin_count(min_bin, max_bin, no_bins, thres, dtype)
    sel = O.distogram_bin_tops(min_bin, max_bin, no_bins, dtype) <= thres
    assert torch.equal(sel, torch.arange(no_bins) < n)
    assert torch.equal(bin_tops(min_bin, max_bin, no_bins, dtype), O.distogram_bin_tops(min_bin, max_bin, no_bins,
                                                                                         dtype))
