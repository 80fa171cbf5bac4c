"""The trunk pair-initialisation restatement in the oracle (relative-position features, z_init,
one recycling step) against the reference's own outputs (tests/golden/trunk, made by
tests/golden/make_trunk_golden.py from the reference modules), and the tile form the Fold-CP
local construction uses against the full plane."""
import os
import sys

import numpy as np
import torch

from oracle import pairformer_oracle as O
from opendde_b200.utils import seeded_params

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
from make_trunk_golden import checksum, trunk_inputs, trunk_param_shapes  # noqa: E402

PATH = os.path.join(HERE, "golden", "trunk", "trunk_init_n23.npz")


def load():
    rec = dict(np.load(PATH))
    params = seeded_params(trunk_param_shapes(), seed=0, perturb_1d=True)
    return rec, params, trunk_inputs()


def test_inputs_and_weights_match_the_fixture():
    rec, params, (feats, bonds, s_init, z_prev) = load()
    assert np.allclose(checksum(s_init), rec["chk_s"]) and np.allclose(checksum(z_prev), rec["chk_z_prev"])
    assert np.allclose(checksum(bonds), rec["chk_bonds"])
    assert list(rec["param_names"]) == sorted(params)
    assert np.allclose(np.stack([checksum(params[k]) for k in sorted(params)]), rec["chk_params"])


def test_relp_features_match_reference():
    rec, _, (feats, _, _, _) = load()
    got = O.relp_features(**feats, r_max=int(rec["r_max"]), s_max=int(rec["s_max"]))
    assert torch.equal(got, torch.from_numpy(rec["relp"]))


def test_trunk_z_init_and_cycle_match_reference():
    rec, params, (feats, bonds, s_init, z_prev) = load()
    z_init = O.trunk_z_init(s_init, feats, bonds, params, int(rec["r_max"]), int(rec["s_max"]))
    assert (z_init - torch.from_numpy(rec["z_init"])).abs().max().item() <= 2e-5
    z_cyc = O.trunk_z_cycle(z_init, z_prev, params)
    assert (z_cyc - torch.from_numpy(rec["z_cycle"])).abs().max().item() <= 2e-5


def test_trunk_z_init_tile_is_a_slice_of_the_plane():
    rec, params, (feats, bonds, s_init, _) = load()
    full = O.trunk_z_init(s_init, feats, bonds, params, int(rec["r_max"]), int(rec["s_max"]))
    tile = O.trunk_z_init(s_init, feats, bonds, params, int(rec["r_max"]), int(rec["s_max"]),
                          rows=slice(6, 17), cols=slice(12, 23))
    assert torch.allclose(tile, full[6:17, 12:23], atol=1e-6)
