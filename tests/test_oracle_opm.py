"""The OuterProductMean restatement in the oracle against the reference's own outputs
(tests/golden/opm/*.npz, made by tests/golden/make_opm_golden.py from the reference module),
including a fully masked sequence, a fully masked residue column and the mask-free path; and
the tile restriction the Fold-CP tile update uses (rows / cols) against the full output."""
import glob
import os
import sys

import numpy as np
import pytest
import torch

from oracle import pairformer_oracle as O
from opendde_b200.utils import seeded_params

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
from make_opm_golden import checksum, opm_inputs  # noqa: E402

FILES = sorted(glob.glob(os.path.join(HERE, "golden", "opm", "*.npz")))


def opm_param_shapes(c_m, c_hidden, c_z):
    return [("layer_norm.weight", (c_m,)), ("layer_norm.bias", (c_m,)), ("linear_1.weight", (c_hidden, c_m)),
            ("linear_2.weight", (c_hidden, c_m)), ("linear_out.weight", (c_z, c_hidden * c_hidden)),
            ("linear_out.bias", (c_z,))]


def load(path):
    rec = dict(np.load(path))
    n_seq, n_res, c_m, c_h, c_z = (int(rec[k]) for k in ("n_seq", "n_res", "c_m", "c_hidden", "c_z"))
    m, mask = opm_inputs(n_seq, n_res, c_m, bool(rec["masked"]))
    params = seeded_params(opm_param_shapes(c_m, c_h, c_z), seed=0, perturb_1d=True)
    return rec, m, mask, params


@pytest.mark.parametrize("path", FILES, ids=[os.path.basename(f) for f in FILES])
def test_oracle_opm_matches_reference(path):
    rec, m, mask, params = load(path)
    assert np.allclose(checksum(m), rec["chk_m"], rtol=1e-10, atol=1e-8)
    if mask is not None:
        assert np.allclose(checksum(mask), rec["chk_mask"])
    assert list(rec["param_names"]) == sorted(params)
    assert np.allclose(np.stack([checksum(params[k]) for k in sorted(params)]), rec["chk_params"], rtol=1e-10)
    out = O.outer_product_mean(m, mask, params)
    err = (out - torch.from_numpy(rec["out"])).abs().max().item()
    assert err <= 2e-5, err


def test_oracle_opm_tile_is_a_slice_of_the_full_output():
    rec, m, mask, params = load(FILES[0])
    full = O.outer_product_mean(m, mask, params)
    tile = O.outer_product_mean(m, mask, params, rows=slice(3, 9), cols=slice(5, 13))
    assert torch.allclose(tile, full[3:9, 5:13], atol=1e-6)
