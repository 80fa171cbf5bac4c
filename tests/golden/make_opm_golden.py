"""Generate the OuterProductMean golden vectors by running the OpenDDE reference module on CPU.

Run in a container that has the reference source tree (it is NOT needed at test time):

    python tests/golden/make_opm_golden.py --reference <path-to-OpenDDE-checkout>

The reference's import chain is stubbed exactly as in make_golden.py (``optree``, ``rdkit``).
Weights are re-initialised with ``opendde_b200.utils.seeded_init_`` (the reference's
``init="final"`` zeroes linear_out). Inputs are regenerated from seeds at test time
(``opm_inputs`` below, imported by the tests); the fixture stores the output plus checksums of
the inputs and weights.
"""

from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
sys.path.insert(0, HERE)

from opendde_b200.utils import seeded_init_  # noqa: E402

# (name, n_seq, n_res, c_m, c_hidden, c_z, masked)
CASES = [
    ("opm_s7_n13_masked", 7, 13, 64, 32, 128, True),
    ("opm_s5_n11_nomask", 5, 11, 16, 8, 24, False),
]


def opm_inputs(n_seq: int, n_res: int, c_m: int, masked: bool):
    """m ~ N(0, 1) [S, N, c_m]; MSA mask with random holes, one fully masked sequence and one
    fully masked residue column (None when ``masked`` is False)."""
    g = torch.Generator().manual_seed(11)
    m = torch.randn((n_seq, n_res, c_m), generator=g)
    if not masked:
        return m, None
    mask = (torch.rand((n_seq, n_res), generator=g) >= 0.2).float()
    mask[n_seq - 1, :] = 0.0
    mask[:, 2] = 0.0
    return m, mask


def checksum(t: torch.Tensor) -> np.ndarray:
    t = t.double()
    return np.array([t.sum().item(), t.abs().sum().item(), (t * t).sum().item()])


@torch.no_grad()
def run_case(n_seq, n_res, c_m, c_hidden, c_z, masked):
    from opendde.model.triangular.layers import OuterProductMean
    mod = OuterProductMean(c_m=c_m, c_z=c_z, c_hidden=c_hidden)
    params = seeded_init_(mod, seed=0, perturb_1d=True)
    m, mask = opm_inputs(n_seq, n_res, c_m, masked)
    out = mod(m, mask=mask)
    rec = {"out": out.numpy().astype(np.float32), "chk_m": checksum(m),
           "chk_params": np.stack([checksum(params[k]) for k in sorted(params)]),
           "param_names": np.array(sorted(params))}
    if mask is not None:
        rec["chk_mask"] = checksum(mask)
    return rec


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path to the OpenDDE source tree")
    args = ap.parse_args()
    sys.path.insert(0, os.path.abspath(args.reference))
    from make_golden import _stub_imports
    _stub_imports()
    for name, n_seq, n_res, c_m, c_hidden, c_z, masked in CASES:
        rec = run_case(n_seq, n_res, c_m, c_hidden, c_z, masked)
        path = os.path.join(HERE, "opm", f"{name}.npz")
        np.savez_compressed(path, n_seq=np.array(n_seq), n_res=np.array(n_res), c_m=np.array(c_m),
                            c_hidden=np.array(c_hidden), c_z=np.array(c_z), masked=np.array(masked), **rec)
        print("wrote", path, os.path.getsize(path))


if __name__ == "__main__":
    main()
