"""Generate golden vectors by running the OpenDDE reference modules on CPU.

Run in a container that has the reference source tree (it is NOT needed at test time):

    python tests/golden/make_golden.py --reference <path-to-OpenDDE-checkout>

The reference's Pairformer import chain needs two unrelated packages that are not
installed here; they are stubbed in ``sys.modules``:
  * ``optree`` (used only by ``opendde/model/utils.py:500`` chunk_layer._fetch_dims),
  * ``rdkit.Chem.GetPeriodicTable`` (used only for element tables,
    ``opendde/data/constants.py:390``).

Weights are re-initialised with ``opendde_b200.utils.seeded_init_`` (the reference's
default init zeroes every output projection). Inputs are regenerated from seeds at test
time; the fixture stores outputs plus checksums of inputs and weights so that a drift
in the generators is caught.
"""

from __future__ import annotations

import argparse
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from opendde_b200.utils import make_inputs, ragged_pair_mask, seeded_init_  # noqa: E402

# (name, kind, n, extra) -- kept small: fixtures are committed.
CASES = [
    ("trimul_out_n13", "trimul_out", 13, {}),
    ("trimul_in_n13", "trimul_in", 13, {}),
    ("triatt_start_n13", "triatt_start", 13, {}),
    ("triatt_end_n13", "triatt_end", 13, {}),
    ("transition_n13", "transition", 13, {}),
    ("apb_n13", "apb", 13, {}),
    ("block_n16", "block", 16, {}),
    ("block_n16_defaultln", "block_defaultln", 16, {}),
]


def _stub_imports():
    import torch.utils._pytree as pt
    optree = types.ModuleType("optree")
    optree.tree_map = lambda f, t, *a, **k: pt.tree_map(f, t)
    optree.tree_flatten = lambda t, *a, **k: pt.tree_flatten(t)
    sys.modules.setdefault("optree", optree)
    rdkit = types.ModuleType("rdkit")
    chem = types.ModuleType("rdkit.Chem")

    class _PeriodicTable:
        def GetElementSymbol(self, i):
            return f"E{i}"

    chem.GetPeriodicTable = lambda: _PeriodicTable()
    rdkit.Chem = chem
    sys.modules.setdefault("rdkit", rdkit)
    sys.modules.setdefault("rdkit.Chem", chem)


def case_mask(kind: str, n: int) -> torch.Tensor:
    # ragged holes + one fully masked row, so the uniform-average semantics are pinned
    return ragged_pair_mask(n, seed=7, drop=0.15, full_rows=[n - 1])


def checksum(t: torch.Tensor) -> np.ndarray:
    t = t.double()
    return np.array([t.sum().item(), t.abs().sum().item(), (t * t).sum().item()])


@torch.no_grad()
def run_case(kind: str, n: int):
    from opendde.model.modules.pairformer import PairformerBlock
    from opendde.model.modules.primitives import Transition
    from opendde.model.modules.transformer import AttentionPairBias
    from opendde.model.triangular.triangular import (
        TriangleAttention,
        TriangleMultiplicationIncoming,
        TriangleMultiplicationOutgoing,
    )

    torch.manual_seed(0)
    s, z, _ = make_inputs(n, c_z=128, c_s=384, seed=1)
    mask = case_mask(kind, n)
    perturb = kind != "block_defaultln"
    if kind in ("trimul_out", "trimul_in"):
        mod = (TriangleMultiplicationOutgoing if kind == "trimul_out" else TriangleMultiplicationIncoming)(c_z=128, c_hidden=128)
        params = seeded_init_(mod, seed=0, perturb_1d=perturb)
        out = {"out": mod(z, mask=mask)}
    elif kind in ("triatt_start", "triatt_end"):
        mod = TriangleAttention(c_in=128, c_hidden=32, no_heads=4, starting=(kind == "triatt_start"))
        params = seeded_init_(mod, seed=0, perturb_1d=perturb)
        out = {"out": mod(z, mask=mask)}
    elif kind == "transition":
        mod = Transition(c_in=128, n=4)
        params = seeded_init_(mod, seed=0, perturb_1d=perturb)
        out = {"out": mod(z)}
    elif kind == "apb":
        mod = AttentionPairBias(has_s=False, create_offset_ln_z=True, n_heads=16, c_a=384, c_z=128)
        params = seeded_init_(mod, seed=0, perturb_1d=perturb)
        out = {"out": mod(a=s, s=None, z=z)}
    elif kind.startswith("block"):
        mod = PairformerBlock(n_heads=16, c_z=128, c_s=384)
        params = seeded_init_(mod, seed=0, perturb_1d=perturb)
        s_out, z_out = mod(s, z, mask)
        out = {"s_out": s_out, "z_out": z_out}
    else:
        raise ValueError(kind)
    rec = {k: v.numpy().astype(np.float32) for k, v in out.items()}
    rec["chk_z"] = checksum(z)
    rec["chk_s"] = checksum(s)
    rec["chk_mask"] = checksum(mask)
    rec["chk_params"] = np.stack([checksum(params[k]) for k in sorted(params)])
    rec["param_names"] = np.array(sorted(params))
    return rec


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path to the OpenDDE source tree")
    args = ap.parse_args()
    sys.path.insert(0, os.path.abspath(args.reference))
    _stub_imports()
    torch.set_num_threads(min(8, os.cpu_count() or 1))
    for name, kind, n, _extra in CASES:
        rec = run_case(kind, n)
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, kind=np.array(kind), n=np.array(n), **rec)
        print("wrote", path, os.path.getsize(path))


if __name__ == "__main__":
    main()
