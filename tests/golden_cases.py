"""Shared helpers: rebuild the inputs/weights of a golden fixture from its seeds."""
import os

import numpy as np
import torch

from opendde_b200.utils import make_inputs, ragged_pair_mask, seeded_params

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
CASE_FILES = sorted(f for f in os.listdir(GOLDEN_DIR) if f.endswith(".npz"))


def checksum(t: torch.Tensor) -> np.ndarray:
    t = t.double()
    return np.array([t.sum().item(), t.abs().sum().item(), (t * t).sum().item()])


def module_for(kind: str):
    """A parameter-shape template with the reference's parameter names (this package's mirror)."""
    from opendde_b200.model import (AttentionPairBias, PairformerBlock, TriangleAttention,
                                    TriangleMultiplicationIncoming, TriangleMultiplicationOutgoing,
                                    Transition)
    if kind == "trimul_out":
        return TriangleMultiplicationOutgoing(c_z=128, c_hidden=128)
    if kind == "trimul_in":
        return TriangleMultiplicationIncoming(c_z=128, c_hidden=128)
    if kind in ("triatt_start", "triatt_end"):
        return TriangleAttention(c_in=128, c_hidden=32, no_heads=4, starting=(kind == "triatt_start"))
    if kind == "transition":
        return Transition(c_in=128, n=4)
    if kind == "apb":
        return AttentionPairBias(has_s=False, create_offset_ln_z=True, n_heads=16, c_a=384, c_z=128)
    if kind.startswith("block"):
        return PairformerBlock(n_heads=16, c_z=128, c_s=384)
    raise ValueError(kind)


def load_case(fname: str):
    rec = dict(np.load(os.path.join(GOLDEN_DIR, fname)))
    kind = str(rec["kind"])
    n = int(rec["n"])
    s, z, _ = make_inputs(n, c_z=128, c_s=384, seed=1)
    mask = ragged_pair_mask(n, seed=7, drop=0.15, full_rows=[n - 1])
    mod = module_for(kind)
    params = seeded_params([(k, tuple(p.shape)) for k, p in mod.named_parameters()], seed=0,
                           perturb_1d=(kind != "block_defaultln"))
    return kind, n, s, z, mask, params, rec, mod
