"""Golden vectors for the reference's closed-form Fold-CP mini-oracles (no projections).

Run in a container that has the reference source tree (it is NOT needed at test time):

    python tests/golden/make_mini_golden.py --reference <path-to-OpenDDE-checkout>

Runs ``serial_triangle_multiplication`` (opendde/distributed/foldcp/triangular_mult.py:278-288),
``serial_triangle_attention_starting`` / ``_ending`` (triangle_attention.py:111-119) and
``online_softmax_update`` (online_softmax.py:10-33) of the reference on seeded inputs and
stores the outputs in ``tests/golden/mini/mini_n7.npz``. The inputs are regenerated from the
same seeds at test time (``mini_inputs``); their checksums are stored to catch generator drift.
"""

from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "mini", "mini_n7.npz")
SPLITS = ((0, 3), (3, 7), (7, 9))   # key blocks merged by the online softmax


def mini_inputs():
    """Seeded inputs of every mini-oracle case (fp64 for tight comparisons)."""
    g = torch.Generator().manual_seed(11)
    a = torch.randn((2, 7, 7, 3), generator=g, dtype=torch.float64)
    b = torch.randn((2, 7, 7, 3), generator=g, dtype=torch.float64)
    z = 0.5 * torch.randn((2, 6, 6, 4), generator=g, dtype=torch.float64)
    q = torch.randn((3, 5, 4), generator=g, dtype=torch.float64)
    k = torch.randn((3, 9, 4), generator=g, dtype=torch.float64)
    v = torch.randn((3, 9, 4), generator=g, dtype=torch.float64)
    return a, b, z, q, k, v


def block_state(q, k, v, lo, hi):
    """One key block's (softmax-weighted output, lse, amax) in the form the merge expects."""
    logits = q @ k[:, lo:hi].transpose(-1, -2)
    amax = logits.amax(-1)
    e = torch.exp(logits - amax[..., None])
    lse = torch.log(e.sum(-1))
    return (e / e.sum(-1, keepdim=True)) @ v[:, lo:hi], lse, amax


def checksum(t: torch.Tensor) -> np.ndarray:
    t = t.double()
    return np.array([t.sum().item(), t.abs().sum().item(), (t * t).sum().item()])


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    sys.path.insert(0, HERE)
    from make_golden import _stub_imports   # the same two sys.modules stubs (optree, rdkit)
    _stub_imports()
    from opendde.distributed.foldcp.online_softmax import online_softmax_update
    from opendde.distributed.foldcp.triangle_attention import (serial_triangle_attention_ending,
                                                               serial_triangle_attention_starting)
    from opendde.distributed.foldcp.triangular_mult import serial_triangle_multiplication

    a, b, z, q, k, v = mini_inputs()
    rec = {
        "tm_out": serial_triangle_multiplication(a, b, "outgoing").numpy(),
        "tm_in": serial_triangle_multiplication(a, b, "incoming").numpy(),
        "ta_start": serial_triangle_attention_starting(z).numpy(),
        "ta_end": serial_triangle_attention_ending(z).numpy(),
    }
    out = lse = amax = None
    for lo, hi in SPLITS:
        out, lse, amax = online_softmax_update(*block_state(q, k, v, lo, hi), out, lse, amax)
    rec.update(os_out=out.numpy(), os_lse=lse.numpy(), os_amax=amax.numpy())
    for name, t in zip("abzqkv", (a, b, z, q, k, v)):
        rec[f"chk_{name}"] = checksum(t)
    os.makedirs(os.path.dirname(OUT), exist_ok=True)
    np.savez_compressed(OUT, **rec)
    print("wrote", OUT)


if __name__ == "__main__":
    main()
