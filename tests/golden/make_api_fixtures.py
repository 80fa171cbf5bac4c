"""Parameter names and shapes of the reference's Pairformer modules in every configuration
its callers instantiate (the trunk, the MSA module's pair stack, the template embedder, the
confidence head, the structural refiner), written to ``tests/golden/api_shapes.json``.

Run in a container that has the reference source tree (not needed at test time):

    python tests/golden/make_api_fixtures.py --reference <path-to-OpenDDE-checkout>

Configurations (constructor keyword arguments), following the call sites:
  trunk             PairformerStack(**configs.model.pairformer)       opendde.py:130
  msa_pair_stack    PairformerBlock(c_z, c_s=0, hidden_scale_up)        pairformer.py:804
  template          PairformerStack(c_s=0, c_z=c, n_blocks, num_intermediate_factor,
                                    hidden_scale_up)                    pairformer.py:1678
  confidence        PairformerStack(c_z, c_s, n_blocks, hidden_scale_up)  confidence.py:98
  refiner           PairformerStack(n_blocks, n_heads, c_z, c_s, num_intermediate_factor,
                                    hidden_scale_up)                    opendde.py:208
"""

from __future__ import annotations

import argparse
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "api_shapes.json")

CONFIGS = {
    "trunk_block": ("PairformerBlock", dict(n_heads=16, c_z=128, c_s=384)),
    "msa_pair_stack": ("PairformerBlock", dict(c_z=128, c_s=0, hidden_scale_up=False)),
    "msa_pair_stack_scaled": ("PairformerBlock", dict(c_z=128, c_s=0, hidden_scale_up=True)),
    "template_stack": ("PairformerStack", dict(c_s=0, c_z=64, n_blocks=2, num_intermediate_factor=2,
                                              hidden_scale_up=False)),
    "confidence_stack": ("PairformerStack", dict(c_z=128, c_s=384, n_blocks=2, hidden_scale_up=False)),
    "refiner_stack_scaled": ("PairformerStack", dict(n_blocks=2, n_heads=16, c_z=384, c_s=384,
                                                    num_intermediate_factor=2, hidden_scale_up=True)),
}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    sys.path.insert(0, HERE)
    from make_golden import _stub_imports
    _stub_imports()
    from opendde.model.modules import pairformer as P
    out = {}
    for name, (cls, kw) in CONFIGS.items():
        mod = getattr(P, cls)(**kw)
        out[name] = {"class": cls, "kwargs": kw,
                     "params": {k: list(v.shape) for k, v in mod.state_dict().items()}}
    with open(OUT, "w") as f:
        json.dump(out, f, indent=1, sort_keys=True)
    print("wrote", OUT, {k: len(v["params"]) for k, v in out.items()})


if __name__ == "__main__":
    main()
