"""Seeded weight initialisation and synthetic inputs for the Pairformer pair stack.

The reference zero-initialises every output projection and gate
(opendde/model/triangular/layers.py:188-197 "gating"/"final", primitives.py:178-180
"zeros", primitives.py:718-721), which makes an untouched block the identity on ``z``.
Parity runs and benchmarks therefore re-initialise every weight here:

* every 2-D weight ~ N(0, 1/fan_in) (plain normal, "LeCun normal" without truncation);
* LayerNorm scale 1 and offset 0, and 1-D linear biases 0 — unless ``perturb_1d`` is set,
  in which case they get small seeded perturbations so that tests exercise them;
* parameters are drawn in sorted-name order from one CPU ``torch.Generator``, so the
  same seed gives the same values for the reference module and for this package's
  mirror classes (their parameter names are identical).
"""

from __future__ import annotations

import math
from typing import Dict, Iterable, Optional, Tuple

import torch


def seeded_params(named_shapes: Iterable[Tuple[str, Tuple[int, ...]]], seed: int = 0,
                  perturb_1d: bool = False) -> Dict[str, torch.Tensor]:
    """Generate fp32 CPU tensors for ``(name, shape)`` pairs, in sorted-name order."""
    g = torch.Generator().manual_seed(seed)
    out: Dict[str, torch.Tensor] = {}
    for name, shape in sorted(named_shapes, key=lambda t: t[0]):
        if len(shape) == 2:
            fan_in = shape[1]
            t = torch.randn(shape, generator=g, dtype=torch.float32) / math.sqrt(fan_in)
        elif len(shape) == 1:
            is_scale = name.endswith("weight")
            if perturb_1d:
                t = torch.randn(shape, generator=g, dtype=torch.float32) * 0.1
                if is_scale:
                    t = t + 1.0
            else:
                t = torch.ones(shape) if is_scale else torch.zeros(shape)
        else:
            raise ValueError(f"unexpected parameter rank for {name}: {shape}")
        out[name] = t
    return out


@torch.no_grad()
def seeded_init_(module: torch.nn.Module, seed: int = 0, perturb_1d: bool = False) -> Dict[str, torch.Tensor]:
    """Overwrite every parameter of ``module`` with :func:`seeded_params` values.

    Returns the generated fp32 CPU dict (keys = ``module.state_dict()`` names).
    """
    named = [(n, tuple(p.shape)) for n, p in module.named_parameters()]
    vals = seeded_params(named, seed=seed, perturb_1d=perturb_1d)
    for n, p in module.named_parameters():
        p.copy_(vals[n].to(device=p.device, dtype=p.dtype))
    return vals


def token_mask(n: int, pad_frac: float = 0.0) -> torch.Tensor:
    """Token mask with the last ceil(pad_frac * n) tokens set to 0 (config C1: 0.1, C4: 0.07)."""
    m = torch.ones(n)
    n_pad = int(math.ceil(pad_frac * n)) if pad_frac > 0 else 0
    if n_pad:
        m[n - n_pad:] = 0.0
    return m


def pair_mask_from_tokens(m: torch.Tensor) -> torch.Tensor:
    """pair_mask = m (outer) m."""
    return m[:, None] * m[None, :]


def make_inputs(n: int, c_z: int = 128, c_s: int = 384, seed: int = 1,
                pad_frac: float = 0.0, with_s: bool = True):
    """z ~ N(0,1) [n, n, c_z], then s ~ N(0,1) [n, c_s] from one generator; pair mask."""
    g = torch.Generator().manual_seed(seed)
    z = torch.randn((n, n, c_z), generator=g, dtype=torch.float32)
    s = torch.randn((n, c_s), generator=g, dtype=torch.float32) if with_s else None
    mask = pair_mask_from_tokens(token_mask(n, pad_frac))
    return s, z, mask


def ragged_pair_mask(n: int, seed: int = 7, drop: float = 0.1, full_rows: Optional[Iterable[int]] = None) -> torch.Tensor:
    """Pair mask with random holes and (optionally) fully masked rows, for edge-case tests."""
    g = torch.Generator().manual_seed(seed)
    m = (torch.rand((n, n), generator=g) >= drop).float()
    for r in (full_rows or ()):
        m[r, :] = 0.0
    return m
