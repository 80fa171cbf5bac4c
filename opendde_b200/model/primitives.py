"""Transition (and the Linear wrappers it uses), drop-in for
``opendde.model.modules.primitives``. CUDA-backed, no CPU fallback."""

from __future__ import annotations

import math
from functools import partial
from typing import Optional

import torch
import torch.nn as nn

from .. import kernels
from .._abi import TransitionParams
from .triangular import LayerNorm


class Linear(nn.Linear):
    """primitives.Linear (primitives.py:24-90): zero bias, truncated-normal weights."""

    def __init__(self, in_features: int, out_features: int, bias: bool = True, device=None,
                 dtype=None, precision: Optional[torch.dtype] = None, initializer: str = "default"):
        self.use_bias = bias
        self.precision = precision
        self.initializer = initializer
        super().__init__(in_features, out_features, bias=bias, device=device, dtype=dtype)
        with torch.no_grad():
            if bias:
                nn.init.zeros_(self.bias)
            if initializer in ("default", "relu"):
                scale = 1.0 if initializer == "default" else 2.0
                std = math.sqrt(scale / max(1, in_features)) / 0.87962566103423978
                nn.init.trunc_normal_(self.weight, std=std, a=-2 * std, b=2 * std)
            elif initializer == "zeros":
                nn.init.zeros_(self.weight)
            else:
                raise ValueError(f"Invalid initializer: {initializer}.")


LinearNoBias = partial(Linear, bias=False)


class Transition(nn.Module):
    """Algorithm 11 in AF3 (primitives.py:158-217): LN -> SiLU(W_a y) * W_b y -> W_out."""

    def __init__(self, c_in: int, n: int) -> None:
        super().__init__()
        self.n = n
        self.c_in = c_in
        self.layernorm1 = LayerNorm(c_in)
        self.linear_no_bias_a = LinearNoBias(in_features=c_in, out_features=n * c_in, initializer="relu")
        self.linear_no_bias_b = LinearNoBias(in_features=c_in, out_features=n * c_in, initializer="relu")
        self.linear_no_bias = LinearNoBias(in_features=n * c_in, out_features=c_in, initializer="zeros")
        self._pack = None

    def weight_pack(self, dtype, device) -> kernels.WeightPack:
        spec = {
            "ln_w": self.layernorm1.weight, "ln_b": self.layernorm1.bias,
            "w_a": self.linear_no_bias_a.weight, "w_b": self.linear_no_bias_b.weight,
            "w_o": self.linear_no_bias.weight,
        }
        key = kernels.pack_key([p for p in spec.values() if p is not None], dtype, device)
        if self._pack is None or self._pack.key != key:
            self._pack = kernels.make_pack(TransitionParams, spec, {"ln_w", "ln_b"}, dtype, device, key)
        return self._pack

    def apply_(self, x: torch.Tensor, out: torch.Tensor, accumulate: bool) -> torch.Tensor:
        """out (+)= Transition(x) for tensors whose leading dims flatten to rows."""
        c = x.shape[-1]
        x2 = x.reshape(-1, c)
        o2 = out.view(-1, c)
        kernels.transition(self.weight_pack(x.dtype, x.device), x2, o2, self.n, accumulate)
        return out

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        kernels.require_cuda(x)
        x = x.contiguous()
        out = torch.empty_like(x)
        return self.apply_(x, out, accumulate=False)
