"""Triangle multiplicative update and triangle attention, drop-in for
``opendde.model.triangular.triangular`` / ``opendde.model.triangular.layers``.

Class names, constructor arguments, parameter names (so reference checkpoints load) and
forward signatures follow the reference; the forward bodies call the CUDA kernels behind
``libpairformer_b200.so``. There is no CPU fallback and no cuEquivariance/Triton dispatch:
``"torch"`` and ``"cuequivariance"`` both route to the CUDA kernels, anything else raises
the reference's ValueError.
"""

from __future__ import annotations

import math
from functools import partialmethod
from typing import Optional

import torch
import torch.nn as nn

from .. import kernels
from .._abi import TriattParams, TrimulParams

_TRIMUL_CHOICES = {"torch", "cuequivariance"}
_TRIATT_CHOICES = {"torch", "cuequivariance"}


def _trunc_normal_fan_in_(w: torch.Tensor, scale: float = 1.0) -> None:
    # LeCun/He truncated normal on [-2, 2] std-units (layers.py:56-73); 0.87962566 is the std
    # of a unit normal truncated to [-2, 2].
    fan_in = max(1, w.shape[1])
    std = math.sqrt(scale / fan_in) / 0.87962566103423978
    with torch.no_grad():
        nn.init.trunc_normal_(w, mean=0.0, std=std, a=-2 * std, b=2 * std)


class OpenfoldLinear(nn.Linear):
    """Linear with the reference initialisers (opendde/model/triangular/layers.py:128-223)."""

    def __init__(self, in_dim: int, out_dim: int, bias: bool = True, init: str = "default",
                 init_fn=None, precision: Optional[torch.dtype] = None):
        super().__init__(in_dim, out_dim, bias=bias)
        if bias:
            with torch.no_grad():
                self.bias.fill_(0)
        with torch.no_grad():
            if init_fn is not None:
                init_fn(self.weight, self.bias)
            elif init == "default":
                _trunc_normal_fan_in_(self.weight, 1.0)
            elif init == "relu":
                _trunc_normal_fan_in_(self.weight, 2.0)
            elif init == "glorot":
                nn.init.xavier_uniform_(self.weight, gain=1)
            elif init == "gating":
                self.weight.fill_(0.0)
                if bias:
                    self.bias.fill_(1.0)
            elif init == "normal":
                nn.init.kaiming_normal_(self.weight, nonlinearity="linear")
            elif init == "final":
                self.weight.fill_(0.0)
            else:
                raise ValueError("Invalid init string.")
        self.precision = precision


class LayerNorm(nn.Module):
    """OpenFoldLayerNorm (layers.py:226-269): eps 1e-5, ``weight``/``bias`` parameters.

    ``forward`` runs the CUDA LayerNorm kernel; inside the fused ops the same parameters
    are applied in the producing kernel's prologue.
    """

    def __init__(self, c_in: int, create_scale: bool = True, create_offset: bool = True,
                 eps: float = 1e-5):
        super().__init__()
        self.c_in = (c_in,)
        self.create_scale = create_scale
        self.create_offset = create_offset
        self.eps = eps
        if create_scale:
            self.weight = nn.Parameter(torch.ones(c_in))
        else:
            self.register_parameter("weight", None)
        if create_offset:
            self.bias = nn.Parameter(torch.zeros(c_in))
        else:
            self.register_parameter("bias", None)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return kernels.layernorm(x, self.weight, self.bias, self.eps)


class Attention(nn.Module):
    """Gated multi-head attention parameters (layers.py:325-385): linear_{q,k,v,o,g}.

    In this package the attention arithmetic runs inside the triangle-attention kernels;
    the module holds the parameters with the reference's names and initialisers.
    """

    def __init__(self, c_q: int, c_k: int, c_v: int, c_hidden: int, no_heads: int,
                 gating: bool = True):
        super().__init__()
        self.c_q, self.c_k, self.c_v = c_q, c_k, c_v
        self.c_hidden = c_hidden
        self.no_heads = no_heads
        self.gating = gating
        self.linear_q = OpenfoldLinear(c_q, c_hidden * no_heads, bias=False)
        self.linear_k = OpenfoldLinear(c_k, c_hidden * no_heads, bias=False)
        self.linear_v = OpenfoldLinear(c_v, c_hidden * no_heads, bias=False)
        self.linear_o = OpenfoldLinear(c_hidden * no_heads, c_q, bias=False, init="final")
        self.linear_g = None
        if gating:
            self.linear_g = OpenfoldLinear(c_q, c_hidden * no_heads, bias=False, init="gating")
        self.sigmoid = nn.Sigmoid()


def _batched(fn, *tensors):
    """Apply ``fn`` over leading batch dims of [*, N, N, C] / [*, N, N] tensors."""
    lead = tensors[0].dim() - 3
    if lead == 0:
        return fn(*tensors)
    outs = []
    flat = [None if t is None else t.reshape((-1,) + tuple(t.shape[lead:])) for t in tensors]
    for b in range(flat[0].shape[0]):
        outs.append(fn(*[None if t is None else t[b] for t in flat]))
    return torch.stack(outs).reshape(tensors[0].shape[:lead] + outs[0].shape)


class TriangleMultiplicativeUpdate(nn.Module):
    """Algorithms 11/12 (triangular.py:159-567), CUDA-backed."""

    def __init__(self, c_z: int, c_hidden: int, _outgoing: bool = True) -> None:
        super().__init__()
        self.c_z = c_z
        self.c_hidden = c_hidden
        self._outgoing = _outgoing
        self.linear_g = OpenfoldLinear(c_z, c_z, bias=False, init="gating")
        self.linear_z = OpenfoldLinear(c_hidden, c_z, bias=False, init="final")
        self.layer_norm_in = LayerNorm(c_z)
        self.layer_norm_out = LayerNorm(c_hidden)
        self.sigmoid = nn.Sigmoid()
        self.linear_a_p = OpenfoldLinear(c_z, c_hidden, bias=False)
        self.linear_a_g = OpenfoldLinear(c_z, c_hidden, bias=False, init="gating")
        self.linear_b_p = OpenfoldLinear(c_z, c_hidden, bias=False)
        self.linear_b_g = OpenfoldLinear(c_z, c_hidden, bias=False, init="gating")
        self._pack = None

    def weight_pack(self, dtype, device) -> kernels.WeightPack:
        spec = {
            "ln_in_w": self.layer_norm_in.weight, "ln_in_b": self.layer_norm_in.bias,
            "w_ap": self.linear_a_p.weight, "w_ag": self.linear_a_g.weight,
            "w_bp": self.linear_b_p.weight, "w_bg": self.linear_b_g.weight,
            "ln_out_w": self.layer_norm_out.weight, "ln_out_b": self.layer_norm_out.bias,
            "w_z": self.linear_z.weight, "w_g": self.linear_g.weight,
        }
        key = kernels.pack_key([p for p in spec.values() if p is not None], dtype, device)
        if self._pack is None or self._pack.key != key:
            self._pack = kernels.make_pack(TrimulParams, spec, {"ln_in_w", "ln_in_b", "ln_out_w", "ln_out_b"},
                                           dtype, device, key)
        return self._pack

    def apply_(self, z: torch.Tensor, mask: Optional[torch.Tensor], out: torch.Tensor,
               accumulate: bool) -> torch.Tensor:
        """out (+)= update(z) for a single [N, N, C] pair tensor; ``out`` may be ``z``."""
        n = z.shape[0]
        m = kernels.prepare_mask(mask, n, n, z.device)
        pack = self.weight_pack(z.dtype, z.device)
        if self._outgoing:
            za, zb, ma, mb = z, z, m, m
        else:
            za, zb, ma, mb = z.transpose(0, 1), z.transpose(0, 1), m.t(), m.t()
        kernels.trimul(pack, za, zb, ma, mb, z, out, self.c_hidden, accumulate)
        return out

    def forward(self, z: torch.Tensor, mask: Optional[torch.Tensor] = None,
                inplace_safe: bool = False, _add_with_inplace: bool = False,
                _inplace_chunk_size: Optional[int] = 256,
                triangle_multiplicative: str = "torch") -> torch.Tensor:
        if triangle_multiplicative not in _TRIMUL_CHOICES:
            raise ValueError(
                "triangle_multiplicative must be 'cuequivariance' or 'torch', "
                f"but got {triangle_multiplicative}")
        kernels.require_cuda(z, mask)
        if inplace_safe and _add_with_inplace:
            if z.dim() == 3 and z.is_contiguous():
                return self.apply_(z, mask, z, accumulate=True)
            return z.copy_(_batched(lambda zz, mm: self.apply_(zz.contiguous(), mm, zz.contiguous().clone(), True), z, mask))

        def one(zz, mm):
            zz = zz.contiguous()
            out = torch.empty_like(zz)
            return self.apply_(zz, mm, out, accumulate=False)

        return _batched(one, z, mask)


class TriangleMultiplicationOutgoing(TriangleMultiplicativeUpdate):
    """Algorithm 11 (triangular.py:570-575)."""

    __init__ = partialmethod(TriangleMultiplicativeUpdate.__init__, _outgoing=True)


class TriangleMultiplicationIncoming(TriangleMultiplicativeUpdate):
    """Algorithm 12 (triangular.py:578-583)."""

    __init__ = partialmethod(TriangleMultiplicativeUpdate.__init__, _outgoing=False)


class TriangleAttention(nn.Module):
    """Triangle attention (triangular.py:586-706), CUDA-backed. Returns the update."""

    def __init__(self, c_in: int, c_hidden: int, no_heads: int, starting: bool = True,
                 inf: float = 1e9) -> None:
        super().__init__()
        self.c_in = c_in
        self.c_hidden = c_hidden
        self.no_heads = no_heads
        self.starting = starting
        self.inf = inf
        self.layer_norm = LayerNorm(c_in)
        self.linear = OpenfoldLinear(c_in, no_heads, bias=False)
        self.mha = Attention(c_in, c_in, c_in, c_hidden, no_heads)
        self._pack = None

    def weight_pack(self, dtype, device) -> kernels.WeightPack:
        spec = {
            "ln_w": self.layer_norm.weight, "ln_b": self.layer_norm.bias,
            "w_bias": self.linear.weight,
            "w_q": self.mha.linear_q.weight, "w_k": self.mha.linear_k.weight,
            "w_v": self.mha.linear_v.weight, "w_g": self.mha.linear_g.weight,
            "w_o": self.mha.linear_o.weight,
        }
        key = kernels.pack_key([p for p in spec.values() if p is not None], dtype, device)
        if self._pack is None or self._pack.key != key:
            self._pack = kernels.make_pack(TriattParams, spec, {"ln_w", "ln_b"}, dtype, device, key)
        return self._pack

    def apply_(self, z: torch.Tensor, mask: Optional[torch.Tensor], out: torch.Tensor,
               accumulate: bool, starting: Optional[bool] = None) -> torch.Tensor:
        """out (+)= update(z) for one [N, N, C] tensor; the ending node uses transposed views."""
        starting = self.starting if starting is None else starting
        n = z.shape[0]
        m = kernels.prepare_mask(mask, n, n, z.device)
        pack = self.weight_pack(z.dtype, z.device)
        if starting:
            zs, ms, zo = z, m, out
        else:
            zs, ms, zo = z.transpose(0, 1), m.t(), out.transpose(0, 1)
        kernels.triatt(pack, zs, ms, zo, self.no_heads, self.c_hidden, self.inf, accumulate)
        return out

    def forward(self, x: torch.Tensor, mask: Optional[torch.Tensor] = None,
                chunk_size: Optional[int] = None, triangle_attention: str = "torch",
                inplace_safe: bool = False) -> torch.Tensor:
        if triangle_attention not in _TRIATT_CHOICES:
            raise ValueError("Invalid triangle_attention. Options: 'cuequivariance', 'torch'.")
        kernels.require_cuda(x, mask)

        def one(zz, mm):
            zz = zz.contiguous()
            out = torch.empty_like(zz)
            return self.apply_(zz, mm, out, accumulate=False)

        return _batched(one, x, mask)
