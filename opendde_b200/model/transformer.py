"""AttentionPairBias (single representation), drop-in for the ``has_s=False`` form of
``opendde.model.modules.transformer.AttentionPairBias`` used by PairformerBlock.
CUDA-backed, no CPU fallback."""

from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn

from .. import kernels
from .._abi import ApbParams
from .primitives import Linear, LinearNoBias
from .triangular import LayerNorm


class Attention(nn.Module):
    """primitives.Attention parameters (primitives.py:645-740): q with bias, k/v/o/g without."""

    def __init__(self, c_q: int, c_k: int, c_v: int, c_hidden: int, num_heads: int,
                 gating: bool = True, q_linear_bias: bool = True,
                 use_efficient_implementation: bool = True, zero_init: bool = True) -> None:
        super().__init__()
        self.c_q, self.c_k, self.c_v = c_q, c_k, c_v
        self.c_hidden = c_hidden
        self.num_heads = num_heads
        self.gating = gating
        self.use_efficient_implementation = use_efficient_implementation
        if q_linear_bias:
            self.linear_q = Linear(in_features=c_q, out_features=c_hidden * num_heads)
        else:
            self.linear_q = LinearNoBias(c_q, c_hidden * num_heads)
        self.linear_k = LinearNoBias(c_k, c_hidden * num_heads)
        self.linear_v = LinearNoBias(c_v, c_hidden * num_heads)
        self.linear_o = LinearNoBias(c_hidden * num_heads, c_q)
        self.linear_g = None
        if gating:
            self.linear_g = LinearNoBias(c_q, c_hidden * num_heads, initializer="zeros")
            self.sigmoid = nn.Sigmoid()
        self.zero_init = zero_init
        if zero_init:
            nn.init.zeros_(self.linear_o.weight)


class AttentionPairBias(nn.Module):
    """Algorithm 24 (transformer.py:39-671) for ``has_s=False`` (the Pairformer usage)."""

    def __init__(self, has_s: bool = True, create_offset_ln_z: bool = False, n_heads: int = 16,
                 c_a: int = 768, c_s: int = 384, c_z: int = 128, biasinit: float = -2.0,
                 cross_attention_mode: bool = False) -> None:
        super().__init__()
        assert c_a % n_heads == 0
        if has_s or cross_attention_mode:
            raise NotImplementedError(
                "opendde_b200 implements AttentionPairBias(has_s=False) as used by PairformerBlock")
        self.n_heads = n_heads
        self.has_s = has_s
        self.create_offset_ln_z = create_offset_ln_z
        self.cross_attention_mode = cross_attention_mode
        self.layernorm_a = LayerNorm(c_a)
        self.attention = Attention(c_q=c_a, c_k=c_a, c_v=c_a, c_hidden=c_a // n_heads,
                                   num_heads=n_heads, gating=True, q_linear_bias=True,
                                   zero_init=not has_s)
        self.layernorm_z = LayerNorm(c_z, create_offset=create_offset_ln_z)
        self.linear_nobias_z = LinearNoBias(in_features=c_z, out_features=n_heads)
        self._pack = None

    def weight_pack(self, dtype, device) -> kernels.WeightPack:
        att = self.attention
        spec = {
            "ln_a_w": self.layernorm_a.weight, "ln_a_b": self.layernorm_a.bias,
            "w_q": att.linear_q.weight, "b_q": att.linear_q.bias,
            "w_k": att.linear_k.weight, "w_v": att.linear_v.weight,
            "w_g": att.linear_g.weight, "w_o": att.linear_o.weight,
            "ln_z_w": self.layernorm_z.weight, "ln_z_b": self.layernorm_z.bias,
            "w_z": self.linear_nobias_z.weight,
        }
        key = kernels.pack_key([p for p in spec.values() if p is not None], dtype, device)
        if self._pack is None or self._pack.key != key:
            self._pack = kernels.make_pack(ApbParams, spec, {"ln_a_w", "ln_a_b", "b_q", "ln_z_w", "ln_z_b"},
                                           dtype, device, key)
        return self._pack

    def pair_bias(self, z: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """[H, R, C] fp32 pair bias of a (tile of the) pair tensor."""
        n_r, n_c = z.shape[0], z.shape[1]
        if out is None:
            out = torch.empty((self.n_heads, n_r, n_c), device=z.device, dtype=torch.float32)
        kernels.apb_pair_bias(self.weight_pack(z.dtype, z.device), z, self.n_heads, out)
        return out

    def apply_(self, s: torch.Tensor, z: Optional[torch.Tensor], out: torch.Tensor,
               accumulate: bool, bias: Optional[torch.Tensor] = None) -> torch.Tensor:
        kernels.apb(self.weight_pack(s.dtype, s.device), s, out, z, bias, self.n_heads, accumulate)
        return out

    def forward(self, a: torch.Tensor, s: Optional[torch.Tensor], z: torch.Tensor,
                n_queries: Optional[int] = None, n_keys: Optional[int] = None,
                inplace_safe: bool = False, chunk_size: Optional[int] = None,
                enable_efficient_fusion: bool = False,
                extra_attn_bias: Optional[torch.Tensor] = None) -> torch.Tensor:
        if n_queries or n_keys:
            raise NotImplementedError("local (windowed) attention is not part of the pair stack")
        kernels.require_cuda(a, z, extra_attn_bias)
        a = a.contiguous()
        z = z.contiguous()
        bias = None
        if extra_attn_bias is not None:
            bias = self.pair_bias(z)
            e = extra_attn_bias.to(device=bias.device, dtype=torch.float32)
            bias = (bias + (e if e.dim() == 3 else e[None])).contiguous()
        out = torch.empty_like(a)
        return self.apply_(a, z if bias is None else None, out, accumulate=False, bias=bias)
