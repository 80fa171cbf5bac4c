"""PairformerBlock / PairformerStack, drop-in for ``opendde.model.modules.pairformer``.

The block keeps the reference's residual order (pairformer.py:228-272): tri_mul_out,
tri_mul_in, tri_att_start, tri_att_end (on the transposed pair, mask transposed),
pair_transition, then (c_s > 0) s += AttentionPairBias(s, z); s += single Transition(s).
Every pair update is fused with its residual add and written in place into one working
copy of ``z``; the ending-node attention reads and writes transposed *views* (no physical
transposes, unlike the reference's two ``.transpose().contiguous()`` copies).

Each forward ends with a status checkpoint: if a device-side bounded wait of an earlier launch
timed out (its outputs are invalid), the forward raises ``PFError`` (``PF_ETIMEOUT``) instead of
returning; the check reads a copy of the device status word made without synchronising, so it
reports the timeout at most one forward late.
"""

from __future__ import annotations

import os
from typing import Optional

import torch
import torch.distributed as dist
import torch.nn as nn

from .. import _abi, kernels
from .primitives import Transition
from .transformer import AttentionPairBias
from .triangular import (
    TriangleAttention,
    TriangleMultiplicationIncoming,
    TriangleMultiplicationOutgoing,
)

_CHOICES = {"torch", "cuequivariance"}


def _check_choices(tm: str, ta: str) -> None:
    if tm not in _CHOICES:
        raise ValueError(f"triangle_multiplicative must be 'cuequivariance' or 'torch', but got {tm}")
    if ta not in _CHOICES:
        raise ValueError("Invalid triangle_attention. Options: 'cuequivariance', 'torch'.")


class PairformerBlock(nn.Module):
    """Algorithm 17 lines 2-8 (pairformer.py:59-273)."""

    def __init__(self, n_heads: int = 16, c_z: int = 128, c_s: int = 384, c_hidden_mul: int = 128,
                 c_hidden_pair_att: int = 32, no_heads_pair: int = 4,
                 num_intermediate_factor: int = 4, hidden_scale_up: bool = False) -> None:
        super().__init__()
        self.n_heads = n_heads
        if hidden_scale_up:
            no_heads_pair = c_z // c_hidden_pair_att
            c_hidden_mul = c_z
        self.tri_mul_out = TriangleMultiplicationOutgoing(c_z=c_z, c_hidden=c_hidden_mul)
        self.tri_mul_in = TriangleMultiplicationIncoming(c_z=c_z, c_hidden=c_hidden_mul)
        self.tri_att_start = TriangleAttention(c_in=c_z, c_hidden=c_hidden_pair_att, no_heads=no_heads_pair)
        self.tri_att_end = TriangleAttention(c_in=c_z, c_hidden=c_hidden_pair_att, no_heads=no_heads_pair)
        self.pair_transition = Transition(c_in=c_z, n=num_intermediate_factor)
        self.c_s = c_s
        if c_s > 0:
            self.attention_pair_bias = AttentionPairBias(has_s=False, create_offset_ln_z=True,
                                                         n_heads=n_heads, c_a=c_s, c_z=c_z)
            self.single_transition = Transition(c_in=c_s, n=4)

    # -- fused in-place pair updates on one [N, N, C] working tensor
    def pair_updates_(self, z: torch.Tensor, mask: torch.Tensor) -> torch.Tensor:
        self.tri_mul_out.apply_(z, mask, z, accumulate=True)
        self.tri_mul_in.apply_(z, mask, z, accumulate=True)
        self.tri_att_start.apply_(z, mask, z, accumulate=True, starting=True)
        self.tri_att_end.apply_(z, mask, z, accumulate=True, starting=False)
        self.pair_transition.apply_(z, z, accumulate=True)
        return z

    def single_updates(self, s: torch.Tensor, z: Optional[torch.Tensor],
                       bias: Optional[torch.Tensor] = None) -> torch.Tensor:
        s_new = s.contiguous().clone()
        self.attention_pair_bias.apply_(s.contiguous(), z, s_new, accumulate=True, bias=bias)
        self.single_transition.apply_(s_new, s_new, accumulate=True)
        return s_new

    def _maybe_forward_foldcp_pair_only(self, s, z, pair_mask, chunk_size=None):
        if os.environ.get("OPENDDE_FOLDCP_MODE", "single") != "distributed":
            return None
        if self.c_s != 0 or s is not None:
            return None
        if not dist.is_available() or not dist.is_initialized():
            return None
        from ..distributed.foldcp import runtime
        return runtime.block_pair_only(self, s, z, pair_mask, chunk_size)

    def forward(self, s: Optional[torch.Tensor], z: torch.Tensor, pair_mask: torch.Tensor,
                triangle_multiplicative: str = "torch", triangle_attention: str = "torch",
                inplace_safe: bool = False, chunk_size: Optional[int] = None,
                extra_attn_bias: Optional[torch.Tensor] = None):
        _check_choices(triangle_multiplicative, triangle_attention)
        res = self._maybe_forward_foldcp_pair_only(s, z, pair_mask, chunk_size)
        if res is not None:
            return res
        kernels.require_cuda(z, s, pair_mask)
        if z.dim() != 3:
            raise ValueError("opendde_b200 PairformerBlock takes an unbatched [N, N, c_z] pair tensor")
        n = z.shape[0]
        mask = kernels.prepare_mask(pair_mask, n, n, z.device)
        if inplace_safe and z.is_contiguous():
            zw = z
        else:
            zw = z.contiguous().clone()
        self.pair_updates_(zw, mask)
        if self.c_s > 0:
            bias = None
            if extra_attn_bias is not None:
                bias = self.attention_pair_bias.pair_bias(zw)
                e = extra_attn_bias.to(device=bias.device, dtype=torch.float32)
                bias = (bias + (e if e.dim() == 3 else e[None])).contiguous()
            s = self.single_updates(s, zw if bias is None else None, bias)
        _abi.status_checkpoint(zw.device)
        return s, zw


class PairformerStack(nn.Module):
    """Algorithm 17 PairformerStack (pairformer.py:276-451); no checkpointing (inference)."""

    def __init__(self, n_blocks: int = 48, n_heads: int = 16, c_z: int = 128, c_s: int = 384,
                 num_intermediate_factor: int = 4, blocks_per_ckpt: Optional[int] = None,
                 hidden_scale_up: bool = False) -> None:
        super().__init__()
        self.n_blocks = n_blocks
        self.n_heads = n_heads
        self.blocks_per_ckpt = blocks_per_ckpt
        self.blocks = nn.ModuleList([
            PairformerBlock(n_heads=n_heads, c_z=c_z, c_s=c_s,
                            num_intermediate_factor=num_intermediate_factor,
                            hidden_scale_up=hidden_scale_up)
            for _ in range(n_blocks)])

    def _maybe_forward_foldcp_pair_only(self, s, z, pair_mask, extra_attn_bias, chunk_size=None):
        if os.environ.get("OPENDDE_FOLDCP_MODE", "single") != "distributed":
            return None
        if not dist.is_available() or not dist.is_initialized():
            return None
        from ..distributed.foldcp import runtime
        return runtime.stack_forward(self, s, z, pair_mask, extra_attn_bias, chunk_size)

    def forward(self, s: torch.Tensor, z: torch.Tensor, pair_mask: torch.Tensor,
                triangle_multiplicative: str = "torch", triangle_attention: str = "torch",
                inplace_safe: bool = False, chunk_size: Optional[int] = None,
                extra_attn_bias: Optional[torch.Tensor] = None):
        _check_choices(triangle_multiplicative, triangle_attention)
        res = self._maybe_forward_foldcp_pair_only(s, z, pair_mask, extra_attn_bias, chunk_size)
        if res is not None:
            return res
        kernels.require_cuda(z, s, pair_mask)
        n = z.shape[0]
        mask = kernels.prepare_mask(pair_mask, n, n, z.device)
        zw = z if (inplace_safe and z.is_contiguous()) else z.contiguous().clone()
        for block in self.blocks:
            block.pair_updates_(zw, mask)
            if block.c_s > 0 and s is not None:
                bias = None
                if extra_attn_bias is not None:
                    bias = block.attention_pair_bias.pair_bias(zw)
                    e = extra_attn_bias.to(device=bias.device, dtype=torch.float32)
                    bias = (bias + (e if e.dim() == 3 else e[None])).contiguous()
                s = block.single_updates(s, zw if bias is None else None, bias)
        _abi.status_checkpoint(zw.device)
        return s, zw
