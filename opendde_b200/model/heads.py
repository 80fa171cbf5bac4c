"""Pair work downstream of the stack, drop-in for the pair parts of the reference's heads:

* ``DistogramHead`` (opendde/model/modules/head.py:12-98): symmetric bin logits and the contact
  probabilities of the Fold-CP contact helper (opendde/distributed/foldcp/distogram.py:133-200);
* ``ConfidencePairHead``: the pair steps of ConfidenceHead (opendde/model/modules/confidence.py):
  the pair input before its stack (:289-296, 540-572) and the pae / pde logits (:598-608), under
  the reference's parameter names, so ``load_state_dict(confidence_head_state, strict=False)``
  takes them from a ConfidenceHead checkpoint;
* ``DiffusionPairConditioning``: the pair half of DiffusionConditioning
  (opendde/model/modules/diffusion.py:128-1107): ``prepare_cache`` and its Fold-CP local form.

Each runs on the library's kernels (pf_pair_head_fwd, pf_confidence_pair_init_fwd,
pf_diffusion_pair_cond_fwd); there is no CPU path.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.nn as nn

from .. import _abi, kernels
from .._abi import ConfidenceInitParams, DiffusionPairParams, PairHeadParams, TransitionParams
from .primitives import Linear, LinearNoBias, Transition
from .triangular import LayerNorm
from .trunk_init import RelativePositionEncoding, _relp_features


def _cached_pack(owner: nn.Module, attr: str, struct_cls, spec, f32_names, dtype, device):
    key = kernels.pack_key([p for p in spec.values() if p is not None], dtype, device)
    cached = getattr(owner, attr, None)
    if cached is None or cached.key != key:
        cached = kernels.make_pack(struct_cls, spec, f32_names, dtype, device, key)
        setattr(owner, attr, cached)
    return cached


def bin_tops(min_bin: float, max_bin: float, no_bins: int, dtype: torch.dtype) -> torch.Tensor:
    """The bins' upper edges of the contact helper (foldcp/distogram.py:115-130): no_bins - 1
    evenly spaced boundaries in the logits' dtype, then 1e8."""
    b = torch.linspace(min_bin, max_bin, no_bins - 1, dtype=dtype)
    return torch.cat([b, b.new_tensor([1e8])])


def contact_bin_count(min_bin: float, max_bin: float, no_bins: int, thres: float, dtype: torch.dtype) -> int:
    """How many leading bins have top <= thres (the tops increase, so the selected bins are a prefix)."""
    sel = bin_tops(min_bin, max_bin, no_bins, dtype) <= thres
    n = int(sel.sum().item())
    if not bool(sel[:n].all()):
        raise ValueError("contact bins must be a prefix of the bins")
    return n


def _transposed(z: torch.Tensor) -> torch.Tensor:
    return z.transpose(0, 1)


class DistogramHead(nn.Module):
    """Algorithm 1 line 17 (head.py:12-46): logits = linear(z) + linear(z)^T, one symmetric GEMM
    pass (W (z + z^T) + 2 b) on the tensor cores."""

    def __init__(self, c_z: int = 128, no_bins: int = 64) -> None:
        super().__init__()
        self.c_z = c_z
        self.no_bins = no_bins
        self.linear = Linear(in_features=c_z, out_features=no_bins, initializer="zeros")

    def _pack(self, dtype, device):
        spec = {"ln_w": None, "ln_b": None, "w": self.linear.weight, "b": self.linear.bias}
        return _cached_pack(self, "_opendde_b200_pack", PairHeadParams, spec, {"b"}, dtype, device)

    def logits_tile(self, z: torch.Tensor, zt: torch.Tensor, logits: torch.Tensor,
                    contact: Optional[torch.Tensor] = None, contact_bins: int = 0) -> None:
        """logits (and contact) of a tile whose transpose partner is ``zt`` (zt[r, s] = z(col, row))."""
        kernels.pair_head(self._pack(z.dtype, z.device), _abi.PF_HEAD_SYM_OUT, z, zt, logits, contact, contact_bins)

    def forward(self, z: torch.Tensor) -> torch.Tensor:
        kernels.require_cuda(z)
        if z.dim() != 3:
            raise ValueError("opendde_b200 takes an unbatched [N, N, c_z] pair tensor")
        out = torch.empty(z.shape[:2] + (self.no_bins,), device=z.device, dtype=z.dtype)
        self.logits_tile(z, _transposed(z), out)
        return out

    def contact_probs(self, z: torch.Tensor, min_bin: float, max_bin: float, no_bins: int,
                      thres: float = 8.0) -> torch.Tensor:
        """[N, N] fp32 probability mass of the bins whose top <= thres (foldcp/distogram.py:159-166),
        from the logits the kernel forms in the same pass."""
        kernels.require_cuda(z)
        if no_bins != self.no_bins:
            raise ValueError(f"no_bins {no_bins} != the head's {self.no_bins}")
        logits = torch.empty(z.shape[:2] + (self.no_bins,), device=z.device, dtype=z.dtype)
        contact = torch.empty(z.shape[:2], device=z.device, dtype=torch.float32)
        self.logits_tile(z, _transposed(z), logits, contact,
                         contact_bin_count(min_bin, max_bin, no_bins, thres, z.dtype))
        return contact

    def contact_probs_foldcp_local(self, z_pair_local, z_pair_spec, mesh, min_bin: float, max_bin: float,
                                   no_bins: int, thres: float = 8.0, gather_to_rank0_only: bool = False):
        from ..distributed.foldcp.heads import distributed_distogram_contact_probs
        return distributed_distogram_contact_probs(z_pair_local=z_pair_local, z_pair_spec=z_pair_spec, mesh=mesh,
                                                   head=self, min_bin=min_bin, max_bin=max_bin, no_bins=no_bins,
                                                   thres=thres, gather_to_rank0_only=gather_to_rank0_only)


class ConfidencePairHead(nn.Module):
    """The pair steps of ConfidenceHead (Algorithm 31), reference parameter names."""

    def __init__(self, c_z: int = 128, c_s_inputs: int = 449, b_pae: int = 64, b_pde: int = 64,
                 distance_bin_start: float = 3.25, distance_bin_end: float = 52.0,
                 distance_bin_step: float = 1.25) -> None:
        super().__init__()
        self.c_z = c_z
        self.c_s_inputs = c_s_inputs
        self.b_pae = b_pae
        self.b_pde = b_pde
        self.linear_no_bias_s1 = LinearNoBias(in_features=c_s_inputs, out_features=c_z)
        self.linear_no_bias_s2 = LinearNoBias(in_features=c_s_inputs, out_features=c_z)
        lower = torch.arange(distance_bin_start, distance_bin_end, distance_bin_step)
        upper = torch.cat([lower[1:], lower.new_tensor([1e6])], dim=-1)
        self.lower_bins = nn.Parameter(lower, requires_grad=False)
        self.upper_bins = nn.Parameter(upper, requires_grad=False)
        self.num_bins = len(lower)
        self.linear_no_bias_d = LinearNoBias(in_features=self.num_bins, out_features=c_z)
        self.linear_no_bias_d_wo_onehot = LinearNoBias(in_features=1, out_features=c_z)
        self.linear_no_bias_pae = LinearNoBias(in_features=c_z, out_features=b_pae)
        self.linear_no_bias_pde = LinearNoBias(in_features=c_z, out_features=b_pde)
        self.pae_ln = LayerNorm(c_z)
        self.pde_ln = LayerNorm(c_z)
        with torch.no_grad():
            nn.init.zeros_(self.linear_no_bias_pae.weight)
            nn.init.zeros_(self.linear_no_bias_pde.weight)

    def _init_pack(self, dtype, device):
        spec = {"w_s1": self.linear_no_bias_s1.weight, "w_s2": self.linear_no_bias_s2.weight,
                "w_d": self.linear_no_bias_d.weight, "w_d0": self.linear_no_bias_d_wo_onehot.weight,
                "lower_bins": self.lower_bins, "upper_bins": self.upper_bins}
        return _cached_pack(self, "_opendde_b200_init_pack", ConfidenceInitParams, spec,
                            {"lower_bins", "upper_bins"}, dtype, device)

    def _head_pack(self, which: str, dtype, device):
        ln = getattr(self, f"{which}_ln")
        spec = {"ln_w": ln.weight, "ln_b": ln.bias, "w": getattr(self, f"linear_no_bias_{which}").weight, "b": None}
        return _cached_pack(self, f"_opendde_b200_{which}_pack", PairHeadParams, spec, {"ln_w", "ln_b"}, dtype,
                            device)

    def embed_pair_tile(self, s_inputs: torch.Tensor, x_rep_coords: torch.Tensor, z_trunk: torch.Tensor,
                        out: torch.Tensor, row0: int = 0, col0: int = 0) -> torch.Tensor:
        """out [R, C, c_z] = the pair input on rows [row0, row0 + R) x cols [col0, col0 + C)
        (out may be z_trunk: updated in place)."""
        kernels.require_cuda(s_inputs, x_rep_coords, z_trunk, out)
        s = s_inputs if s_inputs.stride(-1) == 1 else s_inputs.contiguous()
        coords = x_rep_coords.to(torch.float32).contiguous()
        kernels.confidence_pair_init(self._init_pack(z_trunk.dtype, z_trunk.device), s.to(z_trunk.dtype), coords,
                                     z_trunk, out, row0, col0, self.num_bins)
        return out

    def embed_pair(self, s_inputs: torch.Tensor, z_trunk: torch.Tensor, x_rep_coords: torch.Tensor) -> torch.Tensor:
        """z_trunk + s_inputs projections + the distance embedding of the representative atoms
        (confidence.py:289-296, 540-572): a new [N, N, c_z] tensor."""
        out = torch.empty_like(z_trunk)
        return self.embed_pair_tile(s_inputs, x_rep_coords, z_trunk, out)

    def pair_logits_tile(self, z: torch.Tensor, zt: Optional[torch.Tensor], pae: Optional[torch.Tensor],
                         pde: Optional[torch.Tensor]) -> None:
        """pae / pde (fp32, [R, C, bins]) of a tile whose transpose partner is ``zt``."""
        if pae is not None:
            kernels.pair_head(self._head_pack("pae", z.dtype, z.device), _abi.PF_HEAD_PLAIN, z, None, pae)
        if pde is not None:
            kernels.pair_head(self._head_pack("pde", z.dtype, z.device), _abi.PF_HEAD_SYM_IN, z, zt, pde)

    def pair_logits(self, z: torch.Tensor, compute_pae: bool = True,
                    compute_pde: bool = True) -> Tuple[Optional[torch.Tensor], Optional[torch.Tensor]]:
        """pae = linear_no_bias_pae(pae_ln(z)), pde = linear_no_bias_pde(pde_ln(z + z^T)), fp32
        [N, N, bins] (confidence.py:598-608)."""
        kernels.require_cuda(z)
        n = z.shape[0]
        pae = torch.empty((n, n, self.b_pae), device=z.device, dtype=torch.float32) if compute_pae else None
        pde = torch.empty((n, n, self.b_pde), device=z.device, dtype=torch.float32) if compute_pde else None
        self.pair_logits_tile(z, _transposed(z), pae, pde)
        return pae, pde


class DiffusionPairConditioning(nn.Module):
    """The pair half of DiffusionConditioning (Algorithm 21 lines 1-5), reference parameter names."""

    def __init__(self, c_z: int = 128, c_z_pair_diffusion: Optional[int] = None) -> None:
        super().__init__()
        self.c_z = c_z
        self.c_z_pair_diffusion = c_z if c_z_pair_diffusion is None else c_z_pair_diffusion
        self.compress_pair_z = self.c_z_pair_diffusion != c_z
        c_zd = self.c_z_pair_diffusion
        self.relpe = RelativePositionEncoding(c_z=c_zd)
        if self.compress_pair_z:
            self.layernorm_z_trunk = LayerNorm(c_z, create_offset=False)
            self.linear_no_bias_z_trunk = LinearNoBias(in_features=c_z, out_features=c_zd, precision=torch.float32)
        self.layernorm_z = LayerNorm(2 * c_zd, create_offset=False)
        self.linear_no_bias_z = LinearNoBias(in_features=2 * c_zd, out_features=c_zd, precision=torch.float32)
        self.transition_z1 = Transition(c_in=c_zd, n=2)
        self.transition_z2 = Transition(c_in=c_zd, n=2)

    def _pack(self, dtype, device):
        f32 = {"ln_zt_w", "ln_z_w", "t1_ln_w", "t1_ln_b", "t2_ln_w", "t2_ln_b"}
        spec = {"w_relp": self.relpe.linear_no_bias.weight, "ln_z_w": self.layernorm_z.weight,
                "w_z": self.linear_no_bias_z.weight,
                "ln_zt_w": self.layernorm_z_trunk.weight if self.compress_pair_z else None,
                "w_zt": self.linear_no_bias_z_trunk.weight if self.compress_pair_z else None}
        for tag, t in (("t1", self.transition_z1), ("t2", self.transition_z2)):
            spec.update({f"{tag}_ln_w": t.layernorm1.weight, f"{tag}_ln_b": t.layernorm1.bias,
                         f"{tag}_w_a": t.linear_no_bias_a.weight, f"{tag}_w_b": t.linear_no_bias_b.weight,
                         f"{tag}_w_o": t.linear_no_bias.weight})
        key = kernels.pack_key([p for p in spec.values() if p is not None], dtype, device)
        cached = getattr(self, "_opendde_b200_pack", None)
        if cached is None or cached.key != key:
            tensors = {n: (None if p is None else p.detach().to(device=device, dtype=torch.float32 if n in f32 else
                                                                  dtype).contiguous()) for n, p in spec.items()}
            ptr = {n: (None if t is None else t.data_ptr()) for n, t in tensors.items()}

            def tp(tag):
                return TransitionParams(ln_w=ptr[f"{tag}_ln_w"], ln_b=ptr[f"{tag}_ln_b"], w_a=ptr[f"{tag}_w_a"],
                                        w_b=ptr[f"{tag}_w_b"], w_o=ptr[f"{tag}_w_o"])

            struct = DiffusionPairParams(ln_zt_w=ptr["ln_zt_w"], w_zt=ptr["w_zt"], w_relp=ptr["w_relp"],
                                         ln_z_w=ptr["ln_z_w"], w_z=ptr["w_z"], t1=tp("t1"), t2=tp("t2"))
            cached = kernels.WeightPack(key, tensors, struct)
            self._opendde_b200_pack = cached
        return cached

    def prepare_cache_tile(self, relp_feature, z_trunk: torch.Tensor, out: torch.Tensor, row0: int = 0,
                           col0: int = 0) -> torch.Tensor:
        """out [R, C, c_z_pair_diffusion] = the conditioned pair on rows [row0, row0 + R) x cols
        [col0, col0 + C) of the plane, from the matching tile of z_trunk and the token ids."""
        kernels.require_cuda(z_trunk, out)
        feats = _relp_features(relp_feature)
        kernels.diffusion_pair_cond(self._pack(z_trunk.dtype, z_trunk.device), z_trunk, feats.ids(z_trunk.device),
                                    out, row0, col0, feats.n_token, int(feats.r_max), int(feats.s_max))
        return out

    def prepare_cache(self, relp_feature, z_trunk: torch.Tensor, inplace_safe: bool = False) -> torch.Tensor:
        """diffusion.py:828-847 (+ the transitions of :1019-1040): a new [N, N, c_zd] tensor."""
        del inplace_safe
        kernels.require_cuda(z_trunk)
        if z_trunk.dim() != 3:
            raise ValueError("opendde_b200 takes an unbatched [N, N, c_z] z_trunk")
        n = z_trunk.shape[0]
        out = torch.empty((n, n, self.c_z_pair_diffusion), device=z_trunk.device, dtype=z_trunk.dtype)
        return self.prepare_cache_tile(relp_feature, z_trunk, out)

    def prepare_cache_foldcp_local(self, relp_feature, z_trunk_local: torch.Tensor, z_spec, mesh,
                                   inplace_safe: bool = False):
        from ..distributed.foldcp.heads import diffusion_prepare_cache_local
        del inplace_safe
        return diffusion_prepare_cache_local(self, relp_feature, z_trunk_local, z_spec, mesh)
