"""The trunk's pair input and its recycling step, drop-in for the pieces the reference composes
in opendde/model/opendde.py:812-835 (``linear_no_bias_zinit1/2``, ``relative_position_encoding``,
``linear_no_bias_token_bond``, ``layernorm_z_cycle``, ``linear_no_bias_z_cycle``) and for
``RelativePositionEncoding`` / ``LazyRelativePositionEncodingFeatures``
(opendde/model/modules/embedders.py:87-302).

The relative-position features stay as the five per-token id vectors: the kernel
(pf_trunk_init_fwd) turns each pair's four one-hot indices into a sum of four weight columns,
so the [N, N, 4 r_max + 2 s_max + 7] feature tensor and its GEMM never exist.
"""

from __future__ import annotations

from typing import Any, Dict, Optional

import torch
import torch.nn as nn

from .. import kernels
from .._abi import PairLinearParams, TrunkInitParams
from .primitives import LinearNoBias

_ID_KEYS = ("asym_id", "residue_index", "entity_id", "token_index", "sym_id")


class LazyRelativePositionEncodingFeatures:
    """The per-token ids the relative-position features are built from (embedders.py:87-122)."""

    def __init__(self, asym_id: torch.Tensor, residue_index: torch.Tensor, entity_id: torch.Tensor,
                 token_index: torch.Tensor, sym_id: torch.Tensor, r_max: int, s_max: int) -> None:
        self.asym_id = asym_id
        self.residue_index = residue_index
        self.entity_id = entity_id
        self.token_index = token_index
        self.sym_id = sym_id
        self.r_max = r_max
        self.s_max = s_max

    @property
    def n_token(self) -> int:
        return int(self.asym_id.shape[-1])

    @property
    def feature_dim(self) -> int:
        return 4 * self.r_max + 2 * self.s_max + 7

    @property
    def shape(self):
        return (*self.asym_id.shape[:-1], self.n_token, self.n_token, self.feature_dim)

    @property
    def device(self) -> torch.device:
        return self.asym_id.device

    def ids(self, device) -> tuple:
        """The five id vectors as contiguous int32 tensors on ``device`` (the kernel's input)."""
        out = []
        for k in _ID_KEYS:
            t = getattr(self, k)
            if t.dim() != 1:
                raise ValueError("opendde_b200 takes unbatched [N_token] id vectors")
            out.append(t.to(device=device, dtype=torch.int32).contiguous())
        return tuple(out)


class RelativePositionEncoding(nn.Module):
    """Algorithm 3 (embedders.py:197-302): ``linear_no_bias`` over the one-hot features."""

    def __init__(self, r_max: int = 32, s_max: int = 2, c_z: int = 128) -> None:
        super().__init__()
        self.r_max = r_max
        self.s_max = s_max
        self.c_z = c_z
        self.linear_no_bias = LinearNoBias(in_features=4 * r_max + 2 * s_max + 7, out_features=c_z)
        self.input_feature = {"asym_id": 1, "residue_index": 1, "entity_id": 1, "sym_id": 1, "token_index": 1}

    def generate_relp(self, input_feature_dict: Dict[str, Any], lazy: bool = True) -> Dict[str, Any]:
        """Store the features in ``input_feature_dict["relp"]``, always in the lazy (id) form."""
        input_feature_dict["relp"] = LazyRelativePositionEncodingFeatures(
            *[input_feature_dict[k] for k in _ID_KEYS], r_max=self.r_max, s_max=self.s_max)
        return input_feature_dict


def _relp_features(relp_feature) -> LazyRelativePositionEncodingFeatures:
    if isinstance(relp_feature, LazyRelativePositionEncodingFeatures) or all(
            hasattr(relp_feature, k) for k in _ID_KEYS):
        return relp_feature
    raise TypeError("opendde_b200 builds the relative-position term from the token ids: pass the lazy features "
                    "(RelativePositionEncoding.generate_relp(..., lazy=True)), not a dense feature tensor")


def _init_pack(linear_zinit1, linear_zinit2, relpe, linear_token_bond, dtype, device):
    spec = {"w_zinit1": linear_zinit1.weight, "w_zinit2": linear_zinit2.weight,
            "w_relp": relpe.linear_no_bias.weight, "w_bond": linear_token_bond.weight}
    key = kernels.pack_key(list(spec.values()), dtype, device)
    cached = getattr(relpe, "_opendde_b200_pack", None)
    if cached is None or cached.key != key:
        cached = kernels.make_pack(TrunkInitParams, spec, set(), dtype, device, key)
        relpe._opendde_b200_pack = cached
    return cached


def trunk_pair_init_tile(s_init: torch.Tensor, linear_zinit1: nn.Module, linear_zinit2: nn.Module,
                         relative_position_encoding: nn.Module, linear_token_bond: nn.Module, relp_feature,
                         token_bonds: Optional[torch.Tensor], out: torch.Tensor, row0: int = 0,
                         col0: int = 0) -> torch.Tensor:
    """out [R, C, c_z] = z_init on rows [row0, row0 + R) x cols [col0, col0 + C) (opendde.py:812-827)."""
    kernels.require_cuda(s_init, out, token_bonds)
    if s_init.dim() != 2:
        raise ValueError("opendde_b200 takes an unbatched [N_token, c_s] s_init")
    feats = _relp_features(relp_feature)
    s = s_init if s_init.stride(-1) == 1 else s_init.contiguous()
    bonds = None if token_bonds is None else token_bonds.to(device=s.device, dtype=torch.float32)
    pack = _init_pack(linear_zinit1, linear_zinit2, relative_position_encoding, linear_token_bond, s.dtype, s.device)
    kernels.trunk_init(pack, s, feats.ids(s.device), bonds, out, row0, col0, int(feats.r_max), int(feats.s_max))
    return out


def trunk_pair_init(s_init: torch.Tensor, linear_zinit1: nn.Module, linear_zinit2: nn.Module,
                    relative_position_encoding: nn.Module, linear_token_bond: nn.Module, relp_feature,
                    token_bonds: Optional[torch.Tensor]) -> torch.Tensor:
    """The full [N, N, c_z] z_init of opendde.py:812-827."""
    n = s_init.shape[0]
    out = torch.empty((n, n, linear_zinit1.weight.shape[0]), device=s_init.device, dtype=s_init.dtype)
    return trunk_pair_init_tile(s_init, linear_zinit1, linear_zinit2, relative_position_encoding, linear_token_bond,
                                relp_feature, token_bonds, out)


def trunk_pair_cycle(z_init: torch.Tensor, z: torch.Tensor, layernorm_z_cycle: nn.Module,
                     linear_z_cycle: nn.Module) -> torch.Tensor:
    """z_init + linear_no_bias_z_cycle(layernorm_z_cycle(z)) (opendde.py:835), a new tensor."""
    kernels.require_cuda(z_init, z)
    spec = {"ln_w": layernorm_z_cycle.weight, "ln_b": layernorm_z_cycle.bias, "w": linear_z_cycle.weight}
    key = kernels.pack_key([p for p in spec.values() if p is not None], z.dtype, z.device)
    cached = getattr(linear_z_cycle, "_opendde_b200_pack", None)
    if cached is None or cached.key != key:
        cached = kernels.make_pack(PairLinearParams, spec, {"ln_w", "ln_b"}, z.dtype, z.device, key)
        linear_z_cycle._opendde_b200_pack = cached
    out = z_init.clone()
    kernels.pair_ln_linear(cached, z if z.stride(-1) == 1 else z.contiguous(), out, accumulate=True)
    return out
