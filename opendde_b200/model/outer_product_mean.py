"""OuterProductMean (Algorithm 10), drop-in for ``opendde.model.triangular.layers.OuterProductMean``.

Constructor arguments, parameter names (``layer_norm``, ``linear_1``, ``linear_2``,
``linear_out``) and the forward signature are the reference's (layers.py:497-627); the
forward body calls ``pf_opm_fwd``. ``tile_update`` is the Fold-CP pair-tile form of the same
update (opendde/model/modules/pairformer.py:979-1046): the tile of rows / columns a rank owns,
computed from the full MSA representation without forming the rest of the pair update.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.nn as nn

from .. import kernels
from .._abi import OpmParams
from .triangular import LayerNorm, OpenfoldLinear


class OuterProductMean(nn.Module):
    def __init__(self, c_m: int, c_z: int, c_hidden: int, eps: float = 1e-3) -> None:
        super().__init__()
        self.c_m = c_m
        self.c_z = c_z
        self.c_hidden = c_hidden
        self.eps = eps
        self.layer_norm = LayerNorm(c_m)
        self.linear_1 = OpenfoldLinear(c_m, c_hidden, bias=False)
        self.linear_2 = OpenfoldLinear(c_m, c_hidden, bias=False)
        self.linear_out = OpenfoldLinear(c_hidden ** 2, c_z, init="final")
        self._pack = None

    def weight_pack(self, dtype, device) -> kernels.WeightPack:
        spec = {"ln_w": self.layer_norm.weight, "ln_b": self.layer_norm.bias, "w_1": self.linear_1.weight,
                "w_2": self.linear_2.weight, "w_out": self.linear_out.weight, "b_out": self.linear_out.bias}
        key = kernels.pack_key([p for p in spec.values() if p is not None], dtype, device)
        if self._pack is None or self._pack.key != key:
            self._pack = kernels.make_pack(OpmParams, spec, {"ln_w", "ln_b", "b_out"}, dtype, device, key)
        return self._pack

    def apply_(self, m: torch.Tensor, mask: Optional[torch.Tensor], out: torch.Tensor, accumulate: bool,
               row0: int = 0, col0: int = 0) -> torch.Tensor:
        """out (+)= the update of rows [row0, row0 + out.shape[0]) x cols [col0, col0 + out.shape[1])."""
        if m.dim() != 3:
            raise ValueError("opendde_b200 OuterProductMean takes an unbatched [N_seq, N_res, C_m] MSA tensor")
        m = m if m.stride(-1) == 1 else m.contiguous()
        mk = None
        if mask is not None:
            mk = mask.to(device=m.device, dtype=torch.float32)
        kernels.opm(self.weight_pack(m.dtype, m.device), m, mk, out, row0, col0, self.c_hidden, self.eps,
                    accumulate)
        return out

    def forward(self, m: torch.Tensor, mask: Optional[torch.Tensor] = None, chunk_size: Optional[int] = None,
                inplace_safe: bool = False) -> torch.Tensor:
        """[N_seq, N_res, C_m] MSA embedding (and [N_seq, N_res] mask) -> [N_res, N_res, C_z] update.
        ``chunk_size`` and ``inplace_safe`` are accepted for the reference's signature; the kernels
        do not materialise the [N_res, N_res, C_hidden^2] outer product, so there is nothing to chunk."""
        kernels.require_cuda(m, mask)
        n_res = m.shape[-2]
        out = torch.empty((n_res, n_res, self.c_z), device=m.device, dtype=m.dtype)
        return self.apply_(m, mask, out, accumulate=False)

    def tile_update(self, m: torch.Tensor, mesh_shape: Tuple[int, int], mesh_coord: Tuple[int, int],
                    mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        """The [ceil(N/R), ceil(N/C), c_z] pair tile of mesh position ``mesh_coord`` on an R x C
        mesh, zero-padded past N (the reference's _outer_product_mean_tile_update, pairformer.py
        :979-1046, which is called without a mask)."""
        kernels.require_cuda(m, mask)
        n_res = m.shape[-2]
        rows, cols = mesh_shape
        row_tile, col_tile = -(-n_res // rows), -(-n_res // cols)
        r0, c0 = mesh_coord[0] * row_tile, mesh_coord[1] * col_tile
        r1, c1 = min(r0 + row_tile, n_res), min(c0 + col_tile, n_res)
        out = torch.zeros((row_tile, col_tile, self.c_z), device=m.device, dtype=m.dtype)
        if r0 < r1 and c0 < c1:
            self.apply_(m, mask, out[: r1 - r0, : c1 - c0], accumulate=False, row0=r0, col0=c0)
        return out
