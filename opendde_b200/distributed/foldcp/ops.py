"""Local compute of the Fold-CP pair ops on tiles and bands, through the CUDA kernels.

Each method is one C-ABI call on strided views of the local tile or of an exchanged band
(no reshaping copies). The distributed drivers take any object with these methods, so the
exchange logic can be exercised on CPU process groups with a host implementation.
"""

from __future__ import annotations

import torch

from ... import kernels


class KernelOps:
    """The library's kernels (bf16 -> tcgen05 path where covered, fp32 -> SIMT fp32)."""

    def bias_dtype(self, z_dtype: torch.dtype) -> torch.dtype:
        """Storage type of the triangle-attention bias the kernels exchange: f16 in log2
        units for bf16 pair tensors, fp32 natural units for fp32."""
        return torch.float16 if z_dtype == torch.bfloat16 else torch.float32

    def trimul(self, module, za, zb, ma, mb, zg, zo) -> None:
        """zo += TriangleMultiplicativeUpdate over the band views (x_ij = sum_k a(za_ik) b(zb_jk))."""
        kernels.trimul(module.weight_pack(zo.dtype, zo.device), za, zb, ma, mb, zg, zo, module.c_hidden, True)

    def trimul_project(self, module, z_view, m_view, a_ptr: int, b_ptr: int, ld: int) -> None:
        """a, b projections of ``z_view`` written channel-major [c_h][rows][ld] at raw device
        addresses (a peer window)."""
        kernels.trimul_project(module.weight_pack(z_view.dtype, z_view.device), z_view, m_view, module.c_hidden,
                               a_ptr, b_ptr, ld)

    def trimul_combine(self, module, a, b, n_k: int, zg, zo) -> None:
        """zo += the triangle update from exchanged projection bands."""
        kernels.trimul_combine(module.weight_pack(zo.dtype, zo.device), a, b, n_k, zg, zo, True)

    def triatt_bias(self, module, z_view, out) -> None:
        """out[h, r, s] = triangle bias of z_view(r, s), in ``bias_dtype`` format."""
        kernels.triatt_bias(module.weight_pack(z_view.dtype, z_view.device), z_view, module.no_heads, out)

    def triatt(self, module, zs, m, bias, zo, q_col0: int, n_q: int, n_valid: int) -> None:
        """zo += starting-node attention of rows of ``zs`` for queries [q_col0, q_col0 + n_q)."""
        kernels.triatt(module.weight_pack(zs.dtype, zs.device), zs, m, zo, module.no_heads, module.c_hidden,
                       module.inf, True, bias=bias, q_col0=q_col0, n_q=n_q, n_valid_keys=n_valid)

    def transition(self, module, x2d) -> None:
        kernels.transition(module.weight_pack(x2d.dtype, x2d.device), x2d, x2d, module.n, True)

    def apb_pair_bias(self, module, z_view, out) -> None:
        kernels.apb_pair_bias(module.weight_pack(z_view.dtype, z_view.device), z_view, module.n_heads, out)

    def apb_rows(self, module, s, s_rows, bias_rows, q_row0: int) -> None:
        kernels.apb_rows(module.weight_pack(s.dtype, s.device), s, s_rows, bias_rows, q_row0, module.n_heads, True)

    def single_transition(self, module, s_rows) -> None:
        kernels.transition(module.weight_pack(s_rows.dtype, s_rows.device), s_rows, s_rows, module.n, True)
