"""Pin the CPU oracle against golden vectors produced by the reference modules themselves."""
import numpy as np
import pytest
import torch

from golden_cases import CASE_FILES, checksum, load_case
from oracle import pairformer_oracle as O

TOL = 2e-5  # max-abs, fp32 vs fp32 with a different summation order


@pytest.mark.parametrize("fname", CASE_FILES)
def test_oracle_matches_reference_golden(fname):
    torch.set_num_threads(4)
    kind, n, s, z, mask, params, rec, _ = load_case(fname)
    # the regenerated inputs/weights are the ones the reference saw
    np.testing.assert_allclose(checksum(z), rec["chk_z"], rtol=1e-10)
    np.testing.assert_allclose(checksum(s), rec["chk_s"], rtol=1e-10)
    np.testing.assert_allclose(checksum(mask), rec["chk_mask"], rtol=1e-10)
    assert list(rec["param_names"]) == sorted(params)
    np.testing.assert_allclose(np.stack([checksum(params[k]) for k in sorted(params)]),
                               rec["chk_params"], rtol=1e-10)
    with torch.no_grad():
        if kind == "trimul_out":
            out = {"out": O.triangle_multiplication(z, mask, params, outgoing=True)}
        elif kind == "trimul_in":
            out = {"out": O.triangle_multiplication(z, mask, params, outgoing=False)}
        elif kind == "triatt_start":
            out = {"out": O.triangle_attention(z, mask, params, 4, starting=True)}
        elif kind == "triatt_end":
            out = {"out": O.triangle_attention(z, mask, params, 4, starting=False)}
        elif kind == "transition":
            out = {"out": O.transition(z, params)}
        elif kind == "apb":
            out = {"out": O.attention_pair_bias(s, z, params, 16)}
        else:
            s_out, z_out = O.pairformer_block(s, z, mask, params)
            out = {"s_out": s_out, "z_out": z_out}
    for k, v in out.items():
        ref = torch.from_numpy(rec[k])
        err = (v - ref).abs().max().item()
        assert err <= TOL, f"{fname}:{k} max-abs {err:.3e} > {TOL}"


def test_oracle_fully_masked_row_is_uniform_average():
    """A fully masked query row averages V uniformly (reference semantics, 1e9 additive mask)."""
    _, n, s, z, mask, params, rec, _ = load_case("triatt_start_n13.npz")
    out = torch.from_numpy(rec["out"])
    m2 = mask.clone()
    m2[n - 1] = 0.0
    got = O.triangle_attention(z, m2, params, 4, starting=True)
    assert torch.allclose(got[n - 1], out[n - 1], atol=TOL)
