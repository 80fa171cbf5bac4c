"""Host-side behaviour of the drop-in modules (no GPU): names, errors, no CPU fallback."""
import numpy as np
import pytest
import torch

from golden_cases import GOLDEN_DIR, module_for
from opendde_b200.model import PairformerBlock, PairformerStack, TriangleAttention, TriangleMultiplicationOutgoing


@pytest.mark.parametrize("kind,fname", [("block", "block_n16.npz"), ("trimul_out", "trimul_out_n13.npz"),
                                        ("triatt_start", "triatt_start_n13.npz"), ("apb", "apb_n13.npz")])
def test_parameter_names_match_reference(kind, fname):
    rec = np.load(f"{GOLDEN_DIR}/{fname}")
    names = sorted(n for n, _ in module_for(kind).named_parameters())
    assert names == list(rec["param_names"])


def test_stack_state_dict_keys():
    st = PairformerStack(n_blocks=2)
    keys = set(st.state_dict())
    assert "blocks.1.tri_att_end.mha.linear_g.weight" in keys
    assert "blocks.0.attention_pair_bias.attention.linear_q.bias" in keys


def test_invalid_kernel_strings_raise_reference_errors():
    tm = TriangleMultiplicationOutgoing(c_z=16, c_hidden=16)
    with pytest.raises(ValueError, match="triangle_multiplicative must be 'cuequivariance' or 'torch'"):
        tm(torch.zeros(4, 4, 16), triangle_multiplicative="triton")
    ta = TriangleAttention(16, 8, 2)
    with pytest.raises(ValueError, match="Invalid triangle_attention"):
        ta(torch.zeros(4, 4, 16), triangle_attention="bogus")
    blk = PairformerBlock(c_z=32, c_s=0, c_hidden_mul=32, no_heads_pair=1)
    with pytest.raises(ValueError):
        blk(None, torch.zeros(4, 4, 32), torch.ones(4, 4), triangle_attention="x")


def test_cpu_tensors_are_rejected_no_fallback():
    tm = TriangleMultiplicationOutgoing(c_z=16, c_hidden=16)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        tm(torch.zeros(4, 4, 16))
    blk = PairformerBlock(c_z=32, c_s=0, c_hidden_mul=32, no_heads_pair=1)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        blk(None, torch.zeros(4, 4, 32), torch.ones(4, 4))


@pytest.mark.parametrize("config", ["trunk_block", "msa_pair_stack", "msa_pair_stack_scaled", "template_stack",
                                    "confidence_stack", "refiner_stack_scaled"])
def test_state_dict_matches_reference_in_every_caller_configuration(config):
    """Checkpoints of every Pairformer user load unchanged: the same state_dict keys and
    shapes as the reference modules (tests/golden/api_shapes.json, made by
    tests/golden/make_api_fixtures.py from the reference)."""
    import json
    import os
    from opendde_b200 import model as M
    ref = json.load(open(os.path.join(GOLDEN_DIR, "api_shapes.json")))[config]
    mod = getattr(M, ref["class"])(**ref["kwargs"])
    got = {k: list(v.shape) for k, v in mod.state_dict().items()}
    assert got == ref["params"]


def test_outer_product_mean_parameter_names_match_reference():
    """The parameter names and shapes of the reference OuterProductMean (the golden fixture was
    made by tests/golden/make_opm_golden.py from the reference module)."""
    from opendde_b200.model import OuterProductMean
    rec = np.load(f"{GOLDEN_DIR}/opm/opm_s7_n13_masked.npz")
    mod = OuterProductMean(c_m=int(rec["c_m"]), c_z=int(rec["c_z"]), c_hidden=int(rec["c_hidden"]))
    assert sorted(n for n, _ in mod.named_parameters()) == list(rec["param_names"])
    assert tuple(mod.linear_out.weight.shape) == (int(rec["c_z"]), int(rec["c_hidden"]) ** 2)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        mod(torch.zeros(3, 5, int(rec["c_m"])))


def test_trunk_init_module_api():
    """RelativePositionEncoding keeps the reference's parameter name and shape; the lazy (id)
    features are the only input form; CPU tensors are rejected (no CPU fallback)."""
    from opendde_b200.model import RelativePositionEncoding, trunk_pair_init
    from opendde_b200.model.primitives import LinearNoBias
    rec = np.load(f"{GOLDEN_DIR}/trunk/trunk_init_n23.npz")
    relpe = RelativePositionEncoding(r_max=int(rec["r_max"]), s_max=int(rec["s_max"]), c_z=int(rec["c_z"]))
    assert [n for n, _ in relpe.named_parameters()] == ["linear_no_bias.weight"]
    i = list(rec["param_names"]).index("relative_position_encoding.linear_no_bias.weight")
    assert relpe.linear_no_bias.weight.shape[1] == 4 * int(rec["r_max"]) + 2 * int(rec["s_max"]) + 7
    n, c_s, c_z = 5, int(rec["c_s"]), int(rec["c_z"])
    d = {"asym_id": torch.zeros(n, dtype=torch.long), "residue_index": torch.arange(n),
         "entity_id": torch.zeros(n, dtype=torch.long), "token_index": torch.arange(n),
         "sym_id": torch.zeros(n, dtype=torch.long)}
    feats = relpe.generate_relp(d)["relp"]
    assert feats.shape == (n, n, relpe.linear_no_bias.weight.shape[1]) and i >= 0
    z1, z2, bond = LinearNoBias(c_s, c_z), LinearNoBias(c_s, c_z), LinearNoBias(1, c_z)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        trunk_pair_init(torch.zeros(n, c_s), z1, z2, relpe, bond, feats, None)
    with pytest.raises(TypeError, match="lazy"):
        from opendde_b200.model.trunk_init import _relp_features
        _relp_features(torch.zeros(n, n, 23))
