"""Fold-CP: 2D context parallelism of the Pairformer pair stack over an R x C GPU mesh
(drop-in for opendde/distributed/foldcp; square meshes generalised to R x C)."""

from .config import FOLDCP_ENVIRONMENT_KEYS, FOLDCP_MESH_KEY, FoldCPConfig, apply_foldcp_config
from .layout import FoldCP2DLayout
from .mesh import FoldCPProcessMesh, clear_mesh_cache
from .heads import (
    confidence_pair_input_local,
    confidence_pair_logits_local,
    diffusion_prepare_cache_local,
    distogram_contact_probs_local,
    distributed_confidence_pair_logits,
    distributed_distogram_contact_probs,
)
from .opm import outer_product_mean_local_update
from .trunk_init import apply_trunk_z_cycle_local, build_trunk_z_init_local
from .pair_sharding import (
    FoldCPPairShardSpec,
    gather_pair_tensor,
    gather_pair_tensor_like,
    gather_pair_tensor_like_to_rank,
    infer_pair_dims,
    make_pair_shard_spec,
    shard_pair_feature_dict,
    shard_pair_tensor,
)
from .real_pairformer import (
    FoldCPPairContext,
    distributed_attention_pair_bias_update,
    distributed_pair_transition_update,
    distributed_pairformer_block_pair_update,
    distributed_pairformer_stack_pair_update,
    distributed_pairformer_stack_single_bridge_update,
    distributed_triangle_attention_update,
    distributed_triangle_multiplication_update,
    make_context,
)

__all__ = [
    "FOLDCP_ENVIRONMENT_KEYS", "FOLDCP_MESH_KEY", "FoldCPConfig", "apply_foldcp_config", "FoldCP2DLayout",
    "FoldCPProcessMesh", "clear_mesh_cache", "FoldCPPairShardSpec", "gather_pair_tensor",
    "gather_pair_tensor_like", "gather_pair_tensor_like_to_rank", "infer_pair_dims", "make_pair_shard_spec",
    "shard_pair_feature_dict", "shard_pair_tensor", "FoldCPPairContext", "make_context",
    "distributed_attention_pair_bias_update", "distributed_pair_transition_update",
    "distributed_pairformer_block_pair_update", "distributed_pairformer_stack_pair_update",
    "distributed_pairformer_stack_single_bridge_update", "distributed_triangle_attention_update",
    "distributed_triangle_multiplication_update", "outer_product_mean_local_update", "build_trunk_z_init_local",
    "apply_trunk_z_cycle_local", "distogram_contact_probs_local", "distributed_distogram_contact_probs",
    "confidence_pair_logits_local", "distributed_confidence_pair_logits", "confidence_pair_input_local",
    "diffusion_prepare_cache_local",
]
