"""Module mirror of opendde.model (Pairformer pair stack only)."""
from .heads import ConfidencePairHead, DiffusionPairConditioning, DistogramHead  # noqa: F401
from .outer_product_mean import OuterProductMean  # noqa: F401
from .pairformer import PairformerBlock, PairformerStack  # noqa: F401
from .primitives import Linear, LinearNoBias, Transition  # noqa: F401
from .transformer import AttentionPairBias  # noqa: F401
from .trunk_init import (  # noqa: F401
    LazyRelativePositionEncodingFeatures,
    RelativePositionEncoding,
    trunk_pair_cycle,
    trunk_pair_init,
    trunk_pair_init_tile,
)
from .triangular import (  # noqa: F401
    LayerNorm,
    OpenfoldLinear,
    TriangleAttention,
    TriangleMultiplicationIncoming,
    TriangleMultiplicationOutgoing,
    TriangleMultiplicativeUpdate,
)
