"""B200-native (sm_100a) Pairformer pair stack for OpenDDE.

Drop-in replacements for the reference's TriangleAttention, TriangleMultiplication*,
Transition, AttentionPairBias, PairformerBlock/PairformerStack and the Fold-CP
pair-sharding API, backed by hand-written CUDA kernels behind a C ABI
(``include/pairformer_b200.h``, ``libpairformer_b200.so``).
"""

__version__ = "0.1.0"
