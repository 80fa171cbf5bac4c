"""Multi-GPU execution of the Pairformer pair stack (Fold-CP 2D context parallelism)."""
