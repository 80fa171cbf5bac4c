"""R x C rank layout of a Fold-CP group (generalises opendde/distributed/foldcp/layout.py:11-53,
which requires a square mesh). Ranks are row-major: rank = row * C + col."""

from __future__ import annotations

from dataclasses import dataclass
from typing import Tuple


@dataclass(frozen=True)
class FoldCP2DLayout:
    shape: Tuple[int, int]

    def __post_init__(self) -> None:
        if len(self.shape) != 2:
            raise ValueError("FoldCP2DLayout expects a 2D shape.")
        if self.shape[0] < 1 or self.shape[1] < 1:
            raise ValueError("Fold-CP mesh sides must be positive.")

    @property
    def numel(self) -> int:
        return self.shape[0] * self.shape[1]

    @property
    def is_square(self) -> bool:
        return self.shape[0] == self.shape[1]

    def to_linear(self, coord: Tuple[int, int]) -> int:
        row, col = coord
        rows, cols = self.shape
        if not (0 <= row < rows and 0 <= col < cols):
            raise ValueError(f"Coordinate {coord} is outside mesh shape {self.shape}.")
        return row * cols + col

    def to_coord(self, linear_rank: int) -> Tuple[int, int]:
        if not (0 <= linear_rank < self.numel):
            raise ValueError(f"Rank {linear_rank} is outside mesh with {self.numel} ranks.")
        return divmod(linear_rank, self.shape[1])

    def shifted_rank(self, coord: Tuple[int, int], axis: int, shift: int) -> int:
        if axis not in (0, 1):
            raise ValueError("axis must be 0 for rows or 1 for columns.")
        row, col = coord
        if axis == 0:
            row = (row + shift) % self.shape[0]
        else:
            col = (col + shift) % self.shape[1]
        return self.to_linear((row, col))

    def transpose_rank(self, coord: Tuple[int, int]) -> int:
        """The rank holding the transposed tile (square meshes only)."""
        if not self.is_square:
            raise ValueError("transpose_rank needs a square mesh; R x C meshes use band exchanges.")
        return self.to_linear((coord[1], coord[0]))
