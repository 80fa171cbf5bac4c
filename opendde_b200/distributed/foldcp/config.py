"""Fold-CP launch configuration (drop-in for opendde/distributed/foldcp/config.py:18-140).

Same environment keys, constructor and validation messages as the reference, plus one
extension: the CP mesh may be any R x C grid, not only a square one. The grid comes from
``OPENDDE_FOLDCP_MESH="RxC"`` (or the ``mesh`` argument); without it a perfect-square
``size_cp`` keeps the reference's square mesh and any other ``size_cp`` gets the most
square R x C with R <= C (2 -> 1x2, 8 -> 2x4).
"""

from __future__ import annotations

import math
import os
from dataclasses import asdict, dataclass
from typing import Any, Literal, Tuple

FoldCPMode = Literal["single", "distributed"]
FOLDCP_ENVIRONMENT_KEYS = (
    "OPENDDE_FOLDCP_MODE",
    "OPENDDE_FOLDCP_SIZE_DP",
    "OPENDDE_FOLDCP_SIZE_CP",
    "OPENDDE_FOLDCP_DEVICES",
    "OPENDDE_FOLDCP_METRICS_JSONL",
)
FOLDCP_MESH_KEY = "OPENDDE_FOLDCP_MESH"


def _as_int(value: Any, default: int) -> int:
    if value is None or value == "":
        return default
    return int(value)


def parse_mesh(text: str) -> Tuple[int, int]:
    """'RxC' -> (R, C)."""
    try:
        r, c = text.lower().replace(" ", "").split("x")
        return int(r), int(c)
    except ValueError:
        raise ValueError(f"foldcp mesh must look like 'RxC', got {text!r}") from None


def default_mesh_shape(size_cp: int) -> Tuple[int, int]:
    """Square when size_cp is a perfect square, else the most square R x C with R <= C."""
    r = math.isqrt(size_cp)
    while size_cp % r:
        r -= 1
    return r, size_cp // r


@dataclass(frozen=True)
class FoldCPConfig:
    """Validated Fold-CP launch configuration (config.py:34-118)."""

    mode: FoldCPMode = "single"
    size_dp: int = 1
    size_cp: int = 1
    devices: str = ""
    metrics_jsonl: str = ""
    mesh: str = ""

    @classmethod
    def from_runtime_args(cls, *, mode: str = "single", size_dp: int = 1, size_cp: int = 1,
                          devices: str = "", metrics_jsonl: str = "", mesh: str = "") -> "FoldCPConfig":
        return cls(mode=mode, size_dp=int(size_dp), size_cp=int(size_cp), devices=devices,  # type: ignore[arg-type]
                   metrics_jsonl=metrics_jsonl, mesh=mesh).validate()

    @classmethod
    def from_config(cls, configs: Any) -> "FoldCPConfig":
        return cls.from_runtime_args(
            mode=getattr(configs, "foldcp_mode", "single"),
            size_dp=_as_int(getattr(configs, "foldcp_size_dp", 1), 1),
            size_cp=_as_int(getattr(configs, "foldcp_size_cp", 1), 1),
            devices=getattr(configs, "foldcp_devices", "") or "",
            metrics_jsonl=getattr(configs, "foldcp_metrics_jsonl", "") or "",
            mesh=getattr(configs, "foldcp_mesh", "") or "",
        )

    @classmethod
    def from_env(cls, world_size: int | None = None) -> "FoldCPConfig":
        """The configuration the launcher exported (``OPENDDE_FOLDCP_*``).

        ``size_cp`` defaults to ``world_size // size_dp`` when it is not set.
        """
        size_dp = _as_int(os.environ.get("OPENDDE_FOLDCP_SIZE_DP"), 1)
        default_cp = (world_size // size_dp) if world_size else 1
        return cls.from_runtime_args(
            mode=os.environ.get("OPENDDE_FOLDCP_MODE", "single") or "single",
            size_dp=size_dp,
            size_cp=_as_int(os.environ.get("OPENDDE_FOLDCP_SIZE_CP"), default_cp),
            devices=os.environ.get("OPENDDE_FOLDCP_DEVICES", ""),
            metrics_jsonl=os.environ.get("OPENDDE_FOLDCP_METRICS_JSONL", ""),
            mesh=os.environ.get(FOLDCP_MESH_KEY, ""),
        )

    def validate(self) -> "FoldCPConfig":
        if self.mode not in {"single", "distributed"}:
            raise ValueError("foldcp_mode must be 'single' or 'distributed'.")
        if self.size_dp < 1:
            raise ValueError("foldcp_size_dp must be >= 1.")
        if self.size_cp < 1:
            raise ValueError("foldcp_size_cp must be >= 1.")
        if self.mode == "single" and self.size_cp != 1:
            raise ValueError("foldcp_mode='single' requires foldcp_size_cp=1.")
        if self.mode == "distributed":
            if self.size_cp == 1:
                raise ValueError("foldcp_mode='distributed' requires foldcp_size_cp > 1.")
            r, c = self.cp_mesh_shape
            if r < 1 or c < 1 or r * c != self.size_cp:
                raise ValueError(f"foldcp mesh {r}x{c} does not hold foldcp_size_cp={self.size_cp} ranks.")
        return self

    @property
    def enabled(self) -> bool:
        return self.mode == "distributed"

    @property
    def cp_mesh_shape(self) -> Tuple[int, int]:
        if self.mesh:
            return parse_mesh(self.mesh)
        return default_mesh_shape(self.size_cp)

    def to_dict(self) -> dict[str, Any]:
        data = asdict(self)
        data["enabled"] = self.enabled
        data["cp_mesh_shape"] = self.cp_mesh_shape
        return data

    def launch_hint(self) -> str:
        if self.enabled:
            nproc = self.size_dp * self.size_cp
            r, c = self.cp_mesh_shape
            return (f"OPENDDE_FOLDCP_MESH={r}x{c} torchrun --nproc_per_node {nproc} -m runner.batch_inference "
                    f"pred --foldcp_mode distributed --foldcp_size_dp {self.size_dp} --foldcp_size_cp {self.size_cp}")
        return "python -m runner.batch_inference pred --foldcp_mode single --foldcp_size_cp 1"


def apply_foldcp_config(configs: Any, foldcp: FoldCPConfig) -> Any:
    """Export the settings to the environment and attach them to a mutable config object."""
    values = (foldcp.mode, str(foldcp.size_dp), str(foldcp.size_cp), foldcp.devices, foldcp.metrics_jsonl)
    for key, value in zip(FOLDCP_ENVIRONMENT_KEYS, values, strict=True):
        os.environ[key] = value
    if foldcp.mesh:
        os.environ[FOLDCP_MESH_KEY] = foldcp.mesh
    configs.foldcp_mode = foldcp.mode
    configs.foldcp_size_dp = foldcp.size_dp
    configs.foldcp_size_cp = foldcp.size_cp
    configs.foldcp_devices = foldcp.devices
    configs.foldcp_metrics_jsonl = foldcp.metrics_jsonl
    configs.foldcp_mesh = foldcp.mesh
    configs.foldcp = foldcp.to_dict()
    return configs
