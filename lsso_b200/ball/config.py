"""Operator configuration (mirrors lsso/ball/config.py:15-66 of the reference)."""

from __future__ import annotations

from dataclasses import dataclass
from enum import Enum


class CoreMode(str, Enum):
    """Compact-core modes of the LSSO operator."""

    DYNAMIC = "dynamic"
    STATIC = "static"
    ZERO = "zero"


def _require_int(name: str, value: object) -> None:
    # bool is an int subclass and is rejected explicitly.
    if isinstance(value, bool) or not isinstance(value, int):
        raise TypeError(f"{name} must be an integer, got {type(value).__name__}")


def _require_bool(name: str, value: object) -> None:
    if not isinstance(value, bool):
        raise TypeError(f"{name} must be a bool, got {type(value).__name__}")


@dataclass(frozen=True, slots=True)
class LSSOConfig:
    """Sizes and switches of one LSSO mixer.

    ``dim`` is the model width D, ``num_heads`` H, ``rank`` r; the head width
    is ``dim // num_heads``.  ``core_mode`` and ``rank_rotary`` select the
    ablations; the CUDA path implements DYNAMIC with Rank-Rotary.
    """

    dim: int
    num_heads: int
    rank: int = 16
    core_mode: CoreMode = CoreMode.DYNAMIC
    rank_rotary: bool = True
    bias: bool = False

    def __post_init__(self) -> None:
        _require_int("dim", self.dim)
        _require_int("num_heads", self.num_heads)
        _require_int("rank", self.rank)
        try:
            mode = CoreMode(self.core_mode)
        except (TypeError, ValueError) as error:
            allowed = ", ".join(m.value for m in CoreMode)
            raise ValueError(f"core_mode must be one of {{{allowed}}}, got {self.core_mode!r}") from error
        object.__setattr__(self, "core_mode", mode)
        _require_bool("rank_rotary", self.rank_rotary)
        _require_bool("bias", self.bias)
        if min(self.dim, self.num_heads, self.rank) <= 0:
            raise ValueError("dim, num_heads, and rank must be positive")
        if self.dim % self.num_heads != 0:
            raise ValueError(f"dim={self.dim} must be divisible by num_heads={self.num_heads}")
        if self.rank_rotary and self.rank % 2 != 0:
            raise ValueError(f"Rank-Rotary requires an even rank, got rank={self.rank}")

    @property
    def head_dim(self) -> int:
        return self.dim // self.num_heads


__all__ = ["CoreMode", "LSSOConfig"]
