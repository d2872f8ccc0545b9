"""The LSSO mixer module, its configuration and its CUDA boundary."""

from .config import CoreMode, LSSOConfig
from .model import LSSO

__all__ = ["CoreMode", "LSSO", "LSSOConfig"]
