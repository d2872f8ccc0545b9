"""End-to-end drivers of the mixer: a sequence-model shell and vision position IDs.

``SequenceShell`` stacks pre-LayerNorm residual blocks around ``LSSO`` the way
the reference's experiment encoder does (experiments/train_transformers.py:
479-556, ``SequenceBlock``): ``x + mixer(norm1(x))`` with the normalised
activations cast to the autocast dtype before the mixer, padded tokens zeroed
after each residual, and an optional ``x + mlp(norm2(x))`` (``mlp_ratio=0``
leaves it out, as BASELINE config 4 does).  Tokens enter through an
``Embedding`` initialised N(0, 0.02).

``vision_position_ids`` is the timm adapter's position rule
(integrations/timm.py:143-156): position 0 for the class token and centered
one-dimensional coordinates for the patches.
"""

from __future__ import annotations

import torch
from torch import nn

from .config import LSSOConfig
from .model import LSSO


def vision_position_ids(length: int, device: torch.device | None = None) -> torch.Tensor:
    """FP32 [length]: 0 for the class token, then p - (length - 2)/2 for patch p."""
    if length <= 0:
        return torch.empty(0, device=device, dtype=torch.float32)
    patches = torch.arange(length - 1, device=device, dtype=torch.float32)
    patches -= 0.5 * (length - 2)
    return torch.cat((torch.zeros(1, device=device, dtype=torch.float32), patches))


class ShellBlock(nn.Module):
    """Pre-norm residual block: x + LSSO(norm(x)), padded tokens zero (optional MLP)."""

    def __init__(self, config: LSSOConfig, *, mlp_ratio: float = 0.0) -> None:
        super().__init__()
        self.norm1 = nn.LayerNorm(config.dim)
        self.mixer = LSSO(config)
        self.mlp = None
        if mlp_ratio > 0:
            hidden = int(round(config.dim * mlp_ratio))
            self.norm2 = nn.LayerNorm(config.dim)
            self.mlp = nn.Sequential(nn.Linear(config.dim, hidden, bias=config.bias), nn.GELU(),
                                     nn.Linear(hidden, config.dim, bias=config.bias))

    def forward(self, x: torch.Tensor, valid_mask: torch.Tensor | None, implementation: str) -> torch.Tensor:
        normalized = self.norm1(x)
        if normalized.device.type == "cuda" and torch.is_autocast_enabled():
            amp = torch.get_autocast_dtype("cuda")
            if implementation == "cuda" and amp not in (torch.float16, torch.bfloat16):
                raise TypeError("the CUDA LSSO sequence path supports FP16 or BF16 AMP")
            normalized = normalized.to(dtype=amp)
        x = x + self.mixer(normalized, valid_mask=valid_mask, implementation=implementation)
        if valid_mask is not None:
            x = torch.where(valid_mask[:, :, None], x, torch.zeros_like(x))
        if self.mlp is not None:
            x = x + self.mlp(self.norm2(x))
            if valid_mask is not None:
                x = torch.where(valid_mask[:, :, None], x, torch.zeros_like(x))
        return x


class SequenceShell(nn.Module):
    """Token embedding plus ``depth`` pre-norm LSSO blocks (dim 128, 4 heads,
    rank 48, depth 4, vocabulary 8, no MLP)."""

    def __init__(self, config: LSSOConfig, *, depth: int = 4, vocab: int = 8, mlp_ratio: float = 0.0) -> None:
        super().__init__()
        self.embedding = nn.Embedding(vocab, config.dim)
        nn.init.normal_(self.embedding.weight, mean=0.0, std=0.02)
        self.blocks = nn.ModuleList(ShellBlock(config, mlp_ratio=mlp_ratio) for _ in range(depth))

    def forward(self, token_ids: torch.Tensor, valid_mask: torch.Tensor | None = None, *,
                implementation: str = "reference") -> torch.Tensor:
        x = self.embedding(token_ids)
        if valid_mask is not None:
            x = torch.where(valid_mask[:, :, None], x, torch.zeros_like(x))
        for block in self.blocks:
            x = block(x, valid_mask, implementation)
        return x


__all__ = ["SequenceShell", "ShellBlock", "vision_position_ids"]
