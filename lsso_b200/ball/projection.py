"""Input and output projections of the CUDA path (reference model.py:370-404).

Input projection: ``projected = bf16(x) bf16(W_bc)^T (+ FP32 bias)`` rounded
once to BF16, masked rows zeroed before and after.  Output projection:
``y = bf16(mixed) bf16(W_o)^T (+ FP32 bias)`` stored in ``x.dtype``, masked
rows zeroed.  Both use BF16 multiplicands with FP32 accumulation and the
first-order VJP of the reference's ``_TensorCoreLinear`` (reference.py:170-247).
"""

from __future__ import annotations

import torch

from .reference import tensor_core_linear


def _masked(value: torch.Tensor, mask: torch.Tensor | None) -> torch.Tensor:
    if mask is None:
        return value
    return torch.where(mask[:, :, None], value, torch.zeros_like(value))


def input_projection(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None,
                     mask: torch.Tensor | None) -> torch.Tensor:
    projected = _masked(tensor_core_linear(_masked(x, mask), weight, bias, output_dtype=torch.bfloat16), mask)
    if not projected.is_contiguous():
        raise RuntimeError("implementation='cuda' requires w_bc to produce contiguous projected coordinates")
    return projected


def output_projection(mixed: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None,
                      dtype: torch.dtype, mask: torch.Tensor | None) -> torch.Tensor:
    return _masked(tensor_core_linear(mixed, weight, bias, output_dtype=dtype), mask)


__all__ = ["input_projection", "output_projection"]
