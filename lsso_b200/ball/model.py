"""The LSSO token-mixer module (drop-in for lsso/ball/model.py of the reference).

Public surface kept from the reference: ``LSSO(LSSOConfig(...))``,
``forward(x, valid_mask=None, position_ids=None, *, implementation=...)`` with
``"reference"`` (PyTorch) and ``"cuda"`` (the sm_100a library), ``complement()``
and checkpoint contract 12 (model.py:21,79-140).  The CUDA implementation
never falls back to the reference one.
"""

from __future__ import annotations

import math

import torch
import torch.nn as nn

from .config import CoreMode, LSSOConfig
from .reference import (
    accretive_equilibrium_mix,
    accretive_generator,
    bounded_complement,
    qr_soft_frame,
    rank_rotary,
    tensor_core_linear,
    tensor_core_matmul,
)

_CONTRACT_VERSION = 12
_ETA_INIT_RAW = math.atanh(0.9)
_ACTIVATION_DTYPES = frozenset((torch.float16, torch.bfloat16, torch.float32, torch.float64))


class LSSO(nn.Module):
    r"""Accretive-equilibrium low-rank token mixer.

    Per head: a soft frame P of the rotated relation coordinates, the compact
    state Z = P^T C, a dynamic accretive generator K built from Z, and the
    reflected-resolvent readout Y = eta C + P [2 (I+K)^{-1} Z - (1+eta) Z].
    """

    def __init__(self, config: LSSOConfig) -> None:
        super().__init__()
        self.config = config
        width = config.num_heads * config.rank + config.dim
        self.w_bc = nn.Linear(config.dim, width, bias=config.bias)
        self.w_o = nn.Linear(config.dim, config.dim, bias=config.bias)
        heads, rank = config.num_heads, config.rank
        if config.core_mode is CoreMode.DYNAMIC:
            self.core_base_raw = nn.Parameter(torch.zeros(heads, rank, rank))
            self.core_drive_weight = nn.Parameter(torch.zeros(heads, config.head_dim, rank))
        elif config.core_mode is CoreMode.STATIC:
            self.core_base_raw = nn.Parameter(torch.zeros(heads, rank, rank))
            self.register_parameter("core_drive_weight", None)
        else:
            self.register_parameter("core_base_raw", None)
            self.register_parameter("core_drive_weight", None)
        self.eta_raw = nn.Parameter(torch.full((heads,), _ETA_INIT_RAW, dtype=torch.float32))

    # ------------------------------------------------------------------ contract
    def complement(self) -> torch.Tensor:
        """The learned per-head complement eta in (-1, 1)."""
        return bounded_complement(self.eta_raw)

    def _contract_state(self) -> dict[str, object]:
        c = self.config
        return {
            "version": _CONTRACT_VERSION,
            "operator": "accretive_equilibrium",
            "dim": c.dim,
            "num_heads": c.num_heads,
            "rank": c.rank,
            "core_mode": c.core_mode.value,
            "rank_rotary": c.rank_rotary,
            "eta_parameterization": "per_head_interior_tanh",
            "numerics": "tf32-wbc-ieee-fgram-tc16-v6",
            "bias": c.bias,
        }

    def get_extra_state(self) -> dict[str, object]:
        return self._contract_state()

    def set_extra_state(self, state: object) -> None:
        expected = self._contract_state()
        if not isinstance(state, dict):
            raise RuntimeError("LSSO checkpoint is missing its configuration contract")
        if state != expected:
            diffs = ", ".join(
                f"{key}: checkpoint={state.get(key)!r}, model={expected.get(key)!r}"
                for key in sorted(set(state) | set(expected))
                if state.get(key) != expected.get(key)
            )
            raise RuntimeError(f"incompatible LSSO checkpoint contract ({diffs})")

    def _load_from_state_dict(self, state_dict, prefix, local_metadata, strict, missing_keys, unexpected_keys,
                              error_msgs) -> None:
        key = f"{prefix}_extra_state"
        if key not in state_dict:
            error_msgs.append(f"LSSO checkpoint is missing its configuration contract ({key!r})")
        super()._load_from_state_dict(state_dict, prefix, local_metadata, strict, missing_keys, unexpected_keys,
                                      error_msgs)

    # ------------------------------------------------------------------ inputs
    @staticmethod
    def _validate_mask(valid_mask, *, batch: int, length: int, device: torch.device) -> torch.Tensor:
        if valid_mask is None:
            return torch.ones(batch, length, dtype=torch.bool, device=device)
        if valid_mask.shape != (batch, length):
            raise ValueError(f"valid_mask must have shape {(batch, length)}, got {tuple(valid_mask.shape)}")
        if valid_mask.dtype != torch.bool:
            raise TypeError(f"valid_mask must have dtype torch.bool, got {valid_mask.dtype}")
        return valid_mask.to(device=device)

    @staticmethod
    def _center_positions(position_ids, valid_mask, *, dtype: torch.dtype, all_valid: bool, batch=None, length=None,
                          device=None) -> torch.Tensor:
        """Centered Rank-Rotary coordinates ``[B, N]`` (reference model.py:163-243).

        Integer ids are differenced in int64 before float conversion; FP64 ids
        are centered in FP64.  With a mask: anchor at the first valid token,
        subtract the valid mean, zero the invalid positions.
        """
        if valid_mask is None:
            if not all_valid:
                raise ValueError("valid_mask is required when tokens are masked")
            if batch is None or length is None or device is None:
                raise ValueError("batch, length, and device are required without valid_mask")
        else:
            batch, length = valid_mask.shape
            device = valid_mask.device
        if position_ids is None:
            positions = torch.arange(length, device=device, dtype=dtype).view(1, length).expand(batch, length)
        else:
            if position_ids.is_floating_point():
                if position_ids.dtype not in (torch.float32, torch.float64):
                    raise TypeError(
                        f"floating position_ids must use torch.float32 or torch.float64, got {position_ids.dtype}"
                    )
                pdtype = torch.float64 if position_ids.dtype == torch.float64 else dtype
                positions = position_ids.to(device=device, dtype=pdtype)
            else:
                if position_ids.dtype == torch.bool or position_ids.is_complex():
                    raise TypeError(
                        "position_ids must use an integer dtype, torch.float32, or torch.float64, "
                        f"got {position_ids.dtype}"
                    )
                positions = position_ids.to(device=device, dtype=torch.int64)
            if positions.ndim == 1:
                if positions.numel() != length:
                    raise ValueError(f"position_ids length {positions.numel()} must match N={length}")
                positions = positions.view(1, length).expand(batch, length)
            elif positions.shape != (batch, length):
                raise ValueError(
                    f"position_ids must be None, [N], or [B, N]={batch, length}; got {tuple(positions.shape)}"
                )
        if all_valid:
            centered = positions - positions[:, :1]
            if centered.dtype == torch.int64:
                centered = centered.to(dtype=dtype)
            return (centered - centered.mean(dim=-1, keepdim=True)).to(dtype=dtype)
        first = valid_mask.to(dtype=torch.int64).argmax(dim=-1, keepdim=True)
        centered = positions - positions.gather(dim=1, index=first)
        if centered.dtype == torch.int64:
            centered = centered.to(dtype=dtype)
        weights = valid_mask.to(dtype=centered.dtype)
        count = weights.sum(dim=-1, keepdim=True).clamp_min(1.0)
        mean = (torch.where(valid_mask, centered, torch.zeros_like(centered)) * weights).sum(dim=-1, keepdim=True) / count
        return torch.where(valid_mask, centered - mean, torch.zeros_like(centered)).to(dtype=dtype)

    def _validate_input(self, x: torch.Tensor) -> None:
        dim = self.config.dim
        if x.ndim != 3 or x.shape[-1] != dim:
            raise ValueError(f"x must have shape [B, N, {dim}], got {tuple(x.shape)}")
        if not x.is_floating_point():
            raise TypeError("x must be a floating-point tensor")
        if x.dtype not in _ACTIVATION_DTYPES:
            raise TypeError(
                f"LSSO does not support x with dtype {x.dtype}; use torch.float16, torch.bfloat16, "
                "torch.float32, or torch.float64"
            )
        if x.shape[0] == 0:
            raise ValueError("batch size must be positive")
        if x.shape[1] == 0:
            raise ValueError("sequence length must be positive")

    # ------------------------------------------------------------------ CUDA path
    def _forward_cuda(self, x, valid_mask, position_ids) -> torch.Tensor:
        """The strict sm_100a implementation (reference model.py:270-405)."""
        c = self.config
        if c.core_mode is not CoreMode.DYNAMIC or not c.rank_rotary or c.rank not in (16, 32, 48, 64):
            raise ValueError(
                "implementation='cuda' requires core_mode='dynamic', rank_rotary=True, and rank in {16, 32, 48, 64}"
            )
        if position_ids is not None and position_ids.requires_grad:
            raise ValueError("implementation='cuda' does not support gradients for position_ids")
        if x.device.type != "cuda":
            raise ValueError("implementation='cuda' requires x to be a CUDA tensor")
        if x.dtype not in (torch.float16, torch.bfloat16):
            raise TypeError(
                f"implementation='cuda' supports x with dtype torch.float16 or torch.bfloat16; got {x.dtype}"
            )
        if self.core_base_raw is None or self.core_drive_weight is None:
            raise RuntimeError("dynamic compact parameters are missing")
        for name, parameter in self.named_parameters():
            if parameter.device != x.device:
                raise RuntimeError(f"implementation='cuda' requires {name} on {x.device}, got {parameter.device}")
        for name, parameter in (
            ("w_bc.weight", self.w_bc.weight), ("w_bc.bias", self.w_bc.bias), ("w_o.weight", self.w_o.weight),
            ("w_o.bias", self.w_o.bias), ("core_base_raw", self.core_base_raw),
            ("core_drive_weight", self.core_drive_weight), ("eta_raw", self.eta_raw),
        ):
            if parameter is None:
                continue
            if parameter.dtype != torch.float32:
                raise TypeError(f"implementation='cuda' requires {name} to use torch.float32, got {parameter.dtype}")
            if not parameter.is_contiguous():
                raise RuntimeError(f"implementation='cuda' requires contiguous {name}")

        from . import projection

        batch, length, _ = x.shape
        all_valid = valid_mask is None
        mask = None if all_valid else self._validate_mask(valid_mask, batch=batch, length=length, device=x.device)
        centered_positions = None
        if valid_mask is not None or position_ids is not None:
            centered = self._center_positions(position_ids, mask, dtype=torch.float32, all_valid=all_valid,
                                              batch=batch, length=length, device=x.device)
            if position_ids is None or position_ids.ndim == 1:
                centered_positions = centered[0].contiguous() if all_valid else centered.contiguous()
            else:
                centered_positions = centered.contiguous()
        valid_counts = None
        if not all_valid:
            valid_counts = mask.sum(dim=-1).to(dtype=torch.float32).clamp_min(1.0).contiguous()

        # One launch converts every weight image this step's GEMMs use (forward, and
        # the input-gradient products of the backward when one will run).
        wants_backward = torch.is_grad_enabled() and (
            x.requires_grad or any(p.requires_grad for p in (self.w_bc.weight, self.w_o.weight)))
        images = projection.layer_images(self.w_bc.weight, self.w_o.weight, wants_backward)
        projected = projection.input_projection(x, self.w_bc.weight, self.w_bc.bias, mask, images)
        # the mixer and the output projection as one autograd node: its backward computes the
        # output projection's weight gradient beside the mixer backward's solves
        return projection.mix_output(projected, self.core_base_raw, self.core_drive_weight, self.eta_raw,
                                     centered_positions, valid_counts, self.w_o.weight, self.w_o.bias, x.dtype, mask,
                                     images)

    # ------------------------------------------------------------------ reference path
    def _compact_coordinates(self, compact_state, valid_count):
        c = self.config
        if c.core_mode is CoreMode.DYNAMIC:
            if self.core_base_raw is None or self.core_drive_weight is None:
                raise RuntimeError("dynamic compact parameters are missing")
            drive = tensor_core_matmul(compact_state, self.core_drive_weight.to(dtype=compact_state.dtype))
            base = self.core_base_raw.to(dtype=compact_state.dtype).unsqueeze(0)
            return base + drive / valid_count.sqrt().view(-1, 1, 1, 1)
        if c.core_mode is CoreMode.STATIC:
            if self.core_base_raw is None:
                raise RuntimeError("static compact parameters are missing")
            return self.core_base_raw.to(dtype=compact_state.dtype)
        return None

    def _reference_forward(self, x, valid_mask, position_ids) -> torch.Tensor:
        """PyTorch evaluation (reference model.py:407-496,562-585)."""
        c = self.config
        batch, length, _ = x.shape
        all_valid = valid_mask is None
        mask = None if all_valid else self._validate_mask(valid_mask, batch=batch, length=length, device=x.device)
        safe_x = x if all_valid else torch.where(mask[:, :, None], x, torch.zeros_like(x))
        wide = torch.float64 if x.dtype == torch.float64 else torch.bfloat16
        projected = tensor_core_linear(safe_x, self.w_bc.weight, self.w_bc.bias, output_dtype=wide)
        relation, content = projected.split((c.num_heads * c.rank, c.dim), dim=-1)
        relation = relation.view(batch, length, c.num_heads, c.rank).transpose(1, 2)
        content = content.view(batch, length, c.num_heads, c.head_dim).transpose(1, 2)
        if not all_valid:
            active = mask[:, None, :, None]
            relation = torch.where(active, relation, torch.zeros_like(relation))
            content = torch.where(active, content, torch.zeros_like(content))
        calc = torch.float64 if x.dtype == torch.float64 else torch.float32
        with torch.autocast(device_type=x.device.type, enabled=False):
            relation = relation.to(calc)
            content = content.to(calc)
            if c.rank_rotary:
                centered = self._center_positions(position_ids, mask, dtype=calc, all_valid=all_valid, batch=batch,
                                                  length=length, device=x.device)
                relation = rank_rotary(relation, centered)
            if all_valid:
                count = torch.full((batch,), float(length), dtype=calc, device=x.device)
            else:
                count = mask.sum(dim=-1).to(calc).clamp_min(1.0)
            relation = relation / count.sqrt().view(batch, 1, 1, 1)
            frame = qr_soft_frame(relation)
            state = tensor_core_matmul(frame.mT, content)
            coords = self._compact_coordinates(state, count)
            generator = None if coords is None else accretive_generator(coords)
            eta = self.complement().to(device=x.device, dtype=calc)
            mixed = accretive_equilibrium_mix(frame, generator, state, content, eta)
        if x.dtype != torch.float64:
            mixed = mixed.to(torch.bfloat16)
        mixed = mixed.transpose(1, 2).contiguous().view(batch, length, c.dim)
        out = tensor_core_linear(mixed, self.w_o.weight, self.w_o.bias, output_dtype=x.dtype)
        if mask is None:
            return out
        return torch.where(mask[:, :, None], out, torch.zeros_like(out))

    def forward(self, x, valid_mask=None, position_ids=None, *, implementation: str = "reference") -> torch.Tensor:
        self._validate_input(x)
        if implementation == "cuda":
            return self._forward_cuda(x, valid_mask, position_ids)
        if implementation != "reference":
            raise ValueError(f"implementation must be 'reference' or 'cuda', got {implementation!r}")
        return self._reference_forward(x, valid_mask, position_ids)

    def extra_repr(self) -> str:
        c = self.config
        return (
            f"dim={c.dim}, num_heads={c.num_heads}, rank={c.rank}, core_mode={c.core_mode.value}, "
            f"rank_rotary={c.rank_rotary}, eta=per-head-interior-tanh"
        )


__all__ = ["LSSO"]
