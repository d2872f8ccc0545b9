"""Sequence-parallel LSSO layer: the tokens of each sample split over a process group.

The mixer's only cross-token quantities are, per (sample, head), the moment
sums the solves start from: the Gram and content moments of the forward
(reference lsso/ball/reference.py:411-447, 500-572) and ``A'^T dY`` of the
backward.  Everything else is per token.  So a sequence longer than one GPU
holds can be split into contiguous slices, one per rank (rank order = token
order), and each pass needs exactly one collective: each rank runs the moment
pass over its own tokens (``lsso_forward_moments`` / ``lsso_backward_moments``),
one ``all_reduce(SUM)`` of the small moment buffer (``B*H*2r*(r+d)`` floats,
about 1 MB at B=64, H=8, r=d=32), then every rank runs the same solves and the
readout / gradient pass of its own tokens (``lsso_forward_finish`` /
``lsso_backward_finish``).

Positions are those of the whole sequence: the centered positions and the
valid-token counts are computed from every rank's ``position_ids`` /
``valid_mask`` (gathered, then centered exactly as ``LSSO._center_positions``
does for the unsplit sequence), and each rank keeps its own slice.

Parameter gradients: the projections' and the per-token parts are this rank's
share, and the solve-computed terms (all of ``core_base_raw`` and
``core_drive_weight``'s gradients, the solve's part of ``eta_raw``'s) are
counted on the group's rank 0 only, so the caller SUMS every parameter
gradient over the group (``allreduce_gradients(..., average=False)``), as for
any loss that adds up over the split tokens.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from . import _native


class _SequenceMix(torch.autograd.Function):
    @staticmethod
    def forward(ctx, projected, core_base_raw, core_drive_weight, eta_raw, positions, counts, group, redundant):
        moments = _native.forward_moments(projected, core_base_raw, core_drive_weight, eta_raw, positions)
        dist.all_reduce(moments, op=dist.ReduceOp.SUM, group=group)
        mixed, tape, _ = _native.forward_finish(projected, core_base_raw, core_drive_weight, eta_raw, positions,
                                                counts, moments, train=True)
        ctx.save_for_backward(projected, core_base_raw, core_drive_weight, eta_raw, tape, positions)
        ctx.group = group
        ctx.redundant = redundant
        return mixed

    @staticmethod
    @torch.autograd.function.once_differentiable
    def backward(ctx, grad_mixed):
        projected, core_base_raw, core_drive_weight, eta_raw, tape, positions = ctx.saved_tensors
        grad = grad_mixed.contiguous()
        moments = _native.backward_moments(grad, projected, core_base_raw, core_drive_weight, eta_raw, positions)
        dist.all_reduce(moments, op=dist.ReduceOp.SUM, group=ctx.group)
        grads = _native.backward_finish(grad, projected, core_base_raw, core_drive_weight, eta_raw, tape, positions,
                                        moments, ctx.redundant)
        return (*grads, None, None, None, None)


def sequence_mix(projected, core_base_raw, core_drive_weight, eta_raw, positions, counts, *, group=None):
    """The native mixer over a sequence split across ``group`` (this rank's tokens in ``projected``).

    ``positions``: FP32 [N_local] or [B, N_local] centered positions of this
    rank's tokens within the whole sequence; ``counts``: FP32 [B] valid tokens
    of the whole sequence (at least 1).
    """
    redundant = 1.0 if dist.get_rank(group) == 0 else 0.0
    if torch.is_grad_enabled() and any(
            v.requires_grad for v in (projected, core_base_raw, core_drive_weight, eta_raw)):
        return _SequenceMix.apply(projected, core_base_raw, core_drive_weight, eta_raw, positions, counts, group,
                                  redundant)
    moments = _native.forward_moments(projected, core_base_raw, core_drive_weight, eta_raw, positions)
    dist.all_reduce(moments, op=dist.ReduceOp.SUM, group=group)
    mixed, _, _ = _native.forward_finish(projected, core_base_raw, core_drive_weight, eta_raw, positions, counts,
                                         moments, train=False)
    return mixed


def _gather_tokens(value: torch.Tensor, lengths: list[int], group) -> torch.Tensor:
    """Concatenate every rank's [B, n_r] slice along the token axis (rank order)."""
    longest = max(lengths)
    padded = value.new_zeros((value.shape[0], longest))
    padded[:, :value.shape[1]] = value
    parts = [torch.empty_like(padded) for _ in lengths]
    dist.all_gather(parts, padded.contiguous(), group=group)
    return torch.cat([p[:, :n] for p, n in zip(parts, lengths)], dim=1)


def sequence_positions(batch: int, length: int, valid_mask, position_ids, *, group=None, device=None):
    """Centered positions ([N_local] or [B, N_local], FP32) and valid counts ([B]) of this
    rank's slice, computed over the whole sequence split across ``group``.

    Returns ``(positions, counts, offset, total)``: ``offset`` is the slice's
    first token and ``total`` the sequence length.
    """
    from .model import LSSO

    device = device if device is not None else torch.device("cuda", torch.cuda.current_device())
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    n_local = torch.tensor([length], dtype=torch.int64, device=device)
    everyone = [torch.empty_like(n_local) for _ in range(world)]
    dist.all_gather(everyone, n_local, group=group)
    lengths = [int(v.item()) for v in everyone]
    offset, total = sum(lengths[:rank]), sum(lengths)
    if valid_mask is None and position_ids is None:
        # t - (N - 1)/2 over the whole sequence, in FP32 as the kernels' default.
        positions = (torch.arange(offset, offset + length, dtype=torch.float32, device=device)
                     - torch.tensor(0.5 * (total - 1), dtype=torch.float32, device=device))
        counts = torch.full((batch,), float(total), dtype=torch.float32, device=device)
        return positions.contiguous(), counts, offset, total
    all_valid = valid_mask is None
    mask = None
    if not all_valid:
        mask = LSSO._validate_mask(valid_mask, batch=batch, length=length, device=device)
        mask = _gather_tokens(mask.to(torch.uint8), lengths, group).bool()
    ids = None
    if position_ids is not None:
        ids = position_ids.to(device)
        shared = ids.dim() == 1
        ids2 = ids.unsqueeze(0) if shared else ids
        gathered = _gather_tokens(ids2.to(torch.float64) if ids2.is_floating_point() else ids2, lengths, group)
        ids = gathered.to(position_ids.dtype)
        ids = ids[0] if shared else ids
    centered = LSSO._center_positions(ids, mask, dtype=torch.float32, all_valid=all_valid, batch=batch,
                                      length=total, device=device)
    if position_ids is None or position_ids.dim() == 1:
        full = centered[0] if all_valid else centered
    else:
        full = centered
    positions = (full[..., offset:offset + length]).contiguous()
    if all_valid:
        counts = torch.full((batch,), float(total), dtype=torch.float32, device=device)
    else:
        counts = mask.sum(dim=-1).to(torch.float32).clamp_min(1.0).contiguous()
    return positions, counts, offset, total


def sequence_parallel_forward(layer, x, valid_mask=None, position_ids=None, *, group=None):
    """``layer(x, valid_mask, position_ids, implementation="cuda")`` for this rank's slice.

    ``x`` [B, N_local, D] (FP16 / BF16) holds this rank's contiguous slice of
    every sample's tokens, slices in rank order; ``valid_mask`` [B, N_local]
    and ``position_ids`` ([N_local] or [B, N_local]) are this rank's slices of
    the whole sequence's.  Returns this rank's slice of the output.  Sum the
    parameter gradients over ``group`` after the backward.
    """
    from . import projection

    c = layer.config
    if x.device.type != "cuda" or x.dtype not in (torch.float16, torch.bfloat16):
        raise ValueError("the sequence-parallel layer takes FP16 or BF16 CUDA activations")
    if c.rank not in (16, 32, 48, 64) or not c.rank_rotary or layer.core_base_raw is None:
        raise ValueError("the sequence-parallel layer requires the DYNAMIC Rank-Rotary mixer with rank in "
                         "{16, 32, 48, 64}")
    batch, length, _ = x.shape
    positions, counts, _, _ = sequence_positions(batch, length, valid_mask, position_ids, group=group,
                                                 device=x.device)
    mask = None
    if valid_mask is not None:
        mask = layer._validate_mask(valid_mask, batch=batch, length=length, device=x.device)
    projected = projection.input_projection(x, layer.w_bc.weight, layer.w_bc.bias, mask)
    mixed = sequence_mix(projected, layer.core_base_raw, layer.core_drive_weight, layer.eta_raw, positions, counts,
                         group=group)
    return projection.output_projection(mixed, layer.w_o.weight, layer.w_o.bias, x.dtype, mask)


__all__ = ["sequence_mix", "sequence_parallel_forward", "sequence_positions"]
