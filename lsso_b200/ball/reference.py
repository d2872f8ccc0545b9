"""PyTorch statement of the LSSO operator (the module's ``implementation="reference"``).

Restates lsso/ball/reference.py of the reference project: the QR soft frame
(:411-447), the bounded complement (:450-471), the accretive generator
(:474-497), the direct equilibrium (:500-572), Rank-Rotary (:691-724) and the
BF16 tensor-core projection contract (:170-247, :347-408).  On CPU every
product is FP32 (or FP64); on CUDA low-precision products use BF16
multiplicands with FP32 accumulation.  This path is an explicit
implementation choice of the module, never a fallback of the CUDA path.
"""

from __future__ import annotations

from contextlib import contextmanager
import math

import torch
import torch.nn.functional as F
from torch.autograd.function import once_differentiable

RANK_PHASE_BASE = 10000.0
SOFTPLUS_ONE_OFFSET = math.log(math.expm1(1.0))


def _calc_dtype(value: torch.Tensor) -> torch.dtype:
    return torch.float64 if value.dtype == torch.float64 else torch.float32


@contextmanager
def _strict_bf16_gemm():
    """FP32 accumulation for BF16 GEMMs regardless of ambient AMP settings."""
    matmul = torch.backends.cuda.matmul
    previous = matmul.allow_bf16_reduced_precision_reduction
    matmul.allow_bf16_reduced_precision_reduction = False
    try:
        with torch.autocast(device_type="cuda", enabled=False):
            yield
    finally:
        matmul.allow_bf16_reduced_precision_reduction = previous


def _gemm(left: torch.Tensor, right: torch.Tensor, bias: torch.Tensor | None, out_dtype: torch.dtype) -> torch.Tensor:
    """left @ right (+ bias) with BF16 operands and FP32 accumulation on CUDA.

    A low-precision output with a bias is produced from the FP32 sum with a
    single final rounding (the fused-bias contract of reference.py:58-97).
    """
    with _strict_bf16_gemm():
        if bias is not None:
            full = torch.addmm(bias.to(torch.float32), left, right, out_dtype=torch.float32)
            return full if out_dtype == torch.float32 else full.to(out_dtype)
        if out_dtype == torch.bfloat16:
            return torch.mm(left, right) if left.ndim == 2 else torch.bmm(left, right)
        op = torch.mm if left.ndim == 2 else torch.bmm
        full = op(left, right, out_dtype=torch.float32)
        return full if out_dtype == torch.float32 else full.to(out_dtype)


class _BF16Linear(torch.autograd.Function):
    """y = bf16(x) bf16(W)^T (+ b) with FP32 accumulation and a dtype-aware store."""

    @staticmethod
    def forward(ctx, value, weight, bias, output_dtype):
        x = value.to(torch.bfloat16)
        w = weight.to(torch.bfloat16)
        ctx.save_for_backward(x, w)
        ctx.value_shape = value.shape
        ctx.value_dtype = value.dtype
        ctx.weight_dtype = weight.dtype
        ctx.bias_meta = None if bias is None else (bias.dtype, bias.device)
        direct = output_dtype in (torch.float16, torch.bfloat16) and (bias is not None or output_dtype == torch.bfloat16)
        store = output_dtype if direct else torch.float32
        b = None if bias is None else bias.to(device=value.device, dtype=torch.float32)
        out = _gemm(x.reshape(-1, x.shape[-1]), w.mT, b, store).reshape(*value.shape[:-1], weight.shape[0])
        return out if output_dtype is None else out.to(output_dtype)

    @staticmethod
    @once_differentiable
    def backward(ctx, grad_output):
        x, w = ctx.saved_tensors
        g = grad_output.to(torch.bfloat16).reshape(-1, w.shape[0])
        grad_value = grad_weight = grad_bias = None
        if ctx.needs_input_grad[0]:
            store = torch.bfloat16 if ctx.value_dtype == torch.bfloat16 else torch.float32
            grad_value = _gemm(g, w, None, store).reshape(ctx.value_shape).to(ctx.value_dtype)
        if ctx.needs_input_grad[1]:
            grad_weight = _gemm(g.mT, x.reshape(-1, x.shape[-1]), None, torch.float32).to(ctx.weight_dtype)
        if ctx.bias_meta is not None and ctx.needs_input_grad[2]:
            dims = tuple(range(grad_output.ndim - 1))
            total = grad_output.sum(dim=dims, dtype=torch.float32) if dims else grad_output.to(torch.float32)
            grad_bias = total.to(device=ctx.bias_meta[1], dtype=ctx.bias_meta[0])
        return grad_value, grad_weight, grad_bias, None


class _BF16Matmul(torch.autograd.Function):
    """Batched BF16 tensor-core product with FP32 result and first-order VJP."""

    @staticmethod
    def forward(ctx, left, right):
        batch = torch.broadcast_shapes(left.shape[:-2], right.shape[:-2])
        m, k, n = left.shape[-2], left.shape[-1], right.shape[-1]
        lb = left.to(torch.bfloat16).expand(batch + (m, k)).reshape(-1, m, k)
        rb = right.to(torch.bfloat16).expand(batch + (k, n)).reshape(-1, k, n)
        ctx.save_for_backward(left, right)
        ctx.meta = (batch, m, k, n)
        return _gemm(lb, rb, None, torch.float32).reshape(batch + (m, n))

    @staticmethod
    @once_differentiable
    def backward(ctx, grad_output):
        left, right = ctx.saved_tensors
        batch, m, k, n = ctx.meta
        lb = left.to(torch.bfloat16).expand(batch + (m, k)).reshape(-1, m, k)
        rb = right.to(torch.bfloat16).expand(batch + (k, n)).reshape(-1, k, n)
        g = grad_output.to(torch.bfloat16).reshape(-1, m, n)
        gl = gr = None
        if ctx.needs_input_grad[0]:
            gl = _gemm(g, rb.mT, None, torch.float32).reshape(batch + (m, k)).sum_to_size(*left.shape).to(left.dtype)
        if ctx.needs_input_grad[1]:
            gr = _gemm(lb.mT, g, None, torch.float32).reshape(batch + (k, n)).sum_to_size(*right.shape).to(right.dtype)
        return gl, gr


def tensor_core_matmul(left: torch.Tensor, right: torch.Tensor) -> torch.Tensor:
    """Matrix product under the BF16-multiplicand / FP32-accumulation contract.

    FP64 operands multiply in FP64 (the oracle); CPU operands in FP32.
    """
    if left.ndim < 2 or right.ndim < 2:
        raise ValueError("tensor_core_matmul requires matrix dimensions")
    if not left.is_floating_point() or not right.is_floating_point():
        raise TypeError("tensor_core_matmul requires floating-point inputs")
    if left.device != right.device:
        raise ValueError("tensor_core_matmul inputs must share a device")
    if left.shape[-1] != right.shape[-2]:
        raise ValueError(
            f"tensor_core_matmul inner dimensions must agree, got {left.shape[-1]} and {right.shape[-2]}"
        )
    if torch.float64 in (left.dtype, right.dtype):
        return torch.matmul(left.to(torch.float64), right.to(torch.float64))
    if left.device.type != "cuda":
        return torch.matmul(left.to(torch.float32), right.to(torch.float32))
    return _BF16Matmul.apply(left, right)


def tensor_core_linear(
    value: torch.Tensor,
    weight: torch.Tensor,
    bias: torch.Tensor | None = None,
    *,
    output_dtype: torch.dtype | None = None,
) -> torch.Tensor:
    """value @ weight^T (+ bias) with FP32 accumulation and an optional final cast."""
    if value.ndim < 1:
        raise ValueError("tensor_core_linear requires a feature dimension")
    if weight.ndim != 2:
        raise ValueError("tensor_core_linear weight must have shape [out, in]")
    if value.shape[-1] != weight.shape[-1]:
        raise ValueError(
            f"tensor_core_linear input and weight features must agree, got {value.shape[-1]} and {weight.shape[-1]}"
        )
    if not value.is_floating_point() or not weight.is_floating_point():
        raise TypeError("tensor_core_linear requires floating-point inputs")
    if value.device != weight.device:
        raise ValueError("tensor_core_linear value and weight must share a device")
    if bias is not None and bias.shape != (weight.shape[0],):
        raise ValueError(f"tensor_core_linear bias must have shape [{weight.shape[0]}], got {tuple(bias.shape)}")
    if value.device.type == "cuda" and torch.float64 not in (value.dtype, weight.dtype):
        return _BF16Linear.apply(value, weight, bias, output_dtype)
    out = tensor_core_matmul(value, weight.mT)
    if bias is not None:
        out = out + bias.to(device=out.device, dtype=out.dtype)
    return out if output_dtype is None else out.to(output_dtype)


def qr_soft_frame(relation: torch.Tensor) -> torch.Tensor:
    """Top block of Q in QR([A/s; I/s]), s = max(1, max|A|) detached, diag(R) > 0."""
    if relation.ndim < 2:
        raise ValueError("relation must have at least two matrix dimensions")
    if not relation.is_floating_point():
        raise TypeError("relation must be a floating-point tensor")
    dtype = _calc_dtype(relation)
    with torch.autocast(device_type=relation.device.type, enabled=False):
        a = relation.to(dtype)
        length, rank = a.shape[-2:]
        if length == 0 or rank == 0:
            return a
        scale = a.abs().amax(dim=(-2, -1), keepdim=True).clamp_min(1.0).detach()
        eye = torch.eye(rank, dtype=dtype, device=a.device).expand(a.shape[:-2] + (rank, rank))
        q, r = torch.linalg.qr(torch.cat((a / scale, eye / scale), dim=-2), mode="reduced")
        signs = torch.where(torch.diagonal(r, dim1=-2, dim2=-1) < 0, -1.0, 1.0).to(dtype).detach()
        return (q * signs.unsqueeze(-2))[..., :length, :]


def bounded_complement(raw: torch.Tensor) -> torch.Tensor:
    """(1 - eps) tanh(raw) through the stable logistic identity of each sign."""
    if not raw.is_floating_point():
        raise TypeError("complement coordinates must be a floating-point tensor")
    dtype = _calc_dtype(raw)
    with torch.autocast(device_type=raw.device.type, enabled=False):
        x = raw.to(dtype)
        inner = 1.0 - torch.finfo(dtype).eps
        p = torch.exp(-2.0 * torch.clamp_min(x, 0.0))
        q = torch.exp(2.0 * torch.clamp_max(x, 0.0))
        return inner * torch.where(x >= 0.0, (1.0 - p) / (1.0 + p), (q - 1.0) / (1.0 + q))


class _IEEEFactorGram(torch.autograd.Function):
    """F F^T with full FP32 products on CUDA, and its first-order VJP."""

    @staticmethod
    def forward(ctx, factor):
        f = factor.to(torch.float32)
        ctx.save_for_backward(f)
        ctx.dtype = factor.dtype
        with torch.autocast(device_type=factor.device.type, enabled=False), _ieee(factor.device):
            return torch.matmul(f, f.mT)

    @staticmethod
    @once_differentiable
    def backward(ctx, grad):
        (f,) = ctx.saved_tensors
        with torch.autocast(device_type=f.device.type, enabled=False), _ieee(f.device):
            g = grad.to(torch.float32)
            return torch.matmul(g + g.mT, f).to(ctx.dtype)


@contextmanager
def _ieee(device: torch.device):
    if device.type != "cuda":
        yield
        return
    matmul = torch.backends.cuda.matmul
    previous = matmul.fp32_precision
    matmul.fp32_precision = "ieee"
    try:
        yield
    finally:
        matmul.fp32_precision = previous


def accretive_generator(raw: torch.Tensor) -> torch.Tensor:
    """K = F F^T + Omega from compact coordinates Theta."""
    if raw.ndim < 2:
        raise ValueError("raw must have at least two matrix dimensions")
    if raw.shape[-2] != raw.shape[-1]:
        raise ValueError("raw must be square in its final two dimensions")
    if not raw.is_floating_point():
        raise TypeError("raw must be a floating-point tensor")
    dtype = _calc_dtype(raw)
    with torch.autocast(device_type=raw.device.type, enabled=False):
        theta = raw.to(dtype)
        if theta.shape[-1] == 0:
            return theta
        diag = torch.diagonal(theta, dim1=-2, dim2=-1)
        factor = torch.tril(theta, diagonal=-1) + torch.diag_embed(F.softplus(diag + SOFTPLUS_ONE_OFFSET))
        upper = torch.triu(theta, diagonal=1)
        if factor.dtype == torch.float64:
            gram = factor @ factor.mT
        elif factor.device.type != "cuda":
            gram = factor.float() @ factor.float().mT
        else:
            gram = _IEEEFactorGram.apply(factor)
        return gram + upper - upper.mT


def accretive_equilibrium_mix(frame, generator, compact_state, content, eta):
    """Y = eta C + P [2 (I + K)^{-1} Z - (1 + eta) Z];  generator None: Y = eta C - eta P Z."""
    if frame.ndim != 4:
        raise ValueError("frame must have shape [B, H, N, R]")
    if content.ndim != 4:
        raise ValueError("content must have shape [B, H, N, D]")
    batch, heads, length, rank = frame.shape
    if content.shape[:3] != (batch, heads, length):
        raise ValueError("frame and content must agree on [B, H, N]")
    if compact_state.shape != (batch, heads, rank, content.shape[-1]):
        raise ValueError(
            f"compact_state must have shape {(batch, heads, rank, content.shape[-1])}, got {tuple(compact_state.shape)}"
        )
    if eta.shape != (heads,):
        raise ValueError(f"eta must have shape [{heads}], got {tuple(eta.shape)}")
    tensors = (frame, compact_state, eta)
    if any(t.dtype != content.dtype or t.device != content.device for t in tensors):
        raise ValueError("frame, compact_state, content, and eta must share dtype and device")
    e = eta.view(1, heads, 1, 1)
    if generator is None:
        compact = -e * compact_state
    else:
        if not generator.is_floating_point():
            raise TypeError("generator must be a floating-point tensor")
        if generator.dtype != content.dtype or generator.device != content.device:
            raise ValueError("generator must share content dtype and device")
        if generator.ndim == 3:
            if generator.shape != (heads, rank, rank):
                raise ValueError(f"static generator must have shape {(heads, rank, rank)}, got {tuple(generator.shape)}")
            generator = generator.unsqueeze(0).expand(batch, -1, -1, -1)
        elif generator.ndim == 4:
            if generator.shape != (batch, heads, rank, rank):
                raise ValueError(
                    f"dynamic generator must have shape {(batch, heads, rank, rank)}, got {tuple(generator.shape)}"
                )
        else:
            raise ValueError("generator must have shape [H, R, R] or [B, H, R, R]")
        eye = torch.eye(rank, dtype=content.dtype, device=content.device)
        compact = 2.0 * torch.linalg.solve(generator + eye, compact_state) - (1.0 + e) * compact_state
    return e * content + tensor_core_matmul(frame, compact)


def rank_rotary(relation: torch.Tensor, positions: torch.Tensor) -> torch.Tensor:
    """Rotate rank pairs by pos * 10000^(-k/(r/2)); phases FP16-rounded unless FP64."""
    if relation.ndim != 4:
        raise ValueError("relation must have shape [B, H, N, R]")
    batch, _, length, rank = relation.shape
    if positions.shape != (batch, length):
        raise ValueError(f"positions must have shape {(batch, length)}, got {tuple(positions.shape)}")
    if rank % 2:
        raise ValueError(f"Rank-Rotary requires an even rank, got rank={rank}")
    half = rank // 2
    inv_freq = RANK_PHASE_BASE ** (-torch.arange(half, device=relation.device, dtype=relation.dtype) / half)
    angles = positions[:, :, None] * inv_freq
    cos, sin = angles.cos(), angles.sin()
    if relation.dtype != torch.float64:
        cos = cos.to(torch.float16).to(relation.dtype)
        sin = sin.to(torch.float16).to(relation.dtype)
    cos = cos.view(batch, 1, length, half)
    sin = sin.view(batch, 1, length, half)
    even, odd = relation[..., 0::2], relation[..., 1::2]
    out = torch.empty_like(relation)
    out[..., 0::2] = even * cos - odd * sin
    out[..., 1::2] = even * sin + odd * cos
    return out


__all__ = [
    "accretive_equilibrium_mix",
    "accretive_generator",
    "bounded_complement",
    "qr_soft_frame",
    "rank_rotary",
    "tensor_core_linear",
    "tensor_core_matmul",
]
