"""Helpers of the GPU parity tests: load the native library (failing loudly,
never skipping on a GPU box) and evaluate the CUDA mixer beside the oracle."""

from __future__ import annotations

import numpy as np
import torch

from oracle import lsso_oracle as O

_LOADED = False


def require_native() -> None:
    """Build (if stale) and load the sm_100a library; raise if it cannot be used."""
    global _LOADED
    if _LOADED:
        return
    from lsso_b200 import build
    from lsso_b200.ball import cuda

    build.build()
    cuda.load()
    _LOADED = True


def relative_l2(actual, expected) -> float:
    if isinstance(actual, torch.Tensor):
        actual = actual.detach().double().cpu().numpy()
    if isinstance(expected, torch.Tensor):
        expected = expected.detach().double().cpu().numpy()
    return O.relative_l2(actual, expected)


def max_abs(actual, expected) -> float:
    if isinstance(actual, torch.Tensor):
        actual = actual.detach().double().cpu().numpy()
    return float(np.abs(np.asarray(actual, np.float64) - np.asarray(expected, np.float64)).max())


def scaled_max_abs(actual, expected) -> float:
    """max|actual - expected| / max|expected| (the max-abs bound of the parity tests)."""
    expected = np.asarray(expected.detach().double().cpu().numpy() if isinstance(expected, torch.Tensor)
                          else expected, np.float64)
    return max_abs(actual, expected) / max(float(np.abs(expected).max()), 1e-30)


def seeded_mixer_inputs(seed: int, batch: int, length: int, heads: int, rank: int, head_dim: int, *,
                        core: float = 0.05, eta: float = 0.05, relscale: float = 1.0, mask=None):
    g = torch.Generator().manual_seed(seed)
    dim = heads * head_dim
    projected = torch.randn(batch, length, heads * rank + dim, generator=g)
    projected[..., : heads * rank] *= relscale
    if mask is not None:
        projected = torch.where(mask[:, :, None], projected, torch.zeros_like(projected))
    projected = projected.to(torch.bfloat16).float()
    base = torch.randn(heads, rank, rank, generator=g) * core
    drive = torch.randn(heads, head_dim, rank, generator=g) * core
    eta_raw = torch.randn(heads, generator=g) * eta
    upstream = torch.randn(batch, length, dim, generator=g)
    if mask is not None:
        upstream = torch.where(mask[:, :, None], upstream, torch.zeros_like(upstream))
    return projected, base, drive, eta_raw, upstream


def run_cuda(projected, base, drive, eta_raw, positions=None, counts=None, upstream=None):
    """Forward (and backward when upstream is given) through lsso.ball.cuda.fast_mix."""
    from lsso_b200.ball import cuda

    inputs = [projected.to(torch.bfloat16).cuda(), base.float().cuda(), drive.float().cuda(), eta_raw.float().cuda()]
    pos = None if positions is None else torch.as_tensor(positions, dtype=torch.float32).cuda().contiguous()
    cnt = None if counts is None else torch.as_tensor(counts, dtype=torch.float32).cuda().contiguous()
    if upstream is None:
        with torch.no_grad():
            return cuda.fast_mix(*inputs, pos, cnt), None
    inputs = [t.detach().requires_grad_() for t in inputs]
    out = cuda.fast_mix(*inputs, pos, cnt)
    grads = torch.autograd.grad((out.float() * upstream.cuda()).sum(), inputs)
    torch.cuda.synchronize()
    return out, grads


def run_oracle(projected, base, drive, eta_raw, positions=None, counts=None, upstream=None, *, contract=True):
    """The oracle on the same inputs.

    ``contract=True`` (default): FP64 mixer with the CUDA contract's FP16
    phases, fed the BF16 upstream gradient the native backward receives
    (its grad_output is BF16).  ``contract=False``: the exact FP64 operator
    with the FP32 upstream, the reference tests' FP64 oracle."""
    n = lambda t: None if t is None else np.asarray(t.detach().cpu().numpy() if isinstance(t, torch.Tensor) else t,
                                                     np.float64)  # noqa: E731
    out, state = O.mixer_forward(n(projected), n(base), n(drive), n(eta_raw), n(positions), n(counts),
                                 return_state=True, contract=contract)
    if upstream is None:
        return out, None
    up = n(upstream)
    if contract:
        up = O.round_bf16(up).astype(np.float64)
    return out, O.mixer_backward(up, state)
