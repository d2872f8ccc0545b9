"""CPU oracle for the LSSO DYNAMIC + Rank-Rotary mixer.

TEST INFRASTRUCTURE ONLY.  Nothing in the shipped package imports this file:
it is the checker used by ``tests/``, ``__graft_entry__.smoke()`` and the CPU
legs of ``bench.py`` (``cpu_baseline`` and ``--impl reference``).

It restates, in NumPy, the reference algorithm of Yang916-yy/LSSO for the
hot path (the complete DYNAMIC + Rank-Rotary mixer with its projections),
together with the analytic first-order backward of that algorithm.  Every
function cites the reference file:line it follows (paths inside the LSSO
project).  Parity of this restatement is pinned against outputs and autograd
gradients of the reference's own PyTorch implementation, recorded as golden
fixtures in ``tests/golden/*.npz`` by ``tests/golden/make_golden.py``.

Two numeric modes exist:

* ``float64``: the mathematical operator, the same role as the reference
  tests' FP64 oracle (``tests/cuda/test_fast_path.py:33-86``).
* ``float32``: the reference's CPU ``implementation="reference"`` path, which
  rounds the packed projection to BF16, rounds Rank-Rotary phases to FP16 and
  rounds the mixer output to BF16 (``lsso/ball/model.py:441-446,574-575``,
  ``lsso/ball/reference.py:711-715``).  This is the timed CPU baseline.

and ``contract=True`` (with ``float64``): the mixer core in FP64, with every
rounding the reference's FP32 path on CUDA tensors applies at its tensor
boundaries -- FP16 Rank-Rotary phases from FP32 angles, BF16 projection
operands with wide accumulation, BF16 packed projection and mixer output, and
in the backward the BF16 upstream gradient of each projection, the BF16
gradient of the BF16 mixer output and of the BF16 packed projection
(``lsso/ball/reference.py:170-247``, ``lsso/ball/model.py:441-446,574-575``,
``csrc/ball/backward.cu:295-296``).  A CUDA result compared with this mode
shows the error of its own arithmetic, not of the roundings the contract
prescribes.
"""

from __future__ import annotations

import math

import numpy as np

RANK_PHASE_BASE = 10000.0  # lsso/ball/reference.py:12
SOFTPLUS_ONE_OFFSET = math.log(math.expm1(1.0))  # lsso/ball/reference.py:13
ETA_INIT_RAW = math.atanh(0.9)  # lsso/ball/model.py:22-23


# ---------------------------------------------------------------------------
# Rounding helpers (BF16 has no NumPy dtype: round-to-nearest-even on bits)
# ---------------------------------------------------------------------------

def round_bf16(value: np.ndarray) -> np.ndarray:
    """Round to the nearest BF16 value (ties to even), returned as float32."""
    as32 = np.ascontiguousarray(value, dtype=np.float32)
    bits = as32.view(np.uint32)
    # uint32 cannot overflow here: only NaN bit patterns exceed 0xFFFF7FFF,
    # and those are restored below.
    rounded = ((bits + (((bits >> 16) & 1) + np.uint32(0x7FFF))) >> 16) << 16
    out = rounded.astype(np.uint32).view(np.float32)
    # NaN/Inf keep their class.
    special = ~np.isfinite(as32)
    if special.any():
        out = out.copy()
        out[special] = as32[special]
    return out


def round_fp16(value: np.ndarray) -> np.ndarray:
    return np.asarray(value, dtype=np.float32).astype(np.float16).astype(np.float32)


# ---------------------------------------------------------------------------
# Positions (lsso/ball/model.py:163-243)
# ---------------------------------------------------------------------------

def center_positions(
    position_ids: np.ndarray | None,
    valid_mask: np.ndarray | None,
    batch: int,
    length: int,
    dtype=np.float32,
) -> np.ndarray:
    """Centered Rank-Rotary coordinates, ``[B, N]`` (model.py:163-243).

    Integer ids are differenced in int64 before any float conversion; FP64 ids
    are centered in FP64; FP32 ids in the calculation dtype.  Masked rows are
    anchored at their first valid token, centered on the valid mean and
    invalid positions become zero.
    """
    if position_ids is None:
        positions = np.broadcast_to(np.arange(length, dtype=dtype), (batch, length))
    else:
        position_ids = np.asarray(position_ids)
        if np.issubdtype(position_ids.dtype, np.floating):
            pdtype = np.float64 if position_ids.dtype == np.float64 else dtype
            positions = position_ids.astype(pdtype)
        else:
            positions = position_ids.astype(np.int64)
        if positions.ndim == 1:
            positions = np.broadcast_to(positions[None, :], (batch, length))
    if valid_mask is None:
        centered = positions - positions[:, :1]
        if centered.dtype == np.int64:
            centered = centered.astype(dtype)
        centered = centered - centered.mean(axis=-1, keepdims=True)
        return centered.astype(dtype)
    mask = np.asarray(valid_mask, dtype=bool)
    first = mask.astype(np.int64).argmax(axis=-1)[:, None]
    anchor = np.take_along_axis(positions, first, axis=1)
    centered = positions - anchor
    if centered.dtype == np.int64:
        centered = centered.astype(dtype)
    weights = mask.astype(centered.dtype)
    count = np.maximum(weights.sum(axis=-1, keepdims=True), 1.0)
    safe = np.where(mask, centered, 0.0)
    mean = (safe * weights).sum(axis=-1, keepdims=True) / count
    return np.where(mask, centered - mean, 0.0).astype(dtype)


# ---------------------------------------------------------------------------
# Rank-Rotary (lsso/ball/reference.py:691-724)
# ---------------------------------------------------------------------------

def rank_phases(positions: np.ndarray, rank: int, dtype) -> tuple[np.ndarray, np.ndarray]:
    """cos/sin of ``pos * 10000^(-k/half)``; FP16-rounded unless FP64."""
    half = rank // 2
    k = np.arange(half, dtype=dtype)
    inv_freq = np.power(dtype(RANK_PHASE_BASE), -k / dtype(half)).astype(dtype)
    angles = positions.astype(dtype)[..., None] * inv_freq
    cos = np.cos(angles).astype(dtype)
    sin = np.sin(angles).astype(dtype)
    if dtype != np.float64:
        cos = round_fp16(cos).astype(dtype)
        sin = round_fp16(sin).astype(dtype)
    return cos, sin


def rank_rotary(relation: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """Rotate (even, odd) rank pairs; relation ``[B,H,N,r]``, cos/sin ``[B,N,r/2]``."""
    c = cos[:, None]
    s = sin[:, None]
    even = relation[..., 0::2]
    odd = relation[..., 1::2]
    out = np.empty_like(relation)
    out[..., 0::2] = even * c - odd * s
    out[..., 1::2] = even * s + odd * c
    return out


def rank_rotary_transpose(grad: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """Adjoint of :func:`rank_rotary` (the inverse rotation)."""
    c = cos[:, None]
    s = sin[:, None]
    ge = grad[..., 0::2]
    go = grad[..., 1::2]
    out = np.empty_like(grad)
    out[..., 0::2] = ge * c + go * s
    out[..., 1::2] = -ge * s + go * c
    return out


# ---------------------------------------------------------------------------
# Frame, generator, complement, equilibrium (lsso/ball/reference.py)
# ---------------------------------------------------------------------------

def qr_soft_frame(relation: np.ndarray) -> np.ndarray:
    """Top block of Q in QR([A/s; I/s]) with a positive R diagonal.

    Follows reference.py:411-447: s = max(1, max|A|) per matrix, reduced QR,
    column signs fixed so that diag(R) > 0, rows of A kept.
    """
    length, rank = relation.shape[-2:]
    scale = np.maximum(np.abs(relation).max(axis=(-2, -1), keepdims=True), 1.0)
    eye = np.broadcast_to(np.eye(rank, dtype=relation.dtype), relation.shape[:-2] + (rank, rank))
    augmented = np.concatenate((relation / scale, eye / scale), axis=-2)
    q, r = np.linalg.qr(augmented, mode="reduced")
    diag = np.diagonal(r, axis1=-2, axis2=-1)
    signs = np.where(diag < 0, -1.0, 1.0).astype(relation.dtype)
    return (q * signs[..., None, :])[..., :length, :]


def bounded_complement(raw: np.ndarray) -> np.ndarray:
    """(1 - eps) tanh(raw) through the stable logistic identity (reference.py:450-471)."""
    dtype = raw.dtype
    eps = np.finfo(dtype).eps
    pos = np.exp(-2.0 * np.maximum(raw, 0.0))
    neg = np.exp(2.0 * np.minimum(raw, 0.0))
    positive = (1.0 - pos) / (1.0 + pos)
    negative = (neg - 1.0) / (1.0 + neg)
    return ((1.0 - eps) * np.where(raw >= 0.0, positive, negative)).astype(dtype)


def bounded_complement_derivative(raw: np.ndarray) -> np.ndarray:
    """d/draw of :func:`bounded_complement`: (1-eps) * 4p/(1+p)^2, p = exp(-2|raw|)."""
    dtype = raw.dtype
    eps = np.finfo(dtype).eps
    p = np.exp(-2.0 * np.abs(raw))
    return ((1.0 - eps) * 4.0 * p / (1.0 + p) ** 2).astype(dtype)


def softplus(x: np.ndarray) -> np.ndarray:
    """torch.nn.functional.softplus with beta=1, threshold=20."""
    return np.where(x > 20.0, x, np.log1p(np.exp(np.minimum(x, 20.0))))


def softplus_derivative(x: np.ndarray) -> np.ndarray:
    return np.where(x > 20.0, 1.0, 1.0 / (1.0 + np.exp(-np.minimum(x, 20.0))))


def accretive_parts(theta: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """F = tril(Θ,-1) + diag(softplus(diag Θ + log(e-1))), Ω = triu(Θ,1) - triu(Θ,1)ᵀ.

    reference.py:474-497.
    """
    rank = theta.shape[-1]
    diag = np.diagonal(theta, axis1=-2, axis2=-1)
    factor = np.tril(theta, -1) + np.eye(rank, dtype=theta.dtype) * softplus(diag + SOFTPLUS_ONE_OFFSET)[..., None, :]
    upper = np.triu(theta, 1)
    skew = upper - np.swapaxes(upper, -1, -2)
    return factor, skew


def accretive_generator(theta: np.ndarray) -> np.ndarray:
    factor, skew = accretive_parts(theta)
    return factor @ np.swapaxes(factor, -1, -2) + skew


def accretive_equilibrium_mix(frame, generator, compact_state, content, eta):
    """Y = eta C + P [2 (I+K)^-1 Z - (1+eta) Z]  (reference.py:500-572)."""
    rank = frame.shape[-1]
    eta_b = eta[None, :, None, None]
    system = generator + np.eye(rank, dtype=content.dtype)
    equilibrium = np.linalg.solve(system, compact_state)
    compact = 2.0 * equilibrium - (1.0 + eta_b) * compact_state
    return eta_b * content + frame @ compact


# ---------------------------------------------------------------------------
# The strict native ABI composition (tests/cuda/test_fast_path.py:33-86)
# ---------------------------------------------------------------------------

def split_projected(projected: np.ndarray, heads: int, rank: int):
    batch, length, width = projected.shape
    dim = width - heads * rank
    head_dim = dim // heads
    relation = projected[..., : heads * rank].reshape(batch, length, heads, rank).transpose(0, 2, 1, 3)
    content = projected[..., heads * rank:].reshape(batch, length, heads, head_dim).transpose(0, 2, 1, 3)
    return relation, content


def default_positions(length: int, dtype) -> np.ndarray:
    """Centered default positions ``t - (N-1)/2`` (forward.cu default table)."""
    return np.arange(length, dtype=dtype) - dtype(0.5 * (length - 1))


def mixer_forward(
    projected: np.ndarray,
    core_base_raw: np.ndarray,
    core_drive_weight: np.ndarray,
    eta_raw: np.ndarray,
    centered_positions: np.ndarray | None = None,
    valid_counts: np.ndarray | None = None,
    *,
    dtype=np.float64,
    return_state: bool = False,
    contract: bool = False,
):
    """Mixed coordinates ``[B, N, D]`` of the native ABI (test_fast_path.py:33-86).

    ``contract=True`` takes the phases of the CUDA contract (FP32 angles,
    cos/sin rounded to FP16; reference.py:711-715) into the ``dtype``
    arithmetic.

    ``projected`` is the packed ``[B, N, H*r + D]`` tensor (BF16 values in any
    float dtype), ``centered_positions`` is ``[N]`` or ``[B, N]`` (default
    ``t - (N-1)/2``), ``valid_counts`` is ``[B]`` (default ``N``).  The frame
    uses the QR form of the reference; its Cholesky identity ``P = A L^{-T}``
    (``L L^T = A^T A + I``) supplies the state the backward needs.
    """
    projected = np.asarray(projected, dtype=dtype)
    base = np.asarray(core_base_raw, dtype=dtype)
    drive = np.asarray(core_drive_weight, dtype=dtype)
    eta_raw = np.asarray(eta_raw, dtype=dtype)
    batch, length, width = projected.shape
    heads, rank = base.shape[0], base.shape[-1]
    dim = width - heads * rank
    if valid_counts is None:
        counts = np.full((batch,), float(length), dtype=dtype)
    else:
        counts = np.asarray(valid_counts, dtype=dtype)
    if centered_positions is None:
        positions = np.broadcast_to(default_positions(length, dtype), (batch, length))
    else:
        positions = np.asarray(centered_positions, dtype=dtype)
        if positions.ndim == 1:
            positions = np.broadcast_to(positions[None], (batch, length))
    relation, content = split_projected(projected, heads, rank)
    if contract:
        cos, sin = (v.astype(dtype) for v in rank_phases(positions.astype(np.float32), rank, np.float32))
    else:
        cos, sin = rank_phases(positions, rank, dtype)
    root = np.sqrt(counts)[:, None, None, None]
    A = rank_rotary(relation, cos, sin) / root
    frame = qr_soft_frame(A)
    Z = np.swapaxes(frame, -1, -2) @ content
    theta = base[None] + (Z @ drive[None]) / root
    generator = accretive_generator(theta)
    eta = bounded_complement(eta_raw)
    mixed = accretive_equilibrium_mix(frame, generator, Z, content, eta)
    out = mixed.transpose(0, 2, 1, 3).reshape(batch, length, dim)
    if not return_state:
        return out
    state = dict(
        relation=relation, content=content, cos=cos, sin=sin, root=root, A=A,
        frame=frame, Z=Z, theta=theta, generator=generator, eta=eta,
        eta_raw=eta_raw, drive=drive, heads=heads, rank=rank, dim=dim,
    )
    return out, state


def mixer_backward(grad_output: np.ndarray, state: dict):
    """Analytic VJP of :func:`mixer_forward` (first order).

    Returns ``(grad_projected, grad_core_base_raw, grad_core_drive_weight,
    grad_eta_raw)``.  Derivation (per sample b and head h, dropping indices):

    * ``D = P^T dY``;  ``lam = (I+K)^{-T} (2 D)``;  ``dK = -lam U^T``;
    * ``dTheta`` through ``K = F F^T + Omega`` and softplus';
    * ``dZ = lam - (1+eta) D + dTheta W_drive^T / sqrt(n)``;
    * ``d eta = <dY, C> - <D, Z>``;
    * QR-frame VJP (top block of Q for QR([A/s; I/s]), R-bar = 0):
      ``dA = (dP - P copyltu(dP^T P)) L^{-1}`` with ``dP = dY M'^T + C dZ^T``
      and ``dP^T P = M' D^T + dZ Z^T``;
    * ``dC = eta dY + P dZ``; relation gradient = rotation transpose of
      ``dA / sqrt(n)``.
    """
    heads, rank, dim = state["heads"], state["rank"], state["dim"]
    relation, content = state["relation"], state["content"]
    A, P, Z, theta = state["A"], state["frame"], state["Z"], state["theta"]
    eta, eta_raw, drive, root = state["eta"], state["eta_raw"], state["drive"], state["root"]
    cos, sin = state["cos"], state["sin"]
    dtype = A.dtype
    batch, length = relation.shape[0], relation.shape[2]
    head_dim = dim // heads
    dY = np.asarray(grad_output, dtype=dtype).reshape(batch, length, heads, head_dim).transpose(0, 2, 1, 3)
    eye = np.eye(rank, dtype=dtype)
    T = lambda x: np.swapaxes(x, -1, -2)  # noqa: E731

    factor, _skew = accretive_parts(theta)
    system = eye + state["generator"]
    U = np.linalg.solve(system, Z)
    eta_b = eta[None, :, None, None]
    Mp = 2.0 * U - (1.0 + eta_b) * Z
    D = T(P) @ dY
    lam = np.linalg.solve(T(system), 2.0 * D)
    dK = -lam @ T(U)
    dF = (dK + T(dK)) @ factor
    sig = softplus_derivative(np.diagonal(theta, axis1=-2, axis2=-1) + SOFTPLUS_ONE_OFFSET)
    upper = np.triu(np.ones((rank, rank), dtype=bool), 1)
    lower = np.tril(np.ones((rank, rank), dtype=bool), -1)
    dTheta = np.where(upper, dK - T(dK), 0.0) + np.where(lower, dF, 0.0)
    dTheta = dTheta + eye * (np.diagonal(dF, axis1=-2, axis2=-1) * sig)[..., None, :]
    grad_base = dTheta.sum(axis=0)
    grad_drive = (T(Z) @ dTheta / root).sum(axis=0)
    dZ = lam - (1.0 + eta_b) * D + dTheta @ T(drive)[None] / root
    deta = (dY * content).sum(axis=(-2, -1)) - (D * Z).sum(axis=(-2, -1))
    grad_eta_raw = deta.sum(axis=0) * bounded_complement_derivative(eta_raw)

    G = T(A) @ A + eye
    L = np.linalg.cholesky(G)
    E = Mp @ T(D) + dZ @ T(Z)
    psi = np.tril(E) + T(np.tril(E, -1))
    dP = dY @ T(Mp) + content @ T(dZ)
    inner = dP - P @ psi
    # dA = inner L^{-1}  <=>  dA^T = L^{-T} inner^T
    dA = T(np.linalg.solve(T(L), T(inner)))
    dC = eta_b * dY + P @ dZ
    drel = rank_rotary_transpose(dA / root, cos, sin)
    grad_rel = drel.transpose(0, 2, 1, 3).reshape(batch, length, heads * rank)
    grad_con = dC.transpose(0, 2, 1, 3).reshape(batch, length, dim)
    grad_projected = np.concatenate((grad_rel, grad_con), axis=-1)
    return grad_projected, grad_base, grad_drive, grad_eta_raw


# ---------------------------------------------------------------------------
# Projections and the full module (lsso/ball/model.py:407-585,
# lsso/ball/reference.py:170-247,347-408)
# ---------------------------------------------------------------------------

def linear(value: np.ndarray, weight: np.ndarray, bias: np.ndarray | None, *, bf16_operands: bool):
    """value @ weight^T + bias with FP32/FP64 accumulation.

    With ``bf16_operands`` both multiplicands are rounded to BF16 first, the
    CUDA contract of ``tensor_core_linear`` (reference.py:181-202).
    """
    if bf16_operands:
        value = round_bf16(value).astype(np.float64)
        weight = round_bf16(weight).astype(np.float64)
    out = value @ weight.T
    if bias is not None:
        out = out + bias
    return out


def module_forward(params: dict, x: np.ndarray, valid_mask=None, position_ids=None, *,
                   heads: int, rank: int, dtype=np.float64, return_state: bool = False, contract: bool = False,
                   activation: str | None = None):
    """Complete LSSO forward (model.py:542-585) for DYNAMIC + Rank-Rotary.

    ``dtype=float64`` is the FP64 oracle; ``dtype=float32`` mirrors the
    reference's CPU FP32 path (BF16 packed coordinates and BF16 mixer output);
    ``contract=True`` (FP64) adds the roundings of the reference's path on
    CUDA tensors (module docstring); there ``activation`` ("float16" or
    "bfloat16", x's dtype) also rounds y and the gradient of x to it, as the
    projections store them (reference.py:202,224).  ``params`` holds
    ``w_bc``, ``b_bc`` (or None), ``w_o``, ``b_o``, ``core_base_raw``,
    ``core_drive_weight``, ``eta_raw``.
    """
    if contract:
        return _module_forward_contract(params, x, valid_mask, position_ids, heads=heads, rank=rank,
                                        return_state=return_state, activation=activation)
    x = np.asarray(x, dtype=dtype)
    batch, length, dim = x.shape
    mask = None if valid_mask is None else np.asarray(valid_mask, dtype=bool)
    safe_x = x if mask is None else np.where(mask[:, :, None], x, 0.0)
    w_bc = np.asarray(params["w_bc"], dtype=dtype)
    b_bc = None if params.get("b_bc") is None else np.asarray(params["b_bc"], dtype=dtype)
    projected = (safe_x.reshape(-1, dim) @ w_bc.T).reshape(batch, length, -1)
    if b_bc is not None:
        projected = projected + b_bc
    if dtype != np.float64:
        projected = round_bf16(projected).astype(dtype)
    if mask is not None:
        projected = np.where(mask[:, :, None], projected, 0.0)
    positions = center_positions(position_ids, mask, batch, length, dtype=dtype)
    counts = None if mask is None else np.maximum(mask.sum(axis=-1).astype(dtype), 1.0)
    mixed, state = mixer_forward(projected, params["core_base_raw"], params["core_drive_weight"],
                                 params["eta_raw"], positions, counts, dtype=dtype, return_state=True)
    if dtype != np.float64:
        mixed = round_bf16(mixed).astype(dtype)
    w_o = np.asarray(params["w_o"], dtype=dtype)
    b_o = None if params.get("b_o") is None else np.asarray(params["b_o"], dtype=dtype)
    out = (mixed.reshape(-1, dim) @ w_o.T).reshape(batch, length, dim)
    if b_o is not None:
        out = out + b_o
    if mask is not None:
        out = np.where(mask[:, :, None], out, 0.0)
    if not return_state:
        return out
    return out, dict(mixer=state, x=safe_x, mixed=mixed, mask=mask, w_bc=w_bc, w_o=w_o,
                     has_bias=b_bc is not None)


def _bf16(value: np.ndarray) -> np.ndarray:
    return round_bf16(value).astype(np.float64)


def _round_activation(value: np.ndarray, activation: str | None) -> np.ndarray:
    if activation is None:
        return value
    if activation == "bfloat16":
        return _bf16(value)
    if activation == "float16":
        return round_fp16(value).astype(np.float64)
    raise ValueError(f"activation must be 'float16', 'bfloat16' or None, got {activation!r}")


def _module_forward_contract(params, x, valid_mask, position_ids, *, heads, rank, return_state, activation):
    """FP64 module forward with the CUDA contract's roundings.

    Projections follow ``_TensorCoreLinear.forward`` (reference.py:172-202):
    BF16 value and weight, wide accumulation, FP32 bias added before the one
    store (BF16 for the packed projection, model.py:376-378).  Positions are
    centered in FP32 (model.py:163-243 with the FP32 calculation dtype of the
    CUDA path) and the mixer output is rounded to BF16 (model.py:441-446).
    """
    x = np.asarray(x, dtype=np.float64)
    batch, length, dim = x.shape
    mask = None if valid_mask is None else np.asarray(valid_mask, dtype=bool)
    safe_x = x if mask is None else np.where(mask[:, :, None], x, 0.0)
    x_bf16 = _bf16(safe_x)
    w_bc = _bf16(np.asarray(params["w_bc"], np.float32))
    w_o = _bf16(np.asarray(params["w_o"], np.float32))
    b_bc = None if params.get("b_bc") is None else np.asarray(params["b_bc"], np.float32).astype(np.float64)
    b_o = None if params.get("b_o") is None else np.asarray(params["b_o"], np.float32).astype(np.float64)
    projected = (x_bf16.reshape(-1, dim) @ w_bc.T).reshape(batch, length, -1)
    if b_bc is not None:
        projected = projected + b_bc
    projected = _bf16(projected)
    if mask is not None:
        projected = np.where(mask[:, :, None], projected, 0.0)
    positions = center_positions(position_ids, mask, batch, length, dtype=np.float32)
    counts = None if mask is None else np.maximum(mask.sum(axis=-1).astype(np.float32), 1.0)
    mixed, state = mixer_forward(projected, params["core_base_raw"], params["core_drive_weight"],
                                 params["eta_raw"], positions, counts, dtype=np.float64, return_state=True,
                                 contract=True)
    mixed = _bf16(mixed)
    out = (mixed.reshape(-1, dim) @ w_o.T).reshape(batch, length, dim)
    if b_o is not None:
        out = out + b_o
    out = _round_activation(out, activation)
    if mask is not None:
        out = np.where(mask[:, :, None], out, 0.0)
    if not return_state:
        return out
    return out, dict(mixer=state, x=x_bf16, mixed=mixed, mask=mask, w_bc=w_bc, w_o=w_o,
                     has_bias=b_bc is not None, contract=True, activation=activation)


def module_backward(grad_out: np.ndarray, mstate: dict):
    """Gradients of :func:`module_forward` for x and every parameter.

    For a ``contract`` forward the VJPs follow ``_TensorCoreLinear.backward``
    (reference.py:204-247): the upstream gradient of each projection is
    rounded to BF16 before both GEMMs, the bias gradient sums it unrounded,
    and the gradients of the BF16 tensors (mixer output, packed projection)
    are BF16.
    """
    if mstate.get("contract"):
        return _module_backward_contract(grad_out, mstate)
    mask = mstate["mask"]
    dtype = mstate["x"].dtype
    grad_out = np.asarray(grad_out, dtype=dtype)
    if mask is not None:
        grad_out = np.where(mask[:, :, None], grad_out, 0.0)
    batch, length, dim = grad_out.shape
    go = grad_out.reshape(-1, dim)
    mixed = mstate["mixed"].reshape(-1, dim)
    grad_w_o = go.T @ mixed
    grad_b_o = go.sum(axis=0) if mstate["has_bias"] else None
    grad_mixed = (go @ mstate["w_o"]).reshape(batch, length, dim)
    gproj, gbase, gdrive, geta = mixer_backward(grad_mixed, mstate["mixer"])
    if mask is not None:
        gproj = np.where(mask[:, :, None], gproj, 0.0)
    gp = gproj.reshape(batch * length, -1)
    x = mstate["x"].reshape(-1, dim)
    grad_w_bc = gp.T @ x
    grad_b_bc = gp.sum(axis=0) if mstate["has_bias"] else None
    grad_x = (gp @ mstate["w_bc"]).reshape(batch, length, dim)
    if mask is not None:
        grad_x = np.where(mask[:, :, None], grad_x, 0.0)
    grads = dict(x=grad_x, w_bc=grad_w_bc, b_bc=grad_b_bc, w_o=grad_w_o, b_o=grad_b_o,
                 core_base_raw=gbase, core_drive_weight=gdrive, eta_raw=geta)
    return grads


def _module_backward_contract(grad_out, mstate):
    mask = mstate["mask"]
    grad_out = np.asarray(grad_out, dtype=np.float64)
    if mask is not None:
        grad_out = np.where(mask[:, :, None], grad_out, 0.0)
    batch, length, dim = grad_out.shape
    go_raw = grad_out.reshape(-1, dim)
    go = _bf16(go_raw)
    grad_w_o = go.T @ mstate["mixed"].reshape(-1, dim)
    grad_b_o = go_raw.sum(axis=0) if mstate["has_bias"] else None
    grad_mixed = _bf16(go @ mstate["w_o"]).reshape(batch, length, dim)
    gproj, gbase, gdrive, geta = mixer_backward(grad_mixed, mstate["mixer"])
    gproj = _bf16(gproj)
    if mask is not None:
        gproj = np.where(mask[:, :, None], gproj, 0.0)
    gp = gproj.reshape(batch * length, -1)
    grad_w_bc = gp.T @ mstate["x"].reshape(-1, dim)
    grad_b_bc = gp.sum(axis=0) if mstate["has_bias"] else None
    grad_x = _round_activation((gp @ mstate["w_bc"]).reshape(batch, length, dim), mstate["activation"])
    if mask is not None:
        grad_x = np.where(mask[:, :, None], grad_x, 0.0)
    return dict(x=grad_x, w_bc=grad_w_bc, b_bc=grad_b_bc, w_o=grad_w_o, b_o=grad_b_o,
                core_base_raw=gbase, core_drive_weight=gdrive, eta_raw=geta)


def init_params(dim: int, heads: int, rank: int, *, bias: bool = False, seed: int = 0,
                core_scale: float = 0.0) -> dict:
    """Seeded parameters with the module's shapes (model.py:40-72).

    Weights follow PyTorch's default Linear init distribution
    (U(-1/sqrt(in), 1/sqrt(in))) from a NumPy generator; core parameters are
    zero (times ``core_scale`` noise if given) and eta_raw = atanh(0.9).
    """
    rng = np.random.default_rng(seed)
    width = heads * rank + dim
    bound = 1.0 / math.sqrt(dim)
    params = dict(
        w_bc=rng.uniform(-bound, bound, (width, dim)).astype(np.float32),
        b_bc=rng.uniform(-bound, bound, (width,)).astype(np.float32) if bias else None,
        w_o=rng.uniform(-bound, bound, (dim, dim)).astype(np.float32),
        b_o=rng.uniform(-bound, bound, (dim,)).astype(np.float32) if bias else None,
        core_base_raw=(core_scale * rng.standard_normal((heads, rank, rank))).astype(np.float32),
        core_drive_weight=(core_scale * rng.standard_normal((heads, dim // heads, rank))).astype(np.float32),
        eta_raw=np.full((heads,), ETA_INIT_RAW, dtype=np.float32),
    )
    return params


def relative_l2(actual: np.ndarray, expected: np.ndarray) -> float:
    a = np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    return float(np.linalg.norm(a - e) / max(np.linalg.norm(e), 1e-12))


__all__ = [
    "accretive_equilibrium_mix", "accretive_generator", "bounded_complement",
    "center_positions", "init_params", "linear", "mixer_backward", "mixer_forward",
    "module_backward", "module_forward", "qr_soft_frame", "rank_phases", "rank_rotary",
    "relative_l2", "round_bf16", "round_fp16",
]
