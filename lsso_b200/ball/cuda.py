"""Loader and autograd boundary of the B200 mixer (drop-in for lsso/ball/cuda.py).

``load()`` binds one native library per process (``lsso_equilibrium_sm100.so``,
built for sm_100a), checks its contract version (8) and registers the
``torch.ops.lsso_equilibrium`` operators.  ``fast_mix()`` chooses the
inference or the tape-producing training entry point exactly as the
reference does (cuda.py:283-323); ``_FastMix`` carries the first-order VJP.
There is no fallback: without a loaded library ``fast_mix`` raises.
"""

from __future__ import annotations

import os
from pathlib import Path
from threading import Lock

import torch

from . import _native

_LOAD_LOCK = Lock()
_SUPPORTED_ARCHITECTURES = frozenset((100,))
_NATIVE_CONTRACT_VERSION = _native.CONTRACT_VERSION
_LOADED_ARCHITECTURE: int | None = None
_LIBRARY_DIR = Path(__file__).resolve().parents[1] / "lib"


def _native_operator_abi_is_registered() -> bool:
    namespace = getattr(torch.ops, "lsso_equilibrium", None)
    return (
        namespace is not None
        and hasattr(namespace, "forward_inference")
        and hasattr(namespace, "forward_train")
        and hasattr(namespace, "backward")
    )


def _native_contract_version() -> int | None:
    namespace = getattr(torch.ops, "lsso_equilibrium", None)
    if namespace is None or not hasattr(namespace, "contract_version"):
        return None
    try:
        version = namespace.contract_version()
    except RuntimeError:
        return None
    return version if isinstance(version, int) else None


def _check_native_contract() -> None:
    version = _native_contract_version()
    if version is None:
        raise RuntimeError(
            "the loaded LSSO CUDA extension does not expose the required native contract version "
            f"{_NATIVE_CONTRACT_VERSION}; rebuild it with python -m lsso_b200.build and restart the process"
        )
    if version != _NATIVE_CONTRACT_VERSION:
        raise RuntimeError(
            f"the loaded LSSO CUDA extension has native contract version {version}, but this package requires "
            f"{_NATIVE_CONTRACT_VERSION}; rebuild it with python -m lsso_b200.build and restart the process"
        )


def is_available() -> bool:
    """Whether the strict DYNAMIC + Rank-Rotary operator is registered."""
    return _native_operator_abi_is_registered() and _native_contract_version() == _NATIVE_CONTRACT_VERSION


def require_available() -> None:
    """Reject an explicit CUDA request until its library is loaded."""
    with _LOAD_LOCK:
        if _LOADED_ARCHITECTURE is not None:
            return
        if not is_available():
            if _native_operator_abi_is_registered():
                _check_native_contract()
            raise RuntimeError(
                "the LSSO accretive-equilibrium CUDA extension is not loaded; build it with "
                "python -m lsso_b200.build, then call lsso.ball.cuda.load(); "
                f"native contract version {_NATIVE_CONTRACT_VERSION} is required"
            )


def _device_architecture(device: torch.device | int | None = None) -> int:
    if not torch.cuda.is_available():
        raise RuntimeError("the LSSO CUDA fast path requires an available CUDA device")
    if device is None:
        resolved = torch.device("cuda", torch.cuda.current_device())
    elif isinstance(device, int):
        resolved = torch.device("cuda", device)
    else:
        resolved = torch.device(device)
    if resolved.type != "cuda":
        raise ValueError(f"the LSSO CUDA fast path requires a CUDA device, got {resolved}")
    if resolved.index is None:
        resolved = torch.device("cuda", torch.cuda.current_device())
    major, minor = torch.cuda.get_device_capability(resolved)
    architecture = major * 10 + minor
    if architecture not in _SUPPORTED_ARCHITECTURES:
        raise RuntimeError(f"the LSSO CUDA fast path supports SM100 (B200); got SM{major}{minor}")
    return architecture


def _development_library_path(architecture: int) -> Path:
    return _LIBRARY_DIR / f"lsso_equilibrium_sm{architecture}.so"


def _default_library_path(device: torch.device | int | None = None) -> Path:
    override = os.environ.get("LSSO_CUDA_LIBRARY")
    if override:
        return Path(override).expanduser()
    return _development_library_path(_device_architecture(device))


def _register_library(path: Path) -> None:
    _native.register(path)


def load(path: str | os.PathLike[str] | None = None, *, device: torch.device | int | None = None) -> None:
    """Load the strict sm_100a library once per process."""
    global _LOADED_ARCHITECTURE
    requested = _device_architecture(device)
    with _LOAD_LOCK:
        if is_available():
            if _LOADED_ARCHITECTURE is not None and _LOADED_ARCHITECTURE != requested:
                raise RuntimeError(
                    f"the loaded LSSO CUDA extension targets SM{_LOADED_ARCHITECTURE}, not requested SM{requested}"
                )
            if _LOADED_ARCHITECTURE is None:
                _LOADED_ARCHITECTURE = requested
            return
        if _native_operator_abi_is_registered():
            _check_native_contract()
        library = Path(path) if path is not None else _default_library_path(device)
        library = library.expanduser().resolve()
        expected = f"lsso_equilibrium_sm{requested}.so"
        if library.name != expected:
            raise RuntimeError(
                f"the strict LSSO CUDA fast path requires {expected} for SM{requested}, got {library.name}"
            )
        if not library.is_file():
            raise RuntimeError(
                f"the LSSO CUDA extension was not found at {library}; build it with python -m lsso_b200.build "
                "or pass its path to load()"
            )
        _register_library(library)
        _check_native_contract()
        _LOADED_ARCHITECTURE = requested


class _FastMix(torch.autograd.Function):
    @staticmethod
    def forward(ctx, projected, core_base_raw, core_drive_weight, eta_raw, centered_positions, valid_counts):
        output, tape, pivots = torch.ops.lsso_equilibrium.forward_train(
            projected, core_base_raw, core_drive_weight, eta_raw, centered_positions, valid_counts)
        saved = [projected, core_base_raw, core_drive_weight, eta_raw, tape, pivots]
        if centered_positions is not None:
            saved.append(centered_positions)
        if valid_counts is not None:
            saved.append(valid_counts)
        ctx.save_for_backward(*saved)
        ctx.has_positions = centered_positions is not None
        ctx.has_valid_counts = valid_counts is not None
        return output

    @staticmethod
    @torch.autograd.function.once_differentiable
    def backward(ctx, grad_output):
        saved = ctx.saved_tensors
        projected, core_base_raw, core_drive_weight, eta_raw, tape, pivots = saved[:6]
        index = 6
        centered_positions = saved[index] if ctx.has_positions else None
        index += int(ctx.has_positions)
        valid_counts = saved[index] if ctx.has_valid_counts else None
        gradients = torch.ops.lsso_equilibrium.backward(
            grad_output.contiguous(), projected, core_base_raw, core_drive_weight, eta_raw, tape, pivots,
            centered_positions, valid_counts)
        return (*gradients, None, None)


def fast_mix(projected, core_base_raw, core_drive_weight, eta_raw, centered_positions=None, valid_counts=None):
    """Run the native mixer with first-order autograd support."""
    if centered_positions is not None and centered_positions.requires_grad:
        raise ValueError("the LSSO CUDA fast path does not support gradients for centered_positions")
    if valid_counts is not None and valid_counts.requires_grad:
        raise ValueError("the LSSO CUDA fast path does not support gradients for valid_counts")
    require_available()
    if not torch.is_grad_enabled() or not any(
        value.requires_grad for value in (projected, core_base_raw, core_drive_weight, eta_raw)
    ):
        return torch.ops.lsso_equilibrium.forward_inference(
            projected, core_base_raw, core_drive_weight, eta_raw, centered_positions, valid_counts)
    return _FastMix.apply(projected, core_base_raw, core_drive_weight, eta_raw, centered_positions, valid_counts)


def device_status(reset: bool = True) -> int:
    """Kernel status word of the current device: 0 unless a bounded wait ran out."""
    return _native.device_status(reset)


def check_device_status() -> None:
    """Raise if a kernel of the library gave up waiting since the last check.

    Synchronizes the device.  A kernel whose bounded wait ran out stops,
    frees its resources and leaves its outputs undefined; this reports it
    (once: the status word is reset) so that the caller can discard the
    results of the calls made since the previous check.
    """
    status = _native.device_status(reset=True)
    if status == 2:
        raise RuntimeError(
            "a peer rank did not reach the LSSO gradient exchange within its wait limit (device status 2); the "
            "exchanged gradients since the last check are undefined")
    if status != 0:
        raise RuntimeError(
            f"an LSSO CUDA kernel gave up waiting (device status {status}); the outputs of the calls since the "
            "last check are undefined")


__all__ = ["check_device_status", "device_status", "fast_mix", "is_available", "load", "require_available"]
