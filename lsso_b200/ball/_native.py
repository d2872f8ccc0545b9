"""ctypes binding of ``lsso_equilibrium_sm100.so`` and the ``lsso_equilibrium`` operators.

The native library is a plain C ABI (``include/lsso_equilibrium.h``).  This
module validates tensors with the reference's messages
(csrc/ball/common.cuh:194-269, backward.cu:289-320), allocates outputs and
workspace with PyTorch's caching allocator, passes raw pointers and the
current stream, and registers the four reference operators
(csrc/ball/binding.cpp:79-107) with ``torch.library`` so that
``torch.ops.lsso_equilibrium.*`` behave as in the reference, including the
two autograd-key rejections.  Registration happens once per process, from
``lsso_b200.ball.cuda.load()``.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

import torch

CONTRACT_VERSION = 8
EXPORTED_SYMBOLS = (
    "lsso_contract_version", "lsso_compiled_sm", "lsso_check_device", "lsso_last_error", "lsso_device_status",
    "lsso_set_wait_limit_ns",
    "lsso_tape_stride", "lsso_forward_workspace_size", "lsso_forward", "lsso_backward_workspace_size",
    "lsso_backward", "lsso_profile_start", "lsso_profile_stop", "lsso_forward_inference_noalloc",
    "lsso_linear_workspace_size", "lsso_linear", "lsso_linear_image_size", "lsso_linear_prepare",
    "lsso_linear_prepared", "lsso_linear_wgrad_workspace_size", "lsso_linear_wgrad",
    "lsso_moment_elements", "lsso_forward_moments", "lsso_forward_finish", "lsso_backward_moments",
    "lsso_backward_finish", "lsso_peer_region_bytes", "lsso_peer_region_create", "lsso_peer_region_open",
    "lsso_peer_region_close", "lsso_peer_region_destroy", "lsso_peer_allreduce", "lsso_backward_with_wgrad",
)

_LIBRARY: "NativeLibrary | None" = None
_OPS: torch.library.Library | None = None


class NativeLibrary:
    """Typed handle on the shared library."""

    def __init__(self, path: str | Path) -> None:
        c = ctypes
        lib = c.CDLL(str(path))
        i64, vp, sz, ci = c.c_int64, c.c_void_p, c.c_size_t, c.c_int
        signatures = {
            "lsso_contract_version": (ci, []),
            "lsso_compiled_sm": (ci, []),
            "lsso_check_device": (ci, [ci]),
            "lsso_last_error": (c.c_char_p, []),
            "lsso_device_status": (ci, [ci]),
            "lsso_set_wait_limit_ns": (ci, [c.c_ulonglong]),
            "lsso_tape_stride": (i64, [i64, i64, i64, i64]),
            "lsso_forward_workspace_size": (sz, [i64, i64, i64, i64, i64, ci, ci]),
            "lsso_forward": (ci, [vp, vp, vp, vp, vp, ci, vp, i64, i64, i64, i64, i64, vp, vp, vp, vp, sz, vp]),
            "lsso_backward_workspace_size": (sz, [i64, i64, i64, i64, i64, ci]),
            "lsso_backward": (ci, [vp, vp, vp, vp, vp, vp, vp, vp, ci, vp, i64, i64, i64, i64, i64, vp, vp, vp, vp,
                                   vp, sz, vp]),
            "lsso_backward_with_wgrad": (ci, [vp, vp, vp, vp, vp, vp, vp, vp, ci, vp, i64, i64, i64, i64, i64, vp,
                                              vp, vp, vp, vp, sz, vp, ci, vp, ci, vp, i64, i64, i64, vp, vp, sz,
                                              ci, vp]),
            "lsso_linear_workspace_size": (sz, [i64, i64, i64]),
            "lsso_linear": (ci, [vp, ci, i64, i64, vp, ci, i64, vp, vp, vp, ci, i64, vp, sz, vp]),
            "lsso_linear_image_size": (sz, [i64, i64]),
            "lsso_linear_prepare": (ci, [ci, c.POINTER(vp), c.POINTER(ci), c.POINTER(i64), c.POINTER(i64),
                                         c.POINTER(vp), vp]),
            "lsso_linear_prepared": (ci, [vp, ci, i64, i64, vp, i64, vp, vp, vp, ci, i64, ci, vp]),
            "lsso_linear_wgrad_workspace_size": (sz, [i64, i64, i64]),
            "lsso_linear_wgrad": (ci, [vp, ci, vp, ci, vp, i64, i64, i64, vp, vp, sz, vp]),
            "lsso_forward_inference_noalloc": (ci, [vp, vp, vp, vp, vp, ci, vp, i64, i64, i64, i64, i64, vp, vp]),
            "lsso_moment_elements": (sz, [i64, i64, i64, i64, i64, ci]),
            "lsso_forward_moments": (ci, [vp, vp, ci, i64, i64, i64, i64, i64, vp, vp, sz, vp]),
            "lsso_forward_finish": (ci, [vp, vp, vp, vp, vp, ci, vp, i64, i64, i64, i64, i64, vp, vp, vp, vp, vp,
                                         sz, vp]),
            "lsso_backward_moments": (ci, [vp, vp, vp, ci, i64, i64, i64, i64, i64, vp, vp, sz, vp]),
            "lsso_backward_finish": (ci, [vp, vp, vp, vp, vp, vp, ci, i64, i64, i64, i64, i64, vp, c.c_float, vp,
                                          vp, vp, vp, vp, sz, vp]),
            "lsso_peer_region_bytes": (sz, [i64]),
            "lsso_peer_region_create": (ci, [i64, c.POINTER(vp), c.c_char_p]),
            "lsso_peer_region_open": (ci, [c.c_char_p, c.POINTER(vp)]),
            "lsso_peer_region_close": (ci, [vp]),
            "lsso_peer_region_destroy": (ci, [vp]),
            "lsso_peer_allreduce": (ci, [c.POINTER(vp), ci, ci, i64, i64, c.c_float, vp, c.c_ulonglong, vp]),
            "lsso_profile_start": (ci, []),
            "lsso_profile_stop": (ci, [ci, c.c_char_p, c.POINTER(c.c_float), c.POINTER(c.c_int)]),
        }
        for name, (restype, argtypes) in signatures.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        self.lib = lib
        self.path = Path(path)

    def last_error(self) -> str:
        message = self.lib.lsso_last_error()
        return message.decode() if message else ""

    def check(self, code: int) -> None:
        if code != 0:
            raise RuntimeError(self.last_error() or f"lsso native call failed with code {code}")


def library() -> NativeLibrary:
    if _LIBRARY is None:
        raise RuntimeError("the LSSO CUDA extension is not loaded; call lsso.ball.cuda.load()")
    return _LIBRARY


def open_library(path: str | Path) -> NativeLibrary:
    """Open the shared library (no device work); used by load() and the ABI tests."""
    return NativeLibrary(path)


# ---------------------------------------------------------------------------- validation
def _same_device(value: torch.Tensor, projected: torch.Tensor, name: str) -> None:
    if not value.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor")
    if value.device != projected.device:
        raise RuntimeError(f"{name} must share projected.device() (got {value.device} vs {projected.device})")


def validate_fast_inputs(projected, core_base_raw, core_drive_weight, eta_raw, centered_positions, valid_counts):
    """Shape/dtype/device contract of the native mixer; returns (B, N, H, D, R)."""
    if not projected.is_cuda:
        raise RuntimeError("projected must be a CUDA tensor")
    if not projected.is_contiguous():
        raise RuntimeError("projected must be contiguous [B, N, H*R + D]")
    if projected.dim() != 3:
        raise RuntimeError(f"projected must have shape [B, N, H*R + D], got {list(projected.shape)}")
    if projected.dtype != torch.bfloat16:
        raise RuntimeError(
            f"projected must use bfloat16 under the mixed precision CUDA contract, got {projected.dtype}"
        )
    for name, value in (("core_base_raw", core_base_raw), ("core_drive_weight", core_drive_weight),
                        ("eta_raw", eta_raw)):
        if not value.is_contiguous():
            raise RuntimeError(f"{name} must be contiguous")
        _same_device(value, projected, name)
        if value.dtype != torch.float32:
            raise RuntimeError(f"{name} must use float32")
    if core_base_raw.dim() != 3 or core_base_raw.shape[1] != core_base_raw.shape[2]:
        raise RuntimeError(f"core_base_raw must have shape [H, R, R], got {list(core_base_raw.shape)}")
    batch, length, width = projected.shape
    heads, rank = core_base_raw.shape[0], core_base_raw.shape[1]
    if batch <= 0 or length <= 0 or heads <= 0:
        raise RuntimeError("B, N, and H must be positive")
    if rank not in (16, 32, 48, 64):
        raise RuntimeError(f"the CUDA fast path supports rank in {{16, 32, 48, 64}}, got {rank}")
    if width <= heads * rank:
        raise RuntimeError("projected width must exceed H*R for a nonempty content channel")
    dim = width - heads * rank
    if dim % heads:
        raise RuntimeError("projected content width D must be divisible by H")
    head_dim = dim // heads
    if tuple(core_drive_weight.shape) != (heads, head_dim, rank):
        raise RuntimeError(f"core_drive_weight must have shape [H, D/H, R], got {list(core_drive_weight.shape)}")
    if tuple(eta_raw.shape) != (heads,):
        raise RuntimeError(f"eta_raw must have shape [H], got {list(eta_raw.shape)}")
    if centered_positions is not None:
        _same_device(centered_positions, projected, "centered_positions")
        if not centered_positions.is_contiguous():
            raise RuntimeError("centered_positions must be contiguous")
        if centered_positions.dtype != torch.float32:
            raise RuntimeError("centered_positions must use float32")
        shape = tuple(centered_positions.shape)
        if shape not in ((length,), (batch, length)):
            raise RuntimeError(f"centered_positions must have shape [N] or [B, N], got {list(shape)}")
    if valid_counts is not None:
        _same_device(valid_counts, projected, "valid_counts")
        if not valid_counts.is_contiguous():
            raise RuntimeError("valid_counts must be contiguous")
        if valid_counts.dtype != torch.float32:
            raise RuntimeError("valid_counts must use float32")
        if tuple(valid_counts.shape) != (batch,):
            raise RuntimeError(f"valid_counts must have shape [B], got {list(valid_counts.shape)}")
    return batch, length, heads, dim, rank


def _ptr(value: torch.Tensor | None):
    return None if value is None else value.data_ptr()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


# ---------------------------------------------------------------------------- operator bodies
def forward(projected, core_base_raw, core_drive_weight, eta_raw, centered_positions, valid_counts, *, train: bool):
    """Run the native forward; returns (mixed, tape, pivots) (tape/pivots None unless train)."""
    lib = library()
    batch, length, heads, dim, rank = validate_fast_inputs(
        projected, core_base_raw, core_drive_weight, eta_raw, centered_positions, valid_counts)
    device = projected.device
    batched = centered_positions is not None and centered_positions.dim() == 2
    with torch.cuda.device(device):
        mixed = torch.empty((batch, length, dim), dtype=torch.bfloat16, device=device)
        tape = pivots = None
        if train:
            stride = lib.lib.lsso_tape_stride(length, heads, dim, rank)
            tape = torch.empty((batch * heads, stride), dtype=torch.float32, device=device)
            pivots = torch.empty((batch * heads, rank), dtype=torch.int32, device=device)
        size = lib.lib.lsso_forward_workspace_size(batch, length, heads, dim, rank, int(batched), int(train))
        if size == 0:
            lib.check(1)
        workspace = torch.empty((size,), dtype=torch.uint8, device=device)
        lib.check(lib.lib.lsso_forward(
            _ptr(projected), _ptr(core_base_raw), _ptr(core_drive_weight), _ptr(eta_raw), _ptr(centered_positions),
            int(batched), _ptr(valid_counts), batch, length, heads, dim, rank, _ptr(mixed), _ptr(tape), _ptr(pivots),
            _ptr(workspace), size, _stream(device)))
    return mixed, tape, pivots


def backward(grad_output, projected, core_base_raw, core_drive_weight, eta_raw, tape, pivots, centered_positions,
             valid_counts, wgrad=None):
    """Run the native backward; returns the four gradients.

    ``wgrad``: optionally ``(g, x, row_mask, dw, concurrent)``, one projection
    weight gradient ``dw = bf16(g)^T bf16(x)`` (g ``[T, Nout]``, x ``[T, K]``,
    FP16 / BF16, contiguous; dw a contiguous FP32 ``[Nout, K]`` it writes)
    computed in the same call (``lsso_backward_with_wgrad``): with
    ``concurrent`` its kernels share the SMs with the backward's solves.
    """
    lib = library()
    batch, length, heads, dim, rank = validate_fast_inputs(
        projected, core_base_raw, core_drive_weight, eta_raw, centered_positions, valid_counts)
    _same_device(grad_output, projected, "grad_output")
    if not grad_output.is_contiguous():
        raise RuntimeError("grad_output must be contiguous")
    if grad_output.dtype != torch.bfloat16:
        raise RuntimeError("grad_output must use bfloat16")
    if tuple(grad_output.shape) != (batch, length, dim):
        raise RuntimeError(f"grad_output must have shape [B, N, D], got {list(grad_output.shape)}")
    stride = lib.lib.lsso_tape_stride(length, heads, dim, rank)
    _same_device(tape, projected, "tape")
    _same_device(pivots, projected, "pivots")
    if not tape.is_contiguous():
        raise RuntimeError("tape must be contiguous")
    if tape.dtype != torch.float32:
        raise RuntimeError("tape must use float32")
    if tuple(tape.shape) != (batch * heads, stride):
        raise RuntimeError(f"tape has an incompatible shape {list(tape.shape)}")
    if not pivots.is_contiguous():
        raise RuntimeError("pivots must be contiguous")
    if pivots.dtype != torch.int32:
        raise RuntimeError("pivots must use int32")
    if tuple(pivots.shape) != (batch * heads, rank):
        raise RuntimeError(f"pivots has an incompatible shape {list(pivots.shape)}")
    device = projected.device
    batched = centered_positions is not None and centered_positions.dim() == 2
    with torch.cuda.device(device):
        grad_projected = torch.empty_like(projected)
        grad_base = torch.empty_like(core_base_raw)
        grad_drive = torch.empty_like(core_drive_weight)
        grad_eta = torch.empty_like(eta_raw)
        size = lib.lib.lsso_backward_workspace_size(batch, length, heads, dim, rank, int(batched))
        if size == 0:
            lib.check(1)
        workspace = torch.empty((size,), dtype=torch.uint8, device=device)
        if wgrad is None:
            lib.check(lib.lib.lsso_backward(
                _ptr(grad_output), _ptr(projected), _ptr(core_base_raw), _ptr(core_drive_weight), _ptr(eta_raw),
                _ptr(tape), _ptr(pivots), _ptr(centered_positions), int(batched), _ptr(valid_counts), batch,
                length, heads, dim, rank, _ptr(grad_projected), _ptr(grad_base), _ptr(grad_drive), _ptr(grad_eta),
                _ptr(workspace), size, _stream(device)))
        else:
            g, x, row_mask, dw, concurrent = wgrad
            for name, value in (("wgrad g", g), ("wgrad x", x), ("wgrad dw", dw)):
                _same_device(value, projected, name)
                if not value.is_contiguous():
                    raise RuntimeError(f"{name} must be contiguous")
            if g.dtype not in (torch.float16, torch.bfloat16) or x.dtype not in (torch.float16, torch.bfloat16):
                raise RuntimeError("wgrad g and x must use float16 or bfloat16")
            if dw.dtype != torch.float32:
                raise RuntimeError("wgrad dw must use float32")
            tokens, nout, k = g.shape[0], g.shape[-1], x.shape[-1]
            if g.dim() != 2 or x.dim() != 2 or x.shape[0] != tokens or tuple(dw.shape) != (nout, k):
                raise RuntimeError("wgrad expects g [T, Nout], x [T, K] and dw [Nout, K]")
            mask = None if row_mask is None else row_mask.reshape(-1).contiguous().view(torch.uint8)
            wsize = lib.lib.lsso_linear_wgrad_workspace_size(tokens, nout, k)
            if wsize == 0:
                lib.check(1)
            wspace = torch.empty((wsize,), dtype=torch.uint8, device=device)
            lib.check(lib.lib.lsso_backward_with_wgrad(
                _ptr(grad_output), _ptr(projected), _ptr(core_base_raw), _ptr(core_drive_weight), _ptr(eta_raw),
                _ptr(tape), _ptr(pivots), _ptr(centered_positions), int(batched), _ptr(valid_counts), batch,
                length, heads, dim, rank, _ptr(grad_projected), _ptr(grad_base), _ptr(grad_drive), _ptr(grad_eta),
                _ptr(workspace), size, _ptr(g), 1 if g.dtype == torch.float16 else 0, _ptr(x),
                1 if x.dtype == torch.float16 else 0, _ptr(mask), tokens, nout, k, _ptr(dw), _ptr(wspace), wsize,
                int(bool(concurrent)), _stream(device)))
    return grad_projected, grad_base, grad_drive, grad_eta


# ---------------------------------------------------------------------------- sequence-parallel halves
def _sequence_inputs(projected, centered_positions, valid_counts, need_counts: bool):
    if centered_positions is None:
        raise RuntimeError("the sequence-parallel mixer needs the centered positions of this rank's tokens")
    if need_counts and valid_counts is None:
        raise RuntimeError("the sequence-parallel mixer needs the valid-token counts of the whole sequence")
    return centered_positions.dim() == 2


def moment_elements(batch, length, heads, dim, rank, *, backward: bool) -> int:
    lib = library()
    count = lib.lib.lsso_moment_elements(batch, length, heads, dim, rank, int(backward))
    if count == 0:
        lib.check(1)
    return int(count)


def forward_moments(projected, core_base_raw, core_drive_weight, eta_raw, centered_positions):
    """This rank's forward moment sums (FP32, flat); sum them over the ranks before forward_finish."""
    lib = library()
    batch, length, heads, dim, rank = validate_fast_inputs(
        projected, core_base_raw, core_drive_weight, eta_raw, centered_positions, None)
    batched = _sequence_inputs(projected, centered_positions, None, False)
    device = projected.device
    with torch.cuda.device(device):
        moments = torch.empty((moment_elements(batch, length, heads, dim, rank, backward=False),),
                              dtype=torch.float32, device=device)
        size = lib.lib.lsso_forward_workspace_size(batch, length, heads, dim, rank, int(batched), 1)
        if size == 0:
            lib.check(1)
        workspace = torch.empty((size,), dtype=torch.uint8, device=device)
        lib.check(lib.lib.lsso_forward_moments(
            _ptr(projected), _ptr(centered_positions), int(batched), batch, length, heads, dim, rank, _ptr(moments),
            _ptr(workspace), size, _stream(device)))
    return moments


def forward_finish(projected, core_base_raw, core_drive_weight, eta_raw, centered_positions, valid_counts, moments,
                   *, train: bool):
    """Solves from the summed moments and this rank's readout; returns (mixed, tape, pivots)."""
    lib = library()
    batch, length, heads, dim, rank = validate_fast_inputs(
        projected, core_base_raw, core_drive_weight, eta_raw, centered_positions, valid_counts)
    batched = _sequence_inputs(projected, centered_positions, valid_counts, True)
    _check_moments(moments, projected, moment_elements(batch, length, heads, dim, rank, backward=False))
    device = projected.device
    with torch.cuda.device(device):
        mixed = torch.empty((batch, length, dim), dtype=torch.bfloat16, device=device)
        tape = pivots = None
        if train:
            stride = lib.lib.lsso_tape_stride(length, heads, dim, rank)
            tape = torch.empty((batch * heads, stride), dtype=torch.float32, device=device)
            pivots = torch.empty((batch * heads, rank), dtype=torch.int32, device=device)
        size = lib.lib.lsso_forward_workspace_size(batch, length, heads, dim, rank, int(batched), int(train))
        if size == 0:
            lib.check(1)
        workspace = torch.empty((size,), dtype=torch.uint8, device=device)
        lib.check(lib.lib.lsso_forward_finish(
            _ptr(projected), _ptr(core_base_raw), _ptr(core_drive_weight), _ptr(eta_raw), _ptr(centered_positions),
            int(batched), _ptr(valid_counts), batch, length, heads, dim, rank, _ptr(moments), _ptr(mixed), _ptr(tape),
            _ptr(pivots), _ptr(workspace), size, _stream(device)))
    return mixed, tape, pivots


def backward_moments(grad_output, projected, core_base_raw, core_drive_weight, eta_raw, centered_positions):
    """This rank's backward moment sums (FP32, flat); sum them over the ranks before backward_finish."""
    lib = library()
    batch, length, heads, dim, rank = validate_fast_inputs(
        projected, core_base_raw, core_drive_weight, eta_raw, centered_positions, None)
    batched = _sequence_inputs(projected, centered_positions, None, False)
    _check_grad_output(grad_output, projected, batch, length, dim)
    device = projected.device
    with torch.cuda.device(device):
        moments = torch.empty((moment_elements(batch, length, heads, dim, rank, backward=True),),
                              dtype=torch.float32, device=device)
        size = lib.lib.lsso_backward_workspace_size(batch, length, heads, dim, rank, int(batched))
        if size == 0:
            lib.check(1)
        workspace = torch.empty((size,), dtype=torch.uint8, device=device)
        lib.check(lib.lib.lsso_backward_moments(
            _ptr(grad_output), _ptr(projected), _ptr(centered_positions), int(batched), batch, length, heads, dim,
            rank, _ptr(moments), _ptr(workspace), size, _stream(device)))
    return moments


def backward_finish(grad_output, projected, core_base_raw, core_drive_weight, eta_raw, tape, centered_positions,
                    moments, redundant: float):
    """Backward solves from the summed moments, this rank's gradient pass and the parameter gradients."""
    lib = library()
    batch, length, heads, dim, rank = validate_fast_inputs(
        projected, core_base_raw, core_drive_weight, eta_raw, centered_positions, None)
    batched = _sequence_inputs(projected, centered_positions, None, False)
    _check_grad_output(grad_output, projected, batch, length, dim)
    _check_moments(moments, projected, moment_elements(batch, length, heads, dim, rank, backward=True))
    stride = lib.lib.lsso_tape_stride(length, heads, dim, rank)
    _same_device(tape, projected, "tape")
    if tape.dtype != torch.float32 or not tape.is_contiguous() or tuple(tape.shape) != (batch * heads, stride):
        raise RuntimeError(f"tape has an incompatible shape or dtype {list(tape.shape)} {tape.dtype}")
    device = projected.device
    with torch.cuda.device(device):
        grad_projected = torch.empty_like(projected)
        grad_base = torch.empty_like(core_base_raw)
        grad_drive = torch.empty_like(core_drive_weight)
        grad_eta = torch.empty_like(eta_raw)
        size = lib.lib.lsso_backward_workspace_size(batch, length, heads, dim, rank, int(batched))
        if size == 0:
            lib.check(1)
        workspace = torch.empty((size,), dtype=torch.uint8, device=device)
        lib.check(lib.lib.lsso_backward_finish(
            _ptr(grad_output), _ptr(projected), _ptr(core_drive_weight), _ptr(eta_raw), _ptr(tape),
            _ptr(centered_positions), int(batched), batch, length, heads, dim, rank, _ptr(moments), float(redundant),
            _ptr(grad_projected), _ptr(grad_base), _ptr(grad_drive), _ptr(grad_eta), _ptr(workspace), size,
            _stream(device)))
    return grad_projected, grad_base, grad_drive, grad_eta


def _check_moments(moments, projected, count: int) -> None:
    _same_device(moments, projected, "moments")
    if moments.dtype != torch.float32 or not moments.is_contiguous() or moments.numel() != count:
        raise RuntimeError(f"moments must be a contiguous float32 buffer of {count} elements")


def _check_grad_output(grad_output, projected, batch, length, dim) -> None:
    _same_device(grad_output, projected, "grad_output")
    if not grad_output.is_contiguous():
        raise RuntimeError("grad_output must be contiguous")
    if grad_output.dtype != torch.bfloat16:
        raise RuntimeError("grad_output must use bfloat16")
    if tuple(grad_output.shape) != (batch, length, dim):
        raise RuntimeError(f"grad_output must have shape [B, N, D], got {list(grad_output.shape)}")


# ---------------------------------------------------------------------------- operator registration
def _requires_grad(*values) -> bool:
    return any(v is not None and v.requires_grad for v in values)


def _forward_inference_cuda(projected, core_base_raw, core_drive_weight, eta_raw, centered_positions=None,
                            valid_counts=None):
    return forward(projected, core_base_raw, core_drive_weight, eta_raw, centered_positions, valid_counts,
                   train=False)[0]


def _forward_train_cuda(projected, core_base_raw, core_drive_weight, eta_raw, centered_positions=None,
                        valid_counts=None):
    return forward(projected, core_base_raw, core_drive_weight, eta_raw, centered_positions, valid_counts,
                   train=True)


def _backward_cuda(grad_output, projected, core_base_raw, core_drive_weight, eta_raw, tape, pivots,
                   centered_positions=None, valid_counts=None):
    return backward(grad_output, projected, core_base_raw, core_drive_weight, eta_raw, tape, pivots,
                    centered_positions, valid_counts)


def _forward_inference_autograd(projected, core_base_raw, core_drive_weight, eta_raw, centered_positions=None,
                                valid_counts=None):
    if torch.is_grad_enabled() and _requires_grad(projected, core_base_raw, core_drive_weight, eta_raw,
                                                  centered_positions, valid_counts):
        raise RuntimeError(
            "lsso_equilibrium::forward_inference is an inference-only entry point and cannot participate in "
            "autograd directly; use lsso.ball.cuda.fast_mix()"
        )
    with torch._C._AutoDispatchBelowAutograd():
        return torch.ops.lsso_equilibrium.forward_inference(projected, core_base_raw, core_drive_weight, eta_raw,
                                                            centered_positions, valid_counts)


def _forward_train_autograd(projected, core_base_raw, core_drive_weight, eta_raw, centered_positions=None,
                            valid_counts=None):
    if torch.is_grad_enabled() and _requires_grad(projected, core_base_raw, core_drive_weight, eta_raw,
                                                  centered_positions, valid_counts):
        raise RuntimeError(
            "lsso_equilibrium::forward_train is a private tape-producing entry point and cannot participate in "
            "autograd directly; use lsso.ball.cuda.fast_mix()"
        )
    with torch._C._AutoDispatchBelowAutograd():
        return torch.ops.lsso_equilibrium.forward_train(projected, core_base_raw, core_drive_weight, eta_raw,
                                                        centered_positions, valid_counts)


def _backward_autograd(*args):
    with torch._C._AutoDispatchBelowAutograd():
        return torch.ops.lsso_equilibrium.backward(*args)


def _contract_version() -> int:
    return CONTRACT_VERSION


def register(path: str | Path) -> NativeLibrary:
    """Open the library and register the operators (idempotent per process)."""
    global _LIBRARY, _OPS
    if _LIBRARY is not None:
        return _LIBRARY
    lib = open_library(path)
    version = lib.lib.lsso_contract_version()
    if version != CONTRACT_VERSION:
        raise RuntimeError(
            f"the loaded LSSO CUDA extension has native contract version {version}, but this package requires "
            f"{CONTRACT_VERSION}; rebuild it with python -m lsso_b200.build and restart the process"
        )
    ops = torch.library.Library("lsso_equilibrium", "DEF")
    ops.define("contract_version() -> int")
    ops.define("forward_inference(Tensor projected, Tensor core_base_raw, Tensor core_drive_weight, "
               "Tensor eta_raw, Tensor? centered_positions=None, Tensor? valid_counts=None) -> Tensor")
    ops.define("forward_train(Tensor projected, Tensor core_base_raw, Tensor core_drive_weight, "
               "Tensor eta_raw, Tensor? centered_positions=None, Tensor? valid_counts=None) "
               "-> (Tensor, Tensor, Tensor)")
    ops.define("backward(Tensor grad_output, Tensor projected, Tensor core_base_raw, "
               "Tensor core_drive_weight, Tensor eta_raw, Tensor tape, Tensor pivots, "
               "Tensor? centered_positions=None, Tensor? valid_counts=None) -> (Tensor, Tensor, Tensor, Tensor)")
    ops.impl("contract_version", _contract_version, "CompositeExplicitAutograd")
    ops.impl("forward_inference", _forward_inference_cuda, "CUDA")
    ops.impl("forward_train", _forward_train_cuda, "CUDA")
    ops.impl("backward", _backward_cuda, "CUDA")
    ops.impl("forward_inference", _forward_inference_autograd, "Autograd")
    ops.impl("forward_train", _forward_train_autograd, "Autograd")
    ops.impl("backward", _backward_autograd, "Autograd")
    _OPS = ops
    _LIBRARY = lib
    return lib


def profile_start() -> None:
    """Start per-kernel event timing of the library's launches (instrumentation)."""
    library().lib.lsso_profile_start()


def profile_stop() -> dict[str, tuple[float, int]]:
    """Stop timing; return {kernel: (total milliseconds, launches)} (synchronizes)."""
    capacity = 64
    names = ctypes.create_string_buffer(32 * capacity)
    totals = (ctypes.c_float * capacity)()
    launches = (ctypes.c_int * capacity)()
    count = library().lib.lsso_profile_stop(capacity, names, totals, launches)
    if count < 0:
        raise RuntimeError("lsso_profile_stop failed")
    raw = names.raw
    out = {}
    for k in range(min(count, capacity)):
        name = raw[32 * k: 32 * k + 32].split(b"\0", 1)[0].decode()
        out[name] = (float(totals[k]), int(launches[k]))
    return out


def device_status(reset: bool = True) -> int:
    """Kernel status word of the current device (synchronizes); 0 when no kernel reported a failure."""
    return library().lib.lsso_device_status(int(reset))


def set_wait_limit_ns(limit_ns: int) -> None:
    """Test hook: time limit of the tensor-core kernels' pipeline waits on the
    current device (0 restores the default of one second)."""
    lib = library()
    lib.check(lib.lib.lsso_set_wait_limit_ns(int(limit_ns)))


__all__ = ["CONTRACT_VERSION", "EXPORTED_SYMBOLS", "NativeLibrary", "backward", "device_status", "forward",
           "library", "open_library", "profile_start", "profile_stop", "register", "set_wait_limit_ns",
           "validate_fast_inputs"]
