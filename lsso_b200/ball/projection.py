"""Input and output projections of the CUDA path (reference model.py:370-404).

Input projection: ``projected = bf16(x) bf16(W_bc)^T (+ FP32 bias)`` rounded
once to BF16, masked rows zero.  Output projection:
``y = bf16(mixed) bf16(W_o)^T (+ FP32 bias)`` stored in ``x.dtype``, masked
rows zero.  Both run on the library's tcgen05 GEMM (``lsso_linear``): BF16
multiplicands, FP32 accumulation and bias, a single final rounding, the mask
applied in the epilogue.  The first-order VJP follows the reference's
``_TensorCoreLinear`` (reference.py:170-247): the input gradient is
``bf16(g) bf16(W)`` stored in the input's dtype (same GEMM), the weight
gradient ``bf16(g)^T bf16(x)`` in FP32 and the bias gradient an FP32 sum.
"""

from __future__ import annotations

import ctypes

import torch
import torch.nn.functional as F
from torch.autograd.function import once_differentiable
from torch.utils.weak import WeakIdKeyDictionary

from . import _native

_OUT_CODES = {torch.bfloat16: 0, torch.float16: 1, torch.float32: 2}

# Parameters whose gradient has a preassigned slot (a gradient exchange's flat
# buffer): parameter -> (slot tensor, callback(parameter) run once written).
# (Keyed by identity: tensors compare elementwise.)
_GRADIENT_SLOTS = WeakIdKeyDictionary()


def register_gradient_slot(parameter: torch.Tensor, slot: torch.Tensor | None, on_written=None) -> None:
    """Have the projection backward write ``parameter``'s gradient into ``slot``
    (same shape, FP32) whenever ``parameter.grad`` is None at that point, and
    call ``on_written(parameter)`` right after -- before the input-gradient
    GEMM, so whoever owns the slot can start exchanging it under that GEMM.
    ``slot=None`` removes the registration."""
    if slot is None:
        _GRADIENT_SLOTS.pop(parameter, None)
    else:
        _GRADIENT_SLOTS[parameter] = (slot, on_written)


def _slot_for(parameter: torch.Tensor | None):
    if parameter is None or parameter.grad is not None:
        return None
    return _GRADIENT_SLOTS.get(parameter)


def _pad_features(value: torch.Tensor, multiple: int = 8) -> torch.Tensor:
    extra = (-value.shape[-1]) % multiple
    return value if extra == 0 else F.pad(value, (0, extra))


def prepare_images(specs: list[tuple[torch.Tensor, bool]]) -> list[torch.Tensor]:
    """BF16 tensor-core images of FP32 weights, all converted in one kernel launch.

    ``specs`` holds up to four ``(weight, transposed)`` pairs: ``weight`` FP32
    ``[Nout, K]`` for ``a W^T`` (``transposed=False``) or ``[K, Nout]`` read as
    ``a W`` (``transposed=True``), K and Nout multiples of 8.  Returns one
    uint8 image per pair for :func:`linear`'s ``image`` argument.
    """
    lib = _native.library()
    device = specs[0][0].device
    weights, sizes, shapes = [], [], []
    with torch.cuda.device(device):
        for weight, transposed in specs:
            w = weight.detach().float().contiguous()
            k, nout = (w.shape[0], w.shape[1]) if transposed else (w.shape[1], w.shape[0])
            size = lib.lib.lsso_linear_image_size(k, nout)
            if size == 0:
                lib.check(1)
            weights.append(w)
            sizes.append((size + 255) // 256 * 256)
            shapes.append((k, nout, int(transposed)))
        buffer = torch.empty((sum(sizes),), dtype=torch.uint8, device=device)
        images = list(buffer.split(sizes))
        n = len(specs)
        vp, ci, i64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64
        lib.check(lib.lib.lsso_linear_prepare(
            n, (vp * n)(*[w.data_ptr() for w in weights]), (ci * n)(*[t for _, _, t in shapes]),
            (i64 * n)(*[k for k, _, _ in shapes]), (i64 * n)(*[o for _, o, _ in shapes]),
            (vp * n)(*[im.data_ptr() for im in images]), torch.cuda.current_stream(device).cuda_stream))
    return images


def layer_images(w_bc: torch.Tensor, w_o: torch.Tensor, backward: bool) -> dict | None:
    """The four weight images of one layer step (one launch), or None when a
    feature width is not a multiple of 8 (the per-call conversion then runs)."""
    if any(n % 8 for n in (*w_bc.shape, *w_o.shape)):
        return None
    specs = [(w_bc, False), (w_o, False)] + ([(w_o, True), (w_bc, True)] if backward else [])
    images = prepare_images(specs)
    names = ("bc", "o", "o_t", "bc_t")
    return dict(zip(names, images))


def linear(a: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None, row_mask: torch.Tensor | None,
           out_dtype: torch.dtype, *, weight_transposed: bool = False, image: torch.Tensor | None = None,
           reverse: bool = False) -> torch.Tensor:
    """One native GEMM: ``a [.., K] (BF16/FP16) x W -> [.., Nout]`` in ``out_dtype``.

    ``weight`` is FP32 ``[Nout, K]`` (or ``[K, Nout]`` with ``weight_transposed``).
    ``image``: the same weight already converted by :func:`prepare_images` in
    this orientation (then no conversion kernel runs; the result is identical).
    ``reverse`` (with ``image``): walk the rows of ``a`` from the last to the
    first -- same result; used where the kernel before wrote ``a`` forwards,
    so the rows it wrote last are still in L2 when this product starts.
    """
    lib = _native.library()
    lead = a.shape[:-1]
    k = a.shape[-1]
    if image is not None and k % 8 == 0:
        flat = a.reshape(-1, k).contiguous()
        nout = weight.shape[1] if weight_transposed else weight.shape[0]
        out = torch.empty((flat.shape[0], nout), dtype=out_dtype, device=a.device)
        mask = None if row_mask is None else row_mask.reshape(-1).contiguous().view(torch.uint8)
        with torch.cuda.device(a.device):
            lib.check(lib.lib.lsso_linear_prepared(
                flat.data_ptr(), 1 if flat.dtype == torch.float16 else 0, flat.shape[0], k, image.data_ptr(), nout,
                None if bias is None else bias.detach().float().contiguous().data_ptr(),
                None if mask is None else mask.data_ptr(), out.data_ptr(), _OUT_CODES[out_dtype], nout,
                1 if reverse else 0, torch.cuda.current_stream(a.device).cuda_stream))
        return out.reshape(*lead, nout)
    flat = a.reshape(-1, k)
    w = weight.detach().float()
    if k % 8:
        flat = _pad_features(flat)
        w = F.pad(w, (0, 0, 0, (-k) % 8)) if weight_transposed else _pad_features(w)
    flat = flat.contiguous()
    w = w.contiguous()
    m, kp = flat.shape
    nout = w.shape[1] if weight_transposed else w.shape[0]
    out = torch.empty((m, nout), dtype=out_dtype, device=a.device)
    mask = None
    if row_mask is not None:
        mask = row_mask.reshape(-1).contiguous().view(torch.uint8)
    with torch.cuda.device(a.device):
        size = lib.lib.lsso_linear_workspace_size(m, kp, nout)
        if size == 0:
            lib.check(1)
        workspace = torch.empty((size,), dtype=torch.uint8, device=a.device)
        lib.check(lib.lib.lsso_linear(
            flat.data_ptr(), 1 if flat.dtype == torch.float16 else 0, m, kp, w.data_ptr(), int(weight_transposed),
            nout, None if bias is None else bias.detach().float().contiguous().data_ptr(),
            None if mask is None else mask.data_ptr(), out.data_ptr(), _OUT_CODES[out_dtype], nout,
            workspace.data_ptr(), size, torch.cuda.current_stream(a.device).cuda_stream))
    return out.reshape(*lead, nout)


def weight_gradient(g: torch.Tensor, x: torch.Tensor, row_mask: torch.Tensor | None,
                    out: torch.Tensor | None = None) -> torch.Tensor:
    """``bf16(g)^T bf16(x)`` over valid rows, FP32 ``[Nout, K]`` (native, deterministic).

    ``out``: a contiguous FP32 ``[Nout, K]`` tensor to hold the result (written
    by the kernel itself unless a feature width needs padding)."""
    lib = _native.library()
    nout, k = g.shape[-1], x.shape[-1]
    gf = g.reshape(-1, nout)
    xf = x.reshape(-1, k)
    if gf.dtype not in (torch.float16, torch.bfloat16):
        gf = gf.to(torch.bfloat16)
    if xf.dtype not in (torch.float16, torch.bfloat16):
        xf = xf.to(torch.bfloat16)
    gf = _pad_features(gf).contiguous()
    xf = _pad_features(xf).contiguous()
    t, np_, kp = gf.shape[0], gf.shape[1], xf.shape[1]
    mask = None if row_mask is None else row_mask.reshape(-1).contiguous().view(torch.uint8)
    direct = out is not None and (np_, kp) == (nout, k) and out.is_contiguous() and out.dtype == torch.float32
    dw = out if direct else torch.empty((np_, kp), dtype=torch.float32, device=g.device)
    with torch.cuda.device(g.device):
        size = lib.lib.lsso_linear_wgrad_workspace_size(t, np_, kp)
        if size == 0:
            lib.check(1)
        workspace = torch.empty((size,), dtype=torch.uint8, device=g.device)
        lib.check(lib.lib.lsso_linear_wgrad(
            gf.data_ptr(), 1 if gf.dtype == torch.float16 else 0, xf.data_ptr(),
            1 if xf.dtype == torch.float16 else 0, None if mask is None else mask.data_ptr(), t, np_, kp,
            dw.data_ptr(), workspace.data_ptr(), size, torch.cuda.current_stream(g.device).cuda_stream))
    result = dw[:nout, :k] if (np_ != nout or kp != k) else dw
    if out is not None and not direct:
        out.copy_(result)
        return out
    return result


class _ProjectionFunction(torch.autograd.Function):
    """``value W^T + bias``; ``image`` / ``image_t`` are the weight's prepared
    images for the forward and for the input-gradient product (both made at
    forward time, as the reference keeps its BF16 weight copy for the backward)."""

    @staticmethod
    def forward(ctx, value, weight, bias, row_mask, out_dtype, image, image_t, reverse):
        if value.dtype not in (torch.float16, torch.bfloat16):
            value = value.to(torch.bfloat16)
        out = linear(value, weight, bias, row_mask, out_dtype, image=image, reverse=reverse)
        ctx.save_for_backward(value, weight, row_mask, image_t)
        ctx.reverse = reverse
        ctx.has_bias = bias is not None
        ctx.bias_meta = None if bias is None else (bias.dtype, bias.device)
        ctx.bias_param = bias
        return out

    @staticmethod
    @once_differentiable
    def backward(ctx, grad_output):
        value, weight, row_mask, image_t = ctx.saved_tensors
        grads = _linear_vjp(grad_output, value, weight, row_mask, ctx.needs_input_grad[:3],
                            ctx.bias_meta if ctx.has_bias else None, image_t, ctx.bias_param, ctx.reverse)
        return (*grads, None, None, None, None, None)


def _linear_vjp(grad_output, value, weight, row_mask, needs, bias_meta, image_t=None, bias=None, reverse=False):
    """(grad_value, grad_weight, grad_bias) of ``value W^T + bias`` (reference.py:170-247).

    The weight and bias gradients come first, into their registered slots when
    they have one (``register_gradient_slot``), whose owners are told before
    the input-gradient GEMM runs.
    """
    g = grad_output
    if g.dtype not in (torch.float16, torch.bfloat16):
        g = g.to(torch.bfloat16)
    g = g.contiguous()
    grad_value = grad_weight = grad_bias = None
    written = []
    # Masked rows: the input-gradient GEMM writes them as zero and the
    # weight-gradient kernel skips them, so only the bias sum masks here.
    if needs[1]:
        wslot = _slot_for(weight)
        grad_weight = weight_gradient(g, value, row_mask, out=None if wslot is None else wslot[0])
        if wslot is not None:
            written.append((weight, wslot[1]))
    if bias_meta is not None and needs[2]:
        dims = tuple(range(grad_output.ndim - 1))
        src = grad_output if row_mask is None else torch.where(row_mask[..., None], grad_output,
                                                               torch.zeros_like(grad_output))
        bslot = _slot_for(bias) if bias_meta[0] == torch.float32 else None
        if bslot is not None and dims:
            grad_bias = torch.sum(src, dim=dims, dtype=torch.float32, out=bslot[0])
            written.append((bias, bslot[1]))
        else:
            total = src.sum(dim=dims, dtype=torch.float32) if dims else src.float()
            grad_bias = total.to(device=bias_meta[1], dtype=bias_meta[0])
    for parameter, on_written in written:
        if on_written is not None:
            on_written(parameter)
    if needs[0]:
        grad_value = linear(g, weight, None, row_mask, value.dtype, weight_transposed=True, image=image_t,
                            reverse=reverse)
    return grad_value, grad_weight, grad_bias


class _MixOutput(torch.autograd.Function):
    """The mixer followed by the output projection, as one autograd node.

    Forward: the mixer's training forward, then ``mixed W_o^T + b_o`` (the
    same calls as ``fast_mix`` followed by :func:`output_projection`).
    Backward: the output projection's input-gradient GEMM (d mixed), then the
    mixer's backward and the output projection's weight gradient in ONE native
    call (``lsso_backward_with_wgrad``).  The weight gradient does not depend
    on the mixer's backward, so the library runs it beside the backward's
    latency-bound per-(sample, head) solves, sharing every SM with them
    (reference order: lsso/ball/reference.py:229-234 computes it in the output
    projection's backward, then csrc/ball/binding.cpp:91-96 runs the mixer's).
    Every result is bit-identical to the separate calls.
    """

    @staticmethod
    def forward(ctx, projected, core_base_raw, core_drive_weight, eta_raw, centered_positions, valid_counts, weight,
                bias, row_mask, out_dtype, image, image_t):
        mixed, tape, pivots = _native.forward(projected, core_base_raw, core_drive_weight, eta_raw,
                                              centered_positions, valid_counts, train=True)
        out = linear(mixed, weight, bias, row_mask, out_dtype, image=image, reverse=True)
        ctx.save_for_backward(projected, core_base_raw, core_drive_weight, eta_raw, tape, pivots, centered_positions,
                              valid_counts, mixed, weight, row_mask, image_t)
        ctx.bias_meta = None if bias is None else (bias.dtype, bias.device)
        ctx.bias_param = bias
        return out

    @staticmethod
    @once_differentiable
    def backward(ctx, grad_output):
        (projected, core_base_raw, core_drive_weight, eta_raw, tape, pivots, centered_positions, valid_counts, mixed,
         weight, row_mask, image_t) = ctx.saved_tensors
        needs = ctx.needs_input_grad
        g = grad_output
        if g.dtype not in (torch.float16, torch.bfloat16):
            g = g.to(torch.bfloat16)
        g = g.contiguous()
        written = []
        grad_bias = None
        if ctx.bias_meta is not None and needs[7]:
            dims = tuple(range(grad_output.ndim - 1))
            src = grad_output if row_mask is None else torch.where(row_mask[..., None], grad_output,
                                                                   torch.zeros_like(grad_output))
            bslot = _slot_for(ctx.bias_param) if ctx.bias_meta[0] == torch.float32 else None
            if bslot is not None and dims:
                grad_bias = torch.sum(src, dim=dims, dtype=torch.float32, out=bslot[0])
                written.append((ctx.bias_param, bslot[1]))
            else:
                total = src.sum(dim=dims, dtype=torch.float32) if dims else src.float()
                grad_bias = total.to(device=ctx.bias_meta[1], dtype=ctx.bias_meta[0])
        grad_weight = None
        wgrad = None
        if needs[6]:
            wslot = _slot_for(weight)
            grad_weight = wslot[0] if wslot is not None else torch.empty(weight.shape, dtype=torch.float32,
                                                                          device=weight.device)
            if wslot is not None:
                written.append((weight, wslot[1]))
            d = mixed.shape[-1]
            wgrad = (g.reshape(-1, g.shape[-1]), mixed.reshape(-1, d), row_mask, grad_weight, CONCURRENT_WGRAD)
        mixer_grads = (None, None, None, None)
        # the weight gradient rides on the mixer backward's call when that runs and the feature
        # widths are multiples of 8; otherwise the separate (padding) weight-gradient call
        fuse = (wgrad is not None and any(needs[:4]) and g.shape[-1] % 8 == 0 and mixed.shape[-1] % 8 == 0)
        if any(needs[:4]):
            grad_mixed = linear(g, weight, None, row_mask, mixed.dtype, weight_transposed=True, image=image_t,
                                reverse=True)
            mixer_grads = _native.backward(grad_mixed, projected, core_base_raw, core_drive_weight, eta_raw, tape,
                                           pivots, centered_positions, valid_counts, wgrad=wgrad if fuse else None)
        if wgrad is not None and not fuse:
            weight_gradient(g, mixed, row_mask, out=grad_weight)
        for parameter, on_written in written:
            if on_written is not None:
                on_written(parameter)
        grad_projected, grad_base, grad_drive, grad_eta = mixer_grads
        return (grad_projected if needs[0] else None, grad_base if needs[1] else None,
                grad_drive if needs[2] else None, grad_eta if needs[3] else None, None, None, grad_weight, grad_bias,
                None, None, None, None)


# The output projection's weight gradient runs beside the backward solves
# (lsso_backward_with_wgrad with concurrent=1).  False: the same kernels one
# after the other (identical results).
CONCURRENT_WGRAD = True


def mix_output(projected, core_base_raw, core_drive_weight, eta_raw, centered_positions, valid_counts, weight,
               bias, dtype: torch.dtype, mask: torch.Tensor | None, images: dict | None = None) -> torch.Tensor:
    """``output_projection(fast_mix(projected, ...), ...)`` as one autograd node (see :class:`_MixOutput`)."""
    from . import cuda as cuda_backend

    images = images or {}
    if centered_positions is not None and centered_positions.requires_grad:
        raise ValueError("the LSSO CUDA fast path does not support gradients for centered_positions")
    if valid_counts is not None and valid_counts.requires_grad:
        raise ValueError("the LSSO CUDA fast path does not support gradients for valid_counts")
    cuda_backend.require_available()
    trains = torch.is_grad_enabled() and any(
        v is not None and v.requires_grad for v in (projected, core_base_raw, core_drive_weight, eta_raw, weight, bias))
    if not trains:
        mixed = cuda_backend.fast_mix(projected, core_base_raw, core_drive_weight, eta_raw, centered_positions,
                                      valid_counts)
        return output_projection(mixed, weight, bias, dtype, mask, images)
    return _MixOutput.apply(projected, core_base_raw, core_drive_weight, eta_raw, centered_positions, valid_counts,
                            weight, bias, mask, dtype, images.get("o"), images.get("o_t"))


def input_projection(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None,
                     mask: torch.Tensor | None, images: dict | None = None) -> torch.Tensor:
    images = images or {}
    projected = _ProjectionFunction.apply(x, weight, bias, mask, torch.bfloat16, images.get("bc"),
                                          images.get("bc_t"), False)
    if not projected.is_contiguous():
        raise RuntimeError("implementation='cuda' requires w_bc to produce contiguous projected coordinates")
    return projected


def output_projection(mixed: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None,
                      dtype: torch.dtype, mask: torch.Tensor | None, images: dict | None = None) -> torch.Tensor:
    images = images or {}
    # Rows walked last to first, forward and input-gradient product alike: the
    # readout writes `mixed` forwards, and the loss' gradient arrives written
    # forwards too, so these products start with rows still in L2.
    return _ProjectionFunction.apply(mixed, weight, bias, mask, dtype, images.get("o"), images.get("o_t"), True)


__all__ = ["input_projection", "layer_images", "linear", "mix_output", "output_projection", "prepare_images",
           "register_gradient_slot", "weight_gradient"]
