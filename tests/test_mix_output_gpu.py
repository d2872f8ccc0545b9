"""The mixer + output projection node and lsso_backward_with_wgrad.

The layer's training path runs the mixer and the output projection as one
autograd node whose backward computes the output projection's weight
gradient in the same native call as the mixer's backward; with the
concurrent schedule the weight-gradient kernel shares every SM with the
backward's persistent solve grid (on the library's side stream).  Every
kernel is deterministic and the split of the weight gradient over tokens
does not depend on the schedule, so all outputs must be bit-identical:
  * to the separate calls (fast_mix, then the output projection), and
  * between the concurrent and the one-after-the-other schedule,
at the module level (several ranks, masks, bias, both dtypes) and through
the C ABI (lsso_backward_with_wgrad against lsso_backward followed by
lsso_linear_wgrad, twice in a row).
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from lsso import LSSO, LSSOConfig
from tests.gpu_util import require_native

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def native() -> None:
    require_native()


def _separate_calls(layer, x):
    """The layer's CUDA forward composed of the separate nodes (no mask, shared positions)."""
    from lsso_b200.ball import cuda, projection

    images = projection.layer_images(layer.w_bc.weight, layer.w_o.weight, True)
    projected = projection.input_projection(x, layer.w_bc.weight, layer.w_bc.bias, None, images)
    mixed = cuda.fast_mix(projected, layer.core_base_raw, layer.core_drive_weight, layer.eta_raw, None, None)
    return projection.output_projection(mixed, layer.w_o.weight, layer.w_o.bias, x.dtype, None, images)


def _step(layer, x, forward, mask=None, ids=None):
    x.grad = None
    for p in layer.parameters():
        p.grad = None
    with torch.autocast("cuda", dtype=x.dtype, cache_enabled=False):
        y = forward(layer, x) if forward is not None else layer(x, mask, ids, implementation="cuda")
    (y.float().square().mean() * 65536.0).backward()
    torch.cuda.synchronize()
    return [y.detach().clone(), x.grad.clone()] + [p.grad.clone() for p in layer.parameters()]


def _layer(dim, heads, rank, bias, seed):
    torch.manual_seed(seed)
    layer = LSSO(LSSOConfig(dim, heads, rank, bias=bias)).cuda()
    with torch.no_grad():
        layer.core_base_raw.normal_(0.0, 0.05)
        layer.core_drive_weight.normal_(0.0, 0.05)
    return layer


@pytest.mark.parametrize(("dim", "heads", "rank", "batch", "length", "dtype", "bias"), [
    (256, 8, 32, 4, 1000, torch.float16, False),   # the bench layout: concurrent schedule
    (128, 4, 16, 3, 517, torch.bfloat16, True),    # rank 16, ragged tail
    (256, 8, 64, 2, 700, torch.float16, True),     # rank 64: no room beside the GEMM, sequential
])
def test_node_equals_separate_calls(dim, heads, rank, batch, length, dtype, bias) -> None:
    from lsso_b200.ball import projection

    layer = _layer(dim, heads, rank, bias, seed=rank)
    x = torch.randn(batch, length, dim, generator=torch.Generator().manual_seed(3)).to("cuda", dtype)
    x.requires_grad_()
    separate = _step(layer, x, _separate_calls)
    names = ["y", "x.grad"] + [n for n, _ in layer.named_parameters()]
    for concurrent in (True, False):
        projection.CONCURRENT_WGRAD = concurrent
        try:
            for _ in range(2):
                node = _step(layer, x, None)
                for name, a, b in zip(names, node, separate):
                    assert torch.equal(a, b), (name, concurrent)
        finally:
            projection.CONCURRENT_WGRAD = True


def test_masked_per_sample_positions_both_schedules() -> None:
    from lsso_b200.ball import projection

    layer = _layer(256, 8, 32, True, seed=11)
    batch, length = 3, 900
    gen = torch.Generator().manual_seed(4)
    x = torch.randn(batch, length, 256, generator=gen).to("cuda", torch.bfloat16).requires_grad_()
    lens = torch.tensor([900, 517, 64])
    mask = (torch.arange(length)[None, :] < lens[:, None]).cuda()
    ids = torch.where(mask, torch.arange(length, device="cuda")[None, :], torch.zeros(1, device="cuda",
                                                                                       dtype=torch.int64))
    results = []
    for concurrent in (True, False):
        projection.CONCURRENT_WGRAD = concurrent
        try:
            results.append(_step(layer, x, None, mask, ids))
        finally:
            projection.CONCURRENT_WGRAD = True
    for a, b in zip(*results):
        assert torch.equal(a, b)
    assert torch.isfinite(results[0][0]).all()
    assert (results[0][0][~mask] == 0).all()


def test_c_abi_with_wgrad_equals_backward_then_wgrad() -> None:
    """lsso_backward_with_wgrad (concurrent and not) against lsso_backward + lsso_linear_wgrad, twice."""
    from lsso_b200.ball import _native

    lib = _native.library()
    B, N, H, R, d = 4, 1500, 8, 32, 32
    D = H * d
    W = H * R + D
    gen = torch.Generator(device="cuda").manual_seed(21)
    projected = torch.randn(B, N, W, device="cuda", generator=gen).to(torch.bfloat16)
    base = torch.randn(H, R, R, device="cuda", generator=gen) * 0.05
    drive = torch.randn(H, d, R, device="cuda", generator=gen) * 0.05
    eta = torch.randn(H, device="cuda", generator=gen) * 0.05
    mixed, tape, pivots = _native.forward(projected, base, drive, eta, None, None, train=True)
    grad_mixed = torch.randn(B, N, D, device="cuda", generator=gen).to(torch.bfloat16)
    dy = torch.randn(B * N, D, device="cuda", generator=gen).to(torch.float16)
    mixed_flat = mixed.reshape(-1, D)

    # separate calls
    expected = _native.backward(grad_mixed, projected, base, drive, eta, tape, pivots, None, None)
    from lsso_b200.ball import projection
    dw_expected = projection.weight_gradient(dy, mixed_flat, None)
    torch.cuda.synchronize()

    for concurrent in (1, 0, 1):
        dw = torch.full((D, D), float("nan"), device="cuda")
        got = _native.backward(grad_mixed, projected, base, drive, eta, tape, pivots, None, None,
                               wgrad=(dy, mixed_flat, None, dw, concurrent))
        torch.cuda.synchronize()
        for a, b in zip(got, expected):
            assert torch.equal(a, b), concurrent
        assert torch.equal(dw, dw_expected), concurrent
    assert _native.device_status(reset=True) == 0

    # the entry point rejects a bad weight-gradient shape with a message, launching nothing
    size = lib.lib.lsso_backward_workspace_size(B, N, H, D, R, 0)
    ws = torch.empty(size, dtype=torch.uint8, device="cuda")
    out = [torch.empty_like(t) for t in expected]
    code = lib.lib.lsso_backward_with_wgrad(
        grad_mixed.data_ptr(), projected.data_ptr(), base.data_ptr(), drive.data_ptr(), eta.data_ptr(),
        tape.data_ptr(), pivots.data_ptr(), None, 0, None, B, N, H, D, R, out[0].data_ptr(), out[1].data_ptr(),
        out[2].data_ptr(), out[3].data_ptr(), ws.data_ptr(), size, dy.data_ptr(), 1, mixed_flat.data_ptr(), 0,
        None, B * N, D - 4, D, dw_expected.data_ptr(), ws.data_ptr(), size, 1,
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert code != 0
    assert "multiples of 8" in lib.last_error()
