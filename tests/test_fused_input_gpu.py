"""Input projection fused with the forward moment pass (``lsso_fused_forward``).

The fused kernel computes the packed projection and the moment partials in
one pass over x; it must reproduce the separate projection GEMM followed by
the mixer exactly (same BF16 projection, same partial sums in the same
order), so the layer's outputs and every gradient are compared bit for bit
with the unfused calls (which the module-level oracle comparisons of
test_module_gpu.py cover), and the projection against the reference's
rounding rule.  The path is opt-in (projection.FUSED_INPUT); these tests
turn it on.
"""

from __future__ import annotations

import pytest
import torch

from lsso import LSSO, LSSOConfig
from lsso_b200.ball import _native, projection
from tests.gpu_util import relative_l2, require_native

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def native() -> None:
    require_native()


@pytest.fixture(autouse=True)
def fused_enabled():
    default = projection.FUSED_INPUT
    projection.FUSED_INPUT = True
    yield
    projection.FUSED_INPUT = default


def _layer(config: LSSOConfig, seed: int) -> LSSO:
    torch.manual_seed(seed)
    layer = LSSO(config)
    with torch.no_grad():
        layer.core_base_raw.normal_(0.0, 0.05)
        layer.core_drive_weight.normal_(0.0, 0.05)
        if layer.w_bc.bias is not None:
            layer.w_bc.bias.normal_(0.0, 0.1)
    return layer.cuda()


def _inputs(batch, length, dim, dtype, masked, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(batch, length, dim, generator=g).to("cuda", dtype)
    mask = ids = None
    if masked:
        lens = torch.randint(length // 3, length + 1, (batch,), generator=g)
        lens[0] = length
        mask = (torch.arange(length)[None, :] < lens[:, None]).cuda()
        ids = torch.where(mask.cpu(), torch.arange(length)[None, :].expand(batch, length),
                          torch.zeros(1, dtype=torch.int64)).cuda()
        x[~mask] = float("nan")  # padding content must not reach the output
    return x, mask, ids


def _profiled(fn):
    _native.profile_start()
    try:
        out = fn()
        torch.cuda.synchronize()
    finally:
        names = _native.profile_stop()
    return out, names


CASES = [
    # batch, length, dim, heads, rank, bias, dtype, masked
    (2, 1000, 256, 8, 32, True, torch.float16, False),   # the bench shape's layout, ragged last tile
    (3, 700, 256, 8, 64, False, torch.bfloat16, True),   # value box shared by two groups, masks, per-sample ids
    (2, 333, 128, 2, 64, False, torch.float16, False),   # d = 64, two K blocks, six x stages
    (1, 4096, 256, 4, 64, True, torch.bfloat16, False),  # d = 64, several chunks per sample
    (4, 129, 64, 2, 32, True, torch.float16, True),      # one K block, 129 tokens
]


@pytest.mark.parametrize(("batch", "length", "dim", "heads", "rank", "bias", "dtype", "masked"), CASES)
def test_fused_layer_equals_separate_calls(batch, length, dim, heads, rank, bias, dtype, masked) -> None:
    layer = _layer(LSSOConfig(dim, heads, rank, bias=bias), 7 + rank + dim)
    x, mask, ids = _inputs(batch, length, dim, dtype, masked, 11 + length)
    up = torch.randn(x.shape, generator=torch.Generator().manual_seed(5)).to("cuda", dtype)
    params = list(layer.parameters())

    def run(fused: bool):
        projection.FUSED_INPUT = fused
        xg = x.detach().clone().requires_grad_()
        y = layer(xg, valid_mask=mask, position_ids=ids, implementation="cuda")
        grads = torch.autograd.grad((y.float() * up.float()).sum(), [xg, *params])
        return y, grads

    assert projection.fused_input_covers(x, heads, rank)
    (y1, g1), names = _profiled(lambda: run(True))
    assert "proj_moments" in names and "moments_fwd" not in names, sorted(names)
    (y0, g0), names0 = _profiled(lambda: run(False))
    assert "proj_moments" not in names0 and "moments_fwd" in names0
    assert torch.isfinite(y1).all()
    assert torch.equal(y1, y0)
    for a, b in zip(g1, g0):
        assert torch.equal(a, b)
    if mask is not None:
        assert torch.count_nonzero(y1[~mask]) == 0
        assert torch.count_nonzero(g1[0][~mask]) == 0
    with torch.no_grad():
        projection.FUSED_INPUT = True
        yi = layer(x, valid_mask=mask, position_ids=ids, implementation="cuda")
    assert torch.equal(yi, y1)


@pytest.mark.parametrize(("batch", "length", "dim", "heads", "rank", "bias", "dtype", "masked"), CASES[:3])
def test_fused_projection_and_tape(batch, length, dim, heads, rank, bias, dtype, masked) -> None:
    """The native call's own outputs: projection = the projection GEMM's (masked rows zero, the
    reference's BF16 rounding of bf16(x) bf16(W)^T + b), mixed and tape = lsso_forward on it."""
    layer = _layer(LSSOConfig(dim, heads, rank, bias=bias), 3 + rank)
    x, mask, ids = _inputs(batch, length, dim, dtype, masked, 23 + length)
    counts = pos = None
    if mask is not None:
        pos = LSSO._center_positions(ids, mask, dtype=torch.float32, all_valid=False, batch=batch, length=length,
                                     device=x.device).contiguous()
        counts = mask.sum(-1).float().clamp_min(1.0).contiguous()
    w, b = layer.w_bc.weight.detach(), None if layer.w_bc.bias is None else layer.w_bc.bias.detach()
    base, drive, eta = layer.core_base_raw.detach(), layer.core_drive_weight.detach(), layer.eta_raw.detach()
    proj, mixed, tape, pivots = _native.fused_forward(x, w, b, mask, base, drive, eta, pos, counts, train=True)
    ref_proj = projection.linear(x, w, b, mask, torch.bfloat16)
    assert torch.equal(proj, ref_proj)
    valid = torch.ones(batch, length, dtype=torch.bool, device="cuda") if mask is None else mask
    xs = torch.where(valid[..., None], x.float(), torch.zeros(1, device="cuda"))
    exact = xs.to(torch.bfloat16).double() @ w.to(torch.bfloat16).double().t()
    if b is not None:
        exact = exact + b.double()
    exact = torch.where(valid[..., None], exact, torch.zeros(1, device="cuda", dtype=torch.float64))
    assert relative_l2(proj, exact) <= 4e-3  # one BF16 rounding of an FP32-accumulated product
    ref_mixed, ref_tape, ref_pivots = _native.forward(ref_proj, base, drive, eta, pos, counts, train=True)
    assert torch.equal(mixed, ref_mixed)
    used = length * rank  # a tape row starts with N*R floats the mixer leaves unused
    assert torch.equal(tape[:, used:], ref_tape[:, used:])
    assert torch.equal(pivots, ref_pivots)


def test_uncovered_shapes_take_the_separate_path() -> None:
    """Ranks 16 / 48, a head wider than the rank, D above 256: projection GEMM + mixer as before."""
    for dim, heads, rank in ((256, 8, 16), (192, 4, 48), (256, 4, 32), (512, 8, 64)):
        x = torch.empty(1, 8, dim, device="cuda", dtype=torch.float16)
        assert not projection.fused_input_covers(x, heads, rank), (dim, heads, rank)
    layer = _layer(LSSOConfig(256, 8, 16), 1)
    x = torch.randn(1, 300, 256, device="cuda").half()
    with torch.no_grad():
        y, names = _profiled(lambda: layer(x, implementation="cuda"))
    assert "proj_moments" not in names and "moments_fwd" in names
    assert torch.isfinite(y).all()


def test_fused_entry_point_rejects_uncovered_shapes() -> None:
    lib = _native.library()
    assert lib.lib.lsso_fused_forward_supported(2, 100, 8, 256, 32) == 1
    assert lib.lib.lsso_fused_forward_supported(2, 100, 8, 256, 16) == 0
    assert lib.lib.lsso_fused_forward_workspace_size(2, 100, 8, 256, 16, 0, 1) == 0
    assert "not covered" in lib.last_error()
