"""Complete-module parity on the GPU: ``layer(x, implementation="cuda")``
(projections + native mixer) against the FP64 oracle, and the BASELINE
configurations at full size through size-independent properties."""

from __future__ import annotations

import copy

import numpy as np
import pytest
import torch

from oracle import lsso_oracle as O
from lsso import LSSO, LSSOConfig
from tests.gpu_util import max_abs, relative_l2, require_native

pytestmark = pytest.mark.gpu

_PARAM_KEYS = {"w_bc.weight": "w_bc", "w_bc.bias": "b_bc", "w_o.weight": "w_o", "w_o.bias": "b_o",
               "core_base_raw": "core_base_raw", "core_drive_weight": "core_drive_weight", "eta_raw": "eta_raw"}


@pytest.fixture(scope="module", autouse=True)
def native() -> None:
    require_native()


def _layer(config: LSSOConfig, seed: int, core: float = 0.05) -> LSSO:
    torch.manual_seed(seed)
    layer = LSSO(config)
    with torch.no_grad():
        layer.core_base_raw.normal_(0.0, core)
        layer.core_drive_weight.normal_(0.0, core)
    return layer.cuda()


def _oracle(layer: LSSO, x: torch.Tensor, mask, position_ids, upstream):
    params = {"b_bc": None, "b_o": None}
    for name, p in layer.named_parameters():
        params[_PARAM_KEYS[name]] = p.detach().double().cpu().numpy()
    n = lambda t: None if t is None else t.detach().cpu().numpy()  # noqa: E731
    y, state = O.module_forward(params, n(x).astype(np.float64), n(mask), n(position_ids),
                                heads=layer.config.num_heads, rank=layer.config.rank, return_state=True)
    grads = O.module_backward(n(upstream).astype(np.float64), state)
    return y, grads


def _compare(layer, x, mask=None, position_ids=None, *, fwd=5e-3, grad=3e-2, label=""):
    xg = x.detach().clone().requires_grad_()
    upstream = torch.randn(x.shape, generator=torch.Generator().manual_seed(1)).to(x.device, x.dtype)
    y = layer(xg, valid_mask=mask, position_ids=position_ids, implementation="cuda")
    assert y.dtype == x.dtype
    names = [n for n, _ in layer.named_parameters()]
    grads = torch.autograd.grad((y.float() * upstream.float()).sum(), [xg, *layer.parameters()])
    ry, rg = _oracle(layer, torch.nan_to_num(x.float()), mask, position_ids, upstream.float())
    line = [f"{label} y={relative_l2(y, ry):.2e} maxabs={max_abs(y, ry):.2e}"]
    assert relative_l2(y, ry) <= fwd, line
    checks = [("x", grads[0], rg["x"])] + [(n, g, rg[_PARAM_KEYS[n]]) for n, g in zip(names, grads[1:])]
    for name, g, r in checks:
        assert torch.isfinite(g).all(), name
        e = relative_l2(torch.nan_to_num(g), r)
        line.append(f"{name}={e:.2e}")
        assert e <= grad, (name, line)
    print(" ".join(line))
    return y, grads


@pytest.mark.parametrize(("dim", "heads", "rank", "bias", "dtype"), [
    (32, 2, 16, True, torch.float16), (128, 1, 64, True, torch.float16), (64, 2, 32, False, torch.bfloat16),
    (96, 3, 48, False, torch.float16), (256, 8, 32, False, torch.float16),
])
def test_full_module_matches_fp64_oracle(dim, heads, rank, bias, dtype) -> None:
    layer = _layer(LSSOConfig(dim=dim, num_heads=heads, rank=rank, bias=bias), 59 + rank)
    x = torch.randn(2, 65, dim, generator=torch.Generator().manual_seed(3)).to("cuda", dtype)
    positions = 3 * torch.arange(65, device="cuda") + 7
    _compare(layer, x, None, positions, label=f"module {(dim, heads, rank, bias, dtype)}")


def test_full_module_masked_batch_specific_positions() -> None:
    layer = _layer(LSSOConfig(dim=34, num_heads=2, rank=16, bias=True), 109)
    mask = torch.tensor([[True, False, True, True, False, True, True] * 5, [False] * 35], device="cuda")
    ids = torch.stack((3 * torch.arange(35) + 7, 5 * torch.arange(35) + 101)).cuda()
    x = torch.randn(2, 35, 34, generator=torch.Generator().manual_seed(9)).to("cuda", torch.float16)
    x[~mask] = float("nan")
    y, grads = _compare(layer, x, mask, ids, label="masked module")
    assert torch.count_nonzero(y[1]) == 0
    assert torch.count_nonzero(grads[0][~mask]) == 0


def test_float64_positions_keep_relative_coordinates() -> None:
    layer = _layer(LSSOConfig(dim=32, num_heads=2, rank=16), 113)
    x = torch.randn(1, 9, 32, device="cuda").half()
    pos = torch.arange(9, device="cuda", dtype=torch.float64)
    with torch.no_grad():
        shifted = layer(x, position_ids=pos + 1e12, implementation="cuda")
        plain = layer(x, position_ids=pos, implementation="cuda")
    torch.testing.assert_close(shifted, plain, rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("dtype", (torch.float16, torch.bfloat16))
def test_autocast_matches_production_reference(dtype) -> None:
    torch.manual_seed(20260907)
    native = LSSO(LSSOConfig(32, 2, 16, bias=True)).cuda()
    reference = copy.deepcopy(native)
    x = torch.randn(2, 65, 32, device="cuda", dtype=dtype).requires_grad_()
    rx = x.detach().clone().requires_grad_()
    up = torch.randn_like(x)
    with torch.autocast("cuda", dtype=dtype):
        y = native(x, implementation="cuda")
        ry = reference(rx, implementation="reference")
    g = torch.autograd.grad((y * up).sum(), (x, *native.parameters()))
    rg = torch.autograd.grad((ry * up).sum(), (rx, *reference.parameters()))
    assert y.dtype == dtype
    assert relative_l2(y, ry) <= 5e-3
    for a, b in zip(g, rg):
        assert relative_l2(a, b) <= 3e-2


def test_config3_masked_rank64_bf16_full_size() -> None:
    """B=32, N=2048, D=256, H=8, r=64, BF16, prefix masks, per-sample positions."""
    g = torch.Generator().manual_seed(3)
    B, N = 32, 2048
    lengths = torch.randint(512, 2049, (B,), generator=g)
    mask = (torch.arange(N)[None, :] < lengths[:, None]).cuda()
    ids = torch.where(mask.cpu(), torch.arange(N)[None, :].expand(B, N), torch.zeros(B, N, dtype=torch.int64)).cuda()
    layer = _layer(LSSOConfig(256, 8, 64), 33)
    x = torch.randn(B, N, 256, generator=g).to("cuda", torch.bfloat16)
    xg = x.clone().requires_grad_()
    y = layer(xg, valid_mask=mask, position_ids=ids, implementation="cuda")
    y.float().square().mean().backward()
    assert torch.isfinite(y).all() and torch.count_nonzero(y[~mask]) == 0
    assert torch.isfinite(xg.grad).all() and torch.count_nonzero(xg.grad[~mask]) == 0
    # Two samples of the same batch against the oracle (rows are independent).
    for b in (0, B - 1):
        _compare(layer, x[b:b + 1], mask[b:b + 1], ids[b:b + 1], fwd=1e-2, label=f"config3 sample {b}")


def test_config4_shell_four_layers_bf16() -> None:
    """4 x [x + LSSO(LN(x))], D=128, H=4, r=48, embedding input (64, 4096), BF16."""
    torch.manual_seed(4)
    layers = [_layer(LSSOConfig(128, 4, 48), 40 + i) for i in range(4)]
    norms = [torch.nn.LayerNorm(128).cuda() for _ in range(4)]
    emb = torch.nn.Embedding(8, 128).cuda()
    torch.nn.init.normal_(emb.weight, 0.0, 0.02)
    tokens = torch.randint(0, 8, (64, 4096), device="cuda")

    def shell(mixers, lns, h, impl):
        for ln, mixer in zip(lns, mixers):
            h = h + mixer(ln(h.to(ln.weight.dtype)).to(h.dtype), implementation=impl)
        return h

    out = shell(layers, norms, emb(tokens).to(torch.bfloat16), "cuda")
    out.float().square().mean().backward()
    assert torch.isfinite(out).all()
    assert all(torch.isfinite(p.grad).all() for layer in layers for p in layer.parameters())
    with torch.no_grad():
        fast = shell(layers, norms, emb(tokens[:2]).to(torch.bfloat16), "cuda")
        ref = shell([copy.deepcopy(m).double() for m in layers], [copy.deepcopy(n).double() for n in norms],
                    emb(tokens[:2]).double(), "reference")
    assert relative_l2(fast, ref) <= 1e-2


def test_config5_long_sequence_rank64_slice() -> None:
    """BASELINE config 5 shape on a 2-sample slice (D=512, H=8, r=64, N=16384, FP16)."""
    layer = _layer(LSSOConfig(512, 8, 64), 5)
    x = torch.randn(2, 16384, 512, generator=torch.Generator().manual_seed(5)).to("cuda", torch.float16)
    _compare(layer, x, label="config5 slice")
