"""The projection GEMM (``lsso_linear``) against an FP64 evaluation of its contract.

Contract (reference lsso/ball/reference.py:58-97,170-247): BF16 multiplicands,
FP32 accumulation and bias, one rounding to the output dtype, masked rows zero.
The FP64 product of the BF16-rounded operands differs from an FP32-accumulated
one only by accumulation order, so outputs agree to FP32 accuracy before the
final rounding (a BF16/FP16 store may differ by one rounding step).
"""

from __future__ import annotations

import pytest
import torch

from tests.gpu_util import require_native

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def native() -> None:
    require_native()


def _expected(a, w, bias, mask, transposed):
    ad = a.to(torch.bfloat16).double()
    wd = w.to(torch.bfloat16).double()
    out = ad @ (wd if transposed else wd.T)
    if bias is not None:
        out = out + bias.double()
    if mask is not None:
        out = torch.where(mask.reshape(-1)[:, None], out, torch.zeros_like(out))
    return out


@pytest.mark.parametrize(("m", "k", "nout", "a_dtype", "out_dtype", "bias", "masked", "transposed"), [
    (1000, 256, 512, torch.float16, torch.bfloat16, False, False, False),
    (4096, 256, 256, torch.bfloat16, torch.float16, True, True, False),
    (333, 512, 256, torch.bfloat16, torch.float32, False, False, True),
    (257, 64, 66, torch.float16, torch.float32, True, False, False),
    (130, 40, 1024, torch.bfloat16, torch.bfloat16, False, True, False),
    (128, 24, 48, torch.float16, torch.float16, True, False, True),
    (70000, 256, 512, torch.float16, torch.bfloat16, False, False, False),
])
def test_linear_matches_bf16_contract(m, k, nout, a_dtype, out_dtype, bias, masked, transposed) -> None:
    from lsso_b200.ball.projection import linear

    g = torch.Generator().manual_seed(m + k + nout)
    a = (torch.randn(m, k, generator=g) * 3).to("cuda", a_dtype)
    w = torch.randn((k, nout) if transposed else (nout, k), generator=g).cuda() / k ** 0.5
    b = torch.randn(nout, generator=g).cuda() if bias else None
    mask = (torch.rand(m, generator=g) > 0.3).cuda() if masked else None
    out = linear(a, w, b, mask, out_dtype, weight_transposed=transposed)
    torch.cuda.synchronize()
    ref = _expected(a, w, b, mask, transposed)
    assert out.dtype == out_dtype and out.shape == (m, nout)
    diff = (out.double() - ref).abs()
    if out_dtype == torch.float32:
        tol = 1e-5 * ref.abs().max().item()
    else:
        eps = 2.0 ** -8 if out_dtype == torch.bfloat16 else 2.0 ** -11
        tol = eps * ref.abs().max().item()
    assert diff.max().item() <= tol, (diff.max().item(), tol)
    if mask is not None:
        assert torch.count_nonzero(out[~mask]) == 0


def test_linear_fp16_input_rounds_through_bf16() -> None:
    """An FP16 activation is rounded to BF16 before the product (reference.py:181)."""
    from lsso_b200.ball.projection import linear

    a = torch.full((128, 8), 1.0 + 2.0 ** -10, device="cuda", dtype=torch.float16)  # not representable in BF16
    w = torch.zeros(8, 8, device="cuda")
    w[0, 0] = 1.0
    out = linear(a, w, None, None, torch.float32)
    assert torch.all(out[:, 0] == 1.0)


def test_linear_rejects_misaligned_k_through_the_abi() -> None:
    from lsso_b200.ball import _native

    lib = _native.library()
    assert lib.lib.lsso_linear_workspace_size(128, 12, 64) == 0
    assert "multiple of 8" in lib.last_error()


@pytest.mark.parametrize(("t", "nout", "k", "g_dtype", "x_dtype", "masked"), [
    (262144, 512, 256, torch.bfloat16, torch.float16, False),
    (262144, 256, 256, torch.float16, torch.bfloat16, False),
    (5000, 1024, 512, torch.bfloat16, torch.bfloat16, True),
    (777, 72, 40, torch.float16, torch.float16, True),
])
def test_weight_gradient_matches_fp64(t, nout, k, g_dtype, x_dtype, masked) -> None:
    from lsso_b200.ball.projection import weight_gradient

    gen = torch.Generator().manual_seed(t + nout + k)
    g = torch.randn(t, nout, generator=gen).to("cuda", g_dtype)
    x = torch.randn(t, k, generator=gen).to("cuda", x_dtype)
    mask = (torch.rand(t, generator=gen) > 0.25).cuda() if masked else None
    if masked:
        x[~mask] = float("nan")  # masked rows must not contribute, even when not finite
    dw = weight_gradient(g, x, mask)
    torch.cuda.synchronize()
    gd = g.to(torch.bfloat16).double()
    xd = torch.nan_to_num(x.to(torch.bfloat16).double())
    if masked:
        gd = gd * mask[:, None]
        xd = xd * mask[:, None]
    ref = gd.T @ xd
    err = float((dw.double() - ref).norm() / ref.norm())
    assert dw.shape == (nout, k) and dw.dtype == torch.float32
    assert err < 1e-5, err
    again = weight_gradient(g, x, mask)
    assert torch.equal(dw, again)  # deterministic


@pytest.mark.parametrize(("m", "k", "nout", "a_dtype", "out_dtype", "bias", "masked", "transposed"), [
    (1000, 256, 512, torch.float16, torch.bfloat16, False, False, False),
    (4096, 256, 256, torch.bfloat16, torch.float16, True, True, False),
    (333, 512, 256, torch.bfloat16, torch.float32, False, False, True),
    (257, 64, 72, torch.float16, torch.float32, True, False, False),
    (130, 40, 1024, torch.bfloat16, torch.bfloat16, False, True, False),
    (500, 1024, 512, torch.float16, torch.bfloat16, True, False, False),  # long K: streamed weight k-blocks
])
def test_prepared_weight_image_is_bit_identical(m, k, nout, a_dtype, out_dtype, bias, masked, transposed) -> None:
    """lsso_linear_prepare + lsso_linear_prepared (several images in one launch)
    give exactly lsso_linear's output."""
    from lsso_b200.ball.projection import linear, prepare_images

    g = torch.Generator().manual_seed(7 * m + k)
    a = (torch.randn(m, k, generator=g) * 3).to("cuda", a_dtype)
    w = torch.randn((k, nout) if transposed else (nout, k), generator=g).cuda() / k ** 0.5
    other = torch.randn(nout, k, generator=g).cuda()  # a second image in the same launch
    b = torch.randn(nout, generator=g).cuda() if bias else None
    mask = (torch.rand(m, generator=g) > 0.3).cuda() if masked else None
    images = prepare_images([(other, False), (w, transposed)])
    plain = linear(a, w, b, mask, out_dtype, weight_transposed=transposed)
    prepared = linear(a, w, b, mask, out_dtype, weight_transposed=transposed, image=images[1])
    backwards = linear(a, w, b, mask, out_dtype, weight_transposed=transposed, image=images[1], reverse=True)
    other_out = linear(a, other.T.contiguous(), None, None, out_dtype, weight_transposed=True)
    other_prepared = linear(a, other, None, None, out_dtype, image=images[0]) if k == other.shape[1] else None
    torch.cuda.synchronize()
    assert torch.equal(plain, prepared)
    assert torch.equal(plain, backwards)  # rows walked last to first: same result
    if other_prepared is not None:
        assert torch.equal(other_out, other_prepared)


def test_layer_step_with_prepared_images_matches_per_call_conversion() -> None:
    """A full layer step (forward + backward) through the one-launch weight
    images equals the same step with a conversion kernel per GEMM, bit for bit."""
    from lsso import LSSO, LSSOConfig
    from lsso_b200.ball import projection

    torch.manual_seed(3)
    layer = LSSO(LSSOConfig(dim=128, num_heads=4, rank=32, bias=True)).cuda()
    x = torch.randn(2, 300, 128, device="cuda", dtype=torch.float16)

    def step():
        xg = x.clone().requires_grad_()
        y = layer(xg, implementation="cuda")
        grads = torch.autograd.grad(y.float().square().sum(), [xg, *layer.parameters()])
        return y, grads

    y1, g1 = step()
    original = projection.layer_images
    projection.layer_images = lambda *args: None
    try:
        y2, g2 = step()
    finally:
        projection.layer_images = original
    assert torch.equal(y1, y2)
    for a, b in zip(g1, g2):
        assert torch.equal(a, b)


def test_prepare_rejects_bad_arguments() -> None:
    import ctypes

    from lsso_b200.ball import _native

    lib = _native.library()
    vp, ci, i64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64
    w = torch.zeros(64, 64, device="cuda")
    image = torch.empty(lib.lib.lsso_linear_image_size(64, 64), dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    args = ((vp * 1)(w.data_ptr()), (ci * 1)(0), (i64 * 1)(64), (i64 * 1)(64), (vp * 1)(image.data_ptr()), stream)
    assert lib.lib.lsso_linear_prepare(5, *args) != 0 and "count" in lib.last_error()
    assert lib.lib.lsso_linear_prepare(1, (vp * 1)(w.data_ptr()), (ci * 1)(0), (i64 * 1)(60), (i64 * 1)(64),
                                       (vp * 1)(image.data_ptr()), stream) != 0
    assert lib.lib.lsso_linear_prepare(1, *args) == 0
    assert lib.lib.lsso_linear_image_size(12, 64) == 0
