"""The abort path of the tensor-core kernels, made to run on purpose.

Every wait of the library's kernels is bounded.  The pipeline waits (those
that also watch the CTA's abort flag) take their limit from a per-device
control word, one second unless a test shortens it with
``lsso_set_wait_limit_ns``.  With a 1 ns limit every such wait that is not
already complete runs out: the kernel sets the status word, every role stops,
the in-flight TMA loads, tensor-core operations and bulk stores are awaited
(with the full one-second bound), TMEM is freed and the kernel returns.  The
test checks that the status reads 1, that ``check_device_status`` raises
(and resets it), and that the next calls, with the default limit restored,
give exactly the results of the calls made before -- the context stays usable.
Nothing faults, traps or hangs: only waits that would have completed give up.
"""

from __future__ import annotations

import pytest
import torch

from tests.gpu_util import require_native, run_cuda, seeded_mixer_inputs

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def native() -> None:
    require_native()


def _layer_step(layer, x):
    xg = x.clone().requires_grad_()
    y = layer(xg, implementation="cuda")
    grads = torch.autograd.grad(y.float().square().sum(), [xg, *layer.parameters()])
    torch.cuda.synchronize()
    return y, grads


def test_wait_timeout_takes_the_abort_path_and_the_next_calls_are_exact() -> None:
    from lsso import LSSO, LSSOConfig
    from lsso_b200.ball import _native, cuda

    # a mixer shape on the head-group tile kernels, and a layer whose step also
    # runs the projection and weight-gradient GEMMs
    p, b, d, e, up = seeded_mixer_inputs(31, 2, 1024, 4, 32, 32)
    torch.manual_seed(5)
    layer = LSSO(LSSOConfig(dim=128, num_heads=4, rank=32, bias=True)).cuda()
    x = torch.randn(2, 512, 128, device="cuda", dtype=torch.float16)

    out0, grads0 = run_cuda(p, b, d, e, None, None, up)
    y0, lgrads0 = _layer_step(layer, x)
    cuda.check_device_status()  # clean so far

    _native.set_wait_limit_ns(1)
    try:
        run_cuda(p, b, d, e, None, None, up)
        _layer_step(layer, x)
        assert cuda.device_status(reset=False) == 1
        with pytest.raises(RuntimeError, match="gave up waiting"):
            cuda.check_device_status()
    finally:
        _native.set_wait_limit_ns(0)
    assert cuda.device_status(reset=False) == 0

    out1, grads1 = run_cuda(p, b, d, e, None, None, up)
    y1, lgrads1 = _layer_step(layer, x)
    assert torch.equal(out1, out0)
    assert all(torch.equal(g1, g0) for g1, g0 in zip(grads1, grads0))
    assert torch.equal(y1, y0)
    assert all(torch.equal(g1, g0) for g1, g0 in zip(lgrads1, lgrads0))
    cuda.check_device_status()
