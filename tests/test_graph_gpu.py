"""A training step captured in a CUDA graph and replayed equals the eager step bit for bit.

Every library kernel is launched with programmatic stream serialisation and
waits for its predecessor before touching memory; a kernel that read an input
too early would show up here as a difference between the eagerly launched
step and the graph replay (all kernels are deterministic, so the two must be
identical).  Two shapes: the bench layout (tile kernels, warp solves) and a
masked rank-64 BF16 case with per-sample positions.
"""

from __future__ import annotations

import pytest
import torch

from lsso import LSSO, LSSOConfig
from tests.gpu_util import require_native

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def native() -> None:
    require_native()


@pytest.mark.parametrize(("dim", "heads", "rank", "batch", "length", "dtype", "masked"), [
    (256, 8, 32, 4, 1000, torch.float16, False),
    (256, 8, 64, 3, 700, torch.bfloat16, True),
])
def test_graph_replay_equals_eager_step(dim, heads, rank, batch, length, dtype, masked) -> None:
    torch.manual_seed(5)
    layer = LSSO(LSSOConfig(dim, heads, rank)).cuda()
    params = list(layer.parameters())
    gen = torch.Generator().manual_seed(9)
    x = torch.randn(batch, length, dim, generator=gen).to("cuda", dtype).requires_grad_()
    mask = ids = None
    if masked:
        lens = torch.randint(length // 3, length + 1, (batch,), generator=gen)
        mask = (torch.arange(length)[None, :] < lens[:, None]).cuda()
        ids = torch.where(mask, torch.arange(length, device="cuda")[None, :], torch.zeros(1, device="cuda",
                                                                                           dtype=torch.int64))

    def clear() -> None:
        x.grad = None
        for p in params:
            p.grad = None

    def step():
        with torch.autocast("cuda", dtype=dtype, cache_enabled=False):
            y = layer(x, valid_mask=mask, position_ids=ids, implementation="cuda")
            loss = y.float().square().mean()
        loss.backward()
        return y, loss

    clear()
    y0, l0 = step()
    torch.cuda.synchronize()
    ref = [y0.detach().clone(), l0.detach().clone(), x.grad.clone()] + [p.grad.clone() for p in params]
    del y0, l0  # free the eager autograd graph, so capture creates its own gradient-accumulation nodes

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(2):
            clear()
            step()
    torch.cuda.current_stream().wait_stream(side)
    clear()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        yg, lg = step()
    for _ in range(2):
        graph.replay()
    torch.cuda.synchronize()
    got = [yg, lg, x.grad] + [p.grad for p in params]
    names = ["y", "loss", "x.grad"] + [n for n, _ in layer.named_parameters()]
    for name, a, b in zip(names, got, ref):
        assert torch.equal(a, b), name
    del graph
