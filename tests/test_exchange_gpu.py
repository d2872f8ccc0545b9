"""The overlapped gradient exchange on the GPU.

One process: the exchange's gradients (projection weight gradients written by
the library straight into the flat buffer, the others copied there by hooks)
equal the plain step's bit for bit, eagerly and replayed as a CUDA graph.
Two NCCL ranks (when the box has two GPUs): the exchanged average equals the
one-collective ``allreduce_gradients`` average, in eager steps and in graph
replays that hold the collectives.
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

from tests.gpu_util import require_native

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module", autouse=True)
def native() -> None:
    require_native()


def _step(layer, x):
    for q in layer.parameters():
        q.grad = None
    with torch.autocast("cuda", dtype=torch.float16, cache_enabled=False):
        y = layer(x, implementation="cuda")
    y.float().square().mean().backward()


def test_single_process_exchange_matches_the_plain_step(tmp_path) -> None:
    import torch.distributed as dist

    from lsso import LSSO, LSSOConfig
    from lsso_b200.ball.distributed import GradientExchange, layer_buckets

    store = dist.FileStore(str(tmp_path / "store"), 1)
    dist.init_process_group("nccl", store=store, rank=0, world_size=1)
    try:
        torch.manual_seed(0)
        layer = LSSO(LSSOConfig(256, 8, 32, bias=True)).cuda()
        x = torch.randn(2, 1000, 256, device="cuda").half()
        _step(layer, x)
        plain = [q.grad.clone() for q in layer.parameters()]

        exchange = GradientExchange(layer_buckets(layer))
        _step(layer, x)
        exchange.finish()
        for q, g in zip(layer.parameters(), plain):
            assert q.grad.data_ptr() == exchange.slot[q].data_ptr()
            assert torch.equal(q.grad, g)

        # the same step captured as a CUDA graph and replayed
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(2):
                _step(layer, x)
                exchange.finish()
        torch.cuda.current_stream().wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        for q in layer.parameters():
            q.grad = None
        with torch.cuda.graph(graph):
            _step(layer, x)
            exchange.finish()
        exchange.flat.zero_()
        graph.replay()
        torch.cuda.synchronize()
        for q, g in zip(layer.parameters(), plain):
            assert torch.equal(q.grad, g)
        del graph
        exchange.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_nccl_ranks_exchange_equals_one_collective_average() -> None:
    env = dict(os.environ, MASTER_ADDR="127.0.0.1", MASTER_PORT="29533", PYTHONPATH=str(ROOT),
               NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "540", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port", "29533",
           str(ROOT / "tests" / "exchange_ranks.py")]
    result = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    assert result.returncode == 0, result.stdout[-3000:] + result.stderr[-3000:]
    assert "exchange ok" in result.stdout
