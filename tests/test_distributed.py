"""Data-parallel host logic on CPU with two gloo ranks.

Each rank runs the PyTorch reference path of the layer on its own shard, the
gradients are averaged with ``allreduce_gradients`` (one flat collective) and
must equal the single-process gradients of the full batch's mean loss.  A
second test makes one rank fail before the collective and checks that the
other rank gets an error from the short process-group timeout instead of
waiting for ever.
"""

from __future__ import annotations

import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, result_path: str) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    from lsso import LSSO, LSSOConfig
    from lsso_b200.ball.distributed import allreduce_gradients

    torch.manual_seed(0)
    layer = LSSO(LSSOConfig(32, 2, 16)).double()
    x = torch.randn(4, 9, 32, dtype=torch.float64, generator=torch.Generator().manual_seed(1))
    shard = x[rank * 2:(rank + 1) * 2]
    loss = layer(shard).square().mean()
    loss.backward()
    allreduce_gradients(layer.parameters())
    if rank == 0:
        torch.save({n: p.grad for n, p in layer.named_parameters()}, result_path)
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_gradient_average_matches_full_batch(tmp_path) -> None:
    path = str(tmp_path / "grads.pt")
    mp.spawn(_worker, args=(2, _free_port(), path), nprocs=2, join=True)
    got = torch.load(path)
    from lsso import LSSO, LSSOConfig

    torch.manual_seed(0)
    layer = LSSO(LSSOConfig(32, 2, 16)).double()
    x = torch.randn(4, 9, 32, dtype=torch.float64, generator=torch.Generator().manual_seed(1))
    loss = 0.5 * (layer(x[:2]).square().mean() + layer(x[2:]).square().mean())
    loss.backward()
    for name, p in layer.named_parameters():
        # FP64 on both sides; only LAPACK/BLAS blocking (thread count) differs,
        # which moves the base gradient by ~1e-8; a wrong average is off by 100%.
        err = float((got[name] - p.grad).norm() / p.grad.norm())
        assert err < 1e-6, (name, err)


def _failing_worker(rank: int, world: int, port: int, result_path: str) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    from lsso_b200.ball.distributed import allreduce_gradients

    p = torch.nn.Parameter(torch.zeros(3))
    p.grad = torch.ones(3)
    if rank == 1:
        # This rank fails between steps: it never joins the collective.
        dist.destroy_process_group()
        return
    try:
        allreduce_gradients([p])
        outcome = "completed"
    except RuntimeError as error:  # gloo reports the missing peer / timeout
        outcome = f"error: {type(error).__name__}"
    with open(result_path, "w") as f:
        f.write(outcome)


@pytest.mark.timeout(120)
def test_a_rank_leaving_ends_the_collective_with_an_error(tmp_path) -> None:
    path = tmp_path / "outcome.txt"
    mp.spawn(_failing_worker, args=(2, _free_port(), str(path)), nprocs=2, join=True)
    assert path.read_text().startswith("error")
