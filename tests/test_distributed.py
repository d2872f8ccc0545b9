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


def _exchange_worker(rank: int, world: int, port: int, result_path: str, overlap: bool = True) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    from lsso import LSSO, LSSOConfig
    from lsso_b200.ball.distributed import GradientExchange, layer_buckets

    torch.manual_seed(0)
    layer = LSSO(LSSOConfig(32, 2, 16, bias=True))
    exchange = GradientExchange(layer_buckets(layer), overlap=overlap)
    # CPU ranks: "auto" takes the process group's all_reduce; the peer kernel needs CUDA
    assert exchange.transport == "nccl"
    try:
        GradientExchange(layer_buckets(layer), transport="peer")
    except ValueError as exc:
        assert "needs CUDA" in str(exc)
    else:
        raise AssertionError("transport='peer' accepted CPU parameters")
    x = torch.randn(4, 9, 32, generator=torch.Generator().manual_seed(1))
    steps = []
    for step in range(2):  # two steps: the slots are reused
        for q in layer.parameters():
            q.grad = None
        shard = x[rank * 2:(rank + 1) * 2] * (1 + step)
        layer(shard).square().mean().backward()
        exchange.finish()
        assert all(q.grad.data_ptr() == exchange.slot[q].data_ptr() for q in layer.parameters())
        steps.append({n: q.grad.clone() for n, q in layer.named_parameters()})
    if rank == 0:
        torch.save(steps, result_path)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("overlap", (True, False))
def test_two_rank_gradient_exchange_matches_full_batch(tmp_path, overlap) -> None:
    """GradientExchange (buckets exchanged as the backward completes them, or the
    whole flat buffer after it; each p.grad a view of the averaged buffer) gives
    the full-batch gradient, on two consecutive steps."""
    path = str(tmp_path / "exchange.pt")
    mp.spawn(_exchange_worker, args=(2, _free_port(), path, overlap), nprocs=2, join=True)
    got = torch.load(path)
    from lsso import LSSO, LSSOConfig

    torch.manual_seed(0)
    layer = LSSO(LSSOConfig(32, 2, 16, bias=True))
    x = torch.randn(4, 9, 32, generator=torch.Generator().manual_seed(1))
    for step in range(2):
        for q in layer.parameters():
            q.grad = None
        xs = x * (1 + step)
        loss = 0.5 * (layer(xs[:2]).square().mean() + layer(xs[2:]).square().mean())
        loss.backward()
        for name, q in layer.named_parameters():
            err = float((got[step][name] - q.grad).norm() / q.grad.norm())
            assert err < 1e-5, (step, name, err)


def test_layer_buckets_cover_every_parameter_once() -> None:
    from lsso import LSSO, LSSOConfig
    from lsso_b200.ball.distributed import layer_buckets

    for bias in (False, True):
        layer = LSSO(LSSOConfig(32, 2, 16, bias=bias))
        flat = [p for b in layer_buckets(layer) for p in b]
        assert len(flat) == len(set(map(id, flat))) == len(list(layer.parameters()))
        assert layer_buckets(layer)[-1][0] is layer.w_bc.weight  # the input projection finishes last


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


# ---------------------------------------------------------------------------- sequence-parallel positions
_SEQ_CASES = ("plain", "mask", "mask_ids", "shared_ids", "float_ids")
_SEQ_CUTS = (0, 7, 19)  # two unequal slices of a 19-token sequence


def _seq_inputs(case: str):
    batch, length = 3, _SEQ_CUTS[-1]
    g = torch.Generator().manual_seed(5)
    mask = None
    ids = None
    if case in ("mask", "mask_ids"):
        mask = torch.rand(batch, length, generator=g) > 0.3
        mask[1] = False  # a sample with no valid token
    if case == "mask_ids":
        ids = torch.randint(0, 50, (batch, length), generator=g)
    if case == "shared_ids":
        ids = torch.arange(length) * 3 + 5
    if case == "float_ids":
        ids = torch.linspace(-2.0, 7.5, length, dtype=torch.float32)
    return batch, length, mask, ids


def _seq_worker(rank: int, world: int, port: int, out_dir: str) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    from lsso_b200.ball.sequence_parallel import sequence_positions

    a, b = _SEQ_CUTS[rank], _SEQ_CUTS[rank + 1]
    result = {}
    for case in _SEQ_CASES:
        batch, _, mask, ids = _seq_inputs(case)
        m = None if mask is None else mask[:, a:b]
        i = None if ids is None else ids[..., a:b]
        result[case] = sequence_positions(batch, b - a, m, i, device=torch.device("cpu"))
    torch.save(result, os.path.join(out_dir, f"rank{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


def test_sequence_parallel_positions_are_slices_of_the_whole_sequence(tmp_path) -> None:
    from lsso import LSSO

    mp.spawn(_seq_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    ranks = [torch.load(tmp_path / f"rank{r}.pt") for r in range(2)]
    for case in _SEQ_CASES:
        batch, length, mask, ids = _seq_inputs(case)
        all_valid = mask is None
        if all_valid and ids is None:
            full = torch.arange(length, dtype=torch.float32) - 0.5 * (length - 1)
        else:
            centered = LSSO._center_positions(ids, mask, dtype=torch.float32, all_valid=all_valid, batch=batch,
                                              length=length, device=torch.device("cpu"))
            full = centered[0] if (all_valid and (ids is None or ids.dim() == 1)) else centered
        counts = (torch.full((batch,), float(length)) if all_valid
                  else mask.sum(-1).float().clamp_min(1.0))
        for r in range(2):
            positions, got_counts, offset, total = ranks[r][case]
            a, b = _SEQ_CUTS[r], _SEQ_CUTS[r + 1]
            assert (offset, total) == (a, length), case
            assert torch.equal(positions, full[..., a:b].contiguous()), case
            assert torch.equal(got_counts, counts), case


def test_gradient_slot_registry_keys_by_identity() -> None:
    """Slots are found by parameter identity (tensors compare elementwise, so an
    equality-keyed mapping would fail on any multi-element parameter)."""
    from lsso_b200.ball import projection

    a = torch.nn.Parameter(torch.zeros(4, 4))
    b = torch.nn.Parameter(torch.zeros(4, 4))  # equal values, another parameter
    slot = torch.empty(4, 4)
    projection.register_gradient_slot(a, slot, None)
    try:
        assert projection._slot_for(a)[0] is slot
        assert projection._slot_for(b) is None
        a.grad = torch.zeros(4, 4)
        assert projection._slot_for(a) is None  # an existing gradient accumulates instead
    finally:
        projection.register_gradient_slot(a, None)
    a.grad = None
    assert projection._slot_for(a) is None


def test_exchange_transport_choice_without_a_process_group() -> None:
    """One process: no exchange at all ("none"), whatever transport is asked;
    an unknown transport name is rejected before any hook is installed."""
    from lsso import LSSO, LSSOConfig
    from lsso_b200.ball.distributed import GradientExchange, layer_buckets

    layer = LSSO(LSSOConfig(32, 2, 16, bias=True))
    with pytest.raises(ValueError, match="transport must be"):
        GradientExchange(layer_buckets(layer), transport="mpi")
    for transport in ("auto", "peer", "nccl"):
        exchange = GradientExchange(layer_buckets(layer), transport=transport)
        assert exchange.transport == "none"
        assert exchange.averaged is exchange.flat
        exchange.close()


def test_buckets_go_out_in_bucket_order_whatever_order_they_complete() -> None:
    """Every rank must launch its bucket exchanges in the same order (each launch of the peer
    exchange pairs with the peers' launch of the same number): a bucket that completes before an
    earlier one waits for it, and finish() launches what is left in order.  Each bucket also starts
    at a multiple of four values (16-byte aligned parts of the exchange region)."""
    from lsso import LSSO, LSSOConfig
    from lsso_b200.ball.distributed import GradientExchange

    layer = LSSO(LSSOConfig(36, 2, 16, bias=True))
    params = list(layer.parameters())
    buckets = [[params[0]], [params[1], params[2]], [params[3]], params[4:]]
    exchange = GradientExchange(buckets)
    order: list[int] = []
    real_launch = exchange._launch

    def record(k: int) -> None:
        order.append(k)
        real_launch(k)

    exchange._launch = record
    try:
        assert all(start % 4 == 0 for start in exchange.bucket_start)
        for k, bucket in enumerate(buckets):
            for p in bucket:
                assert exchange.slot[p].data_ptr() >= exchange.flat.data_ptr() + 4 * exchange.bucket_start[k]
        # bucket 2 completes first, then 0 (which releases 0 only: 1 is still open), then 1 (releases 1, 2)
        for p in buckets[2]:
            exchange._mark(p)
        assert order == []
        for p in buckets[0]:
            exchange._mark(p)
        assert order == [0]
        for p in buckets[1]:
            exchange._mark(p)
        assert order == [0, 1, 2]
        exchange.finish()  # bucket 3 never completed: zero-filled and launched last
        assert order == [0, 1, 2, 3]
        assert all(torch.count_nonzero(p.grad) == 0 for p in buckets[3])
        order.clear()
        exchange.finish()  # a step with no backward at all: every bucket, in order
        assert order == [0, 1, 2, 3]
    finally:
        exchange.close()
