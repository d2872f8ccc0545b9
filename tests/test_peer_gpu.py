"""The peer-memory exchange kernel on one GPU.

A rank's exchange kernel waits for flags that the other ranks' kernels write
into its region.  On one GPU no second kernel may be made to wait on it, so
these tests plant the other ranks: their regions are ordinary regions of this
process, and the host writes their arrive / depart flags into this rank's
header before the launch.  The kernel then runs its whole protocol (signal,
wait, rank-order sum, depart, exchange count) without waiting on anything
that runs.  The timeout test leaves one flag unset, with a 2 ms limit: the
kernel must record status 2, return, and leave the context usable.
"""

from __future__ import annotations

import pytest
import torch

from tests.gpu_util import require_native

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def native() -> None:
    require_native()


def _regions(world: int, count: int, seed: int):
    from lsso_b200.ball import peer

    g = torch.Generator(device="cuda").manual_seed(seed)
    regions = [peer.PeerRegion(count, torch.device("cuda", torch.cuda.current_device())) for _ in range(world)]
    for r in regions:
        r.values.copy_(torch.randn(count, device="cuda", generator=g) * 10.0 ** (seed % 5 - 2))
    return regions


def _plant(mine, rank: int, world: int, epoch: int, *, arrive: bool = True, depart: bool = True) -> None:
    """Write the other ranks' flags for exchange `epoch` into this rank's header."""
    from lsso_b200.ball import peer

    for j in range(world):
        if j == rank:
            continue
        if arrive:
            mine.header[peer.ARRIVE + j] = epoch
        if depart:
            mine.header[peer.DEPART + j] = epoch


def _expected(regions, scale: float) -> torch.Tensor:
    total = regions[0].values.clone()
    for r in regions[1:]:
        total = total + r.values  # rank order, FP32, as the kernel sums
    return total * scale


def test_one_rank_exchange_scales_its_own_values() -> None:
    from lsso_b200.ball import _native, peer

    (mine,) = _regions(1, 10_001, seed=3)
    out = torch.full((10_004,), float("nan"), device="cuda")
    for k in range(1, 4):
        peer.allreduce([mine.ptr], 0, mine.count, out, scale=0.5)
        torch.cuda.synchronize()
        assert torch.equal(out[: mine.count], mine.values * 0.5)
        assert int(mine.header[peer.EPOCH]) == k
        assert int(mine.header[peer.COUNTER]) == 0
    assert torch.isnan(out[mine.count:]).all()  # nothing beyond count is written
    assert _native.device_status(reset=True) == 0


@pytest.mark.parametrize("world,rank,count", [(2, 0, 212_373), (2, 1, 4096), (4, 2, 3), (8, 5, 231_557),
                                              (8, 0, 0), (3, 1, 70_001)])
def test_planted_peers_full_protocol(world: int, rank: int, count: int) -> None:
    from lsso_b200.ball import _native, peer

    regions = _regions(world, count, seed=world * 10 + rank)
    mine = regions[rank]
    out = torch.empty(max(count, 1), device="cuda")
    scale = 1.0 / world
    for k in range(1, 3):
        _plant(mine, rank, world, k)
        peer.allreduce([r.ptr for r in regions], rank, count, out, scale=scale)
        torch.cuda.synchronize()
        if count:
            assert torch.equal(out[:count], _expected(regions, scale))
        assert int(mine.header[peer.EPOCH]) == k
        assert int(mine.header[peer.COUNTER]) == 0
        for j, other in enumerate(regions):  # this rank signalled every peer, arrive and depart
            if j != rank:
                assert int(other.header[peer.ARRIVE + rank]) == k
                assert int(other.header[peer.DEPART + rank]) == k
    assert _native.device_status(reset=True) == 0


def test_exchange_replays_from_a_cuda_graph() -> None:
    from lsso_b200.ball import _native, peer

    regions = _regions(2, 50_000, seed=7)
    mine = regions[0]
    out = torch.empty(50_000, device="cuda")
    _plant(mine, 0, 2, 1)  # one eager exchange first (loads the kernel outside the capture)
    peer.allreduce([r.ptr for r in regions], 0, mine.count, out, scale=0.5)
    torch.cuda.synchronize()
    stream = torch.cuda.Stream()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        peer.allreduce([r.ptr for r in regions], 0, mine.count, out, scale=0.5)
    for k in range(2, 5):
        _plant(mine, 0, 2, k)
        regions[1].values.mul_(-1.5)
        torch.cuda.synchronize()
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, _expected(regions, 0.5))
        assert int(mine.header[peer.EPOCH]) == k
    del graph
    assert _native.device_status(reset=True) == 0


def test_missing_peer_times_out_with_status_2() -> None:
    from lsso_b200.ball import _native, peer

    regions = _regions(2, 4096, seed=11)
    mine = regions[0]
    out = torch.empty(4096, device="cuda")
    _native.device_status(reset=True)
    # nobody sets rank 1's arrive flag: the bounded wait runs out after 2 ms
    peer.allreduce([r.ptr for r in regions], 0, mine.count, out, scale=0.5, wait_limit_ns=2_000_000)
    torch.cuda.synchronize()
    assert _native.device_status(reset=True) == 2
    # only the depart flag missing: the data is summed, the final wait runs out
    _plant(mine, 0, 2, 2, depart=False)
    peer.allreduce([r.ptr for r in regions], 0, mine.count, out, scale=0.5, wait_limit_ns=2_000_000)
    torch.cuda.synchronize()
    assert torch.equal(out, _expected(regions, 0.5))
    assert _native.device_status(reset=True) == 2
    from lsso.ball import cuda

    # the context stays usable: a complete exchange afterwards succeeds and reports nothing
    _plant(mine, 0, 2, 3)
    peer.allreduce([r.ptr for r in regions], 0, mine.count, out, scale=0.5)
    torch.cuda.synchronize()
    assert torch.equal(out, _expected(regions, 0.5))
    cuda.check_device_status()


def test_invalid_arguments_are_rejected() -> None:
    from lsso_b200.ball import peer

    (mine,) = _regions(1, 64, seed=1)
    out = torch.empty(64, device="cuda")
    with pytest.raises(RuntimeError, match="1 to 8 ranks"):
        peer.allreduce([mine.ptr] * 9, 0, 64, out)
    with pytest.raises(RuntimeError, match="rank 1 outside"):
        peer.allreduce([mine.ptr], 1, 64, out)
    with pytest.raises(RuntimeError, match="16-byte aligned"):
        peer.allreduce([mine.ptr], 0, 60, out[1:])
    with pytest.raises(RuntimeError, match="not an exchange region"):
        peer.allreduce([mine.ptr + 4], 0, 64, out)


def test_bucketed_exchanges_take_their_part_of_the_buffer() -> None:
    """Two exchanges per step over [0, 4096) and [4096, 10_001) (first a multiple of four), as the
    overlapped gradient exchange launches its buckets: each sums only its part, in rank order."""
    from lsso_b200.ball import _native, peer

    regions = _regions(4, 10_001, seed=17)
    rank = 1
    mine = regions[rank]
    out = torch.full((10_004,), float("nan"), device="cuda")
    parts = [(0, 4096), (4096, 10_001 - 4096)]
    epoch = 0
    for _ in range(2):
        for first, count in parts:
            epoch += 1
            _plant(mine, rank, 4, epoch)
            peer.allreduce([r.ptr for r in regions], rank, count, out[first:], scale=0.25, first=first)
            torch.cuda.synchronize()
            assert int(mine.header[peer.EPOCH]) == epoch
        assert torch.equal(out[:10_001], _expected(regions, 0.25))
        for r in regions:
            r.values.mul_(-0.5)
    assert torch.isnan(out[10_001:]).all()
    assert _native.device_status(reset=True) == 0
    with pytest.raises(RuntimeError, match="multiple of 4"):
        peer.allreduce([r.ptr for r in regions], rank, 16, out, first=6)
