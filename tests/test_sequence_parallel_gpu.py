"""Sequence-parallel mixer: tokens of each sample split over ranks, one moment all-reduce per pass.

On one GPU the ranks are emulated through the C ABI (each shard's moment
pass, the moments summed by hand, each shard's finish), and compared with
the unsplit mixer and the oracle; a one-rank process group must reproduce
the unsplit layer bit for bit; with two or more GPUs, two NCCL ranks run the
layer end to end and are compared with one GPU's unsplit result.
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from tests.gpu_util import relative_l2, require_native, run_oracle, seeded_mixer_inputs

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module", autouse=True)
def native() -> None:
    require_native()


def _shards(length: int, parts: int) -> list[tuple[int, int]]:
    cuts = np.linspace(0, length, parts + 1).round().astype(int)
    return [(int(a), int(b)) for a, b in zip(cuts[:-1], cuts[1:])]


def _emulated(projected, base, drive, eta, positions, counts, upstream, parts: int):
    """Every shard's moment pass, the moments summed in rank order, every shard's finish."""
    from lsso_b200.ball import _native

    spans = _shards(projected.shape[1], parts)
    batched = positions.dim() == 2
    piece = lambda t, a, b: t[:, a:b].contiguous()  # noqa: E731
    ppiece = lambda a, b: (positions[:, a:b] if batched else positions[a:b]).contiguous()  # noqa: E731
    moments = sum(_native.forward_moments(piece(projected, a, b), base, drive, eta, ppiece(a, b)) for a, b in spans)
    outs, tapes = [], []
    for a, b in spans:
        out, tape, _ = _native.forward_finish(piece(projected, a, b), base, drive, eta, ppiece(a, b), counts, moments,
                                              train=True)
        outs.append(out)
        tapes.append(tape)
    grad = upstream.to(torch.bfloat16)
    bmoments = sum(_native.backward_moments(piece(grad, a, b), piece(projected, a, b), base, drive, eta, ppiece(a, b))
                   for a, b in spans)
    gproj, gb, gd, ge = [], 0, 0, 0
    for k, (a, b) in enumerate(spans):
        g = _native.backward_finish(piece(grad, a, b), piece(projected, a, b), base, drive, eta, tapes[k],
                                    ppiece(a, b), bmoments, 1.0 if k == 0 else 0.0)
        gproj.append(g[0])
        gb, gd, ge = gb + g[1], gd + g[2], ge + g[3]
    return torch.cat(outs, dim=1), (torch.cat(gproj, dim=1), gb, gd, ge)


@pytest.mark.parametrize(("batch", "rank", "heads", "head_dim", "length", "parts", "masked"), [
    (2, 32, 8, 32, 1000, 2, False),   # head-group tile kernels
    (1, 32, 8, 32, 4096, 4, False),
    (2, 64, 2, 32, 700, 3, True),     # r = 64 tiles, masked, per-sample positions
    (1, 16, 3, 17, 301, 2, False),    # per-head kernels
    (1, 48, 2, 24, 333, 3, True),
])
def test_emulated_ranks_match_unsplit(batch, rank, heads, head_dim, length, parts, masked) -> None:
    from lsso import LSSO
    from lsso_b200.ball import _native

    mask = None
    if masked:
        g = torch.Generator().manual_seed(3)
        lens = torch.randint(length // 3, length + 1, (batch,), generator=g)
        mask = torch.arange(length)[None, :] < lens[:, None]
    p, b, d, e, up = seeded_mixer_inputs(11 + rank + length, batch, length, heads, rank, head_dim, mask=mask)
    if mask is None:
        pos = (torch.arange(length, dtype=torch.float32) - 0.5 * (length - 1))
        counts = torch.full((batch,), float(length))
    else:
        ids = torch.where(mask, torch.arange(length)[None, :].expand(batch, length), torch.zeros(1, dtype=torch.long))
        pos = LSSO._center_positions(ids, mask, dtype=torch.float32, all_valid=False)
        counts = mask.sum(-1).float().clamp_min(1.0)
    cu = lambda t: t.cuda().contiguous()  # noqa: E731
    P, B_, D_, E_ = cu(p.to(torch.bfloat16)), cu(b), cu(d), cu(e)
    pos_c, cnt_c, up_c = cu(pos), cu(counts), cu(up)
    out, grads = _emulated(P, B_, D_, E_, pos_c, cnt_c, up_c, parts)
    ref_out, tape, pivots = _native.forward(P, B_, D_, E_, pos_c, cnt_c, train=True)
    ref_grads = _native.backward(up_c.to(torch.bfloat16), P, B_, D_, E_, tape, pivots, pos_c, cnt_c)
    torch.cuda.synchronize()
    assert relative_l2(out, ref_out) <= 2e-3
    for g, r in zip(grads, ref_grads):
        assert relative_l2(g, r) <= 2e-3
    if mask is not None:
        assert torch.count_nonzero(out[~mask.cuda()]) == 0
    # and against the oracle (the reference algorithm on the unsplit sequence)
    o_out, o_grads = run_oracle(p, b, d, e, pos, counts, up.to(torch.bfloat16).float())
    assert relative_l2(out, o_out) <= 5e-3
    for g, r in zip(grads, o_grads):
        assert relative_l2(g, r) <= 5e-3


def test_one_rank_group_reproduces_the_layer_bit_for_bit(tmp_path) -> None:
    import torch.distributed as dist

    from lsso import LSSO, LSSOConfig
    from lsso_b200.ball.sequence_parallel import sequence_parallel_forward

    store = dist.FileStore(str(tmp_path / "store"), 1)
    dist.init_process_group("nccl", store=store, rank=0, world_size=1)
    try:
        torch.manual_seed(0)
        layer = LSSO(LSSOConfig(256, 8, 32)).cuda()
        x = torch.randn(2, 1000, 256, device="cuda").half().requires_grad_()
        with torch.autocast("cuda", dtype=torch.float16):
            y = sequence_parallel_forward(layer, x)
        y.float().square().mean().backward()
        grads = [x.grad.clone()] + [q.grad.clone() for q in layer.parameters()]
        x.grad = None
        for q in layer.parameters():
            q.grad = None
        with torch.autocast("cuda", dtype=torch.float16):
            y2 = layer(x, implementation="cuda")
        y2.float().square().mean().backward()
        grads2 = [x.grad] + [q.grad for q in layer.parameters()]
        assert torch.equal(y, y2)
        for g, h in zip(grads, grads2):
            assert torch.equal(g, h)
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_nccl_ranks_match_one_gpu() -> None:
    env = dict(os.environ, MASTER_ADDR="127.0.0.1", MASTER_PORT="29531", PYTHONPATH=str(ROOT))
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr", "127.0.0.1", "--master-port", "29531", str(ROOT / "tests" / "sequence_parallel_ranks.py")]
    result = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    assert result.returncode == 0, result.stdout[-3000:] + result.stderr[-3000:]
    assert "sequence-parallel ok" in result.stdout
