"""Parity of the sm_100a mixer with the oracle and the reference's golden fixtures.

Each case is checked twice:

* against the oracle with the contract's roundings (FP16 Rank-Rotary phases,
  the BF16 upstream gradient the native backward receives): relative L2
  <= 5e-3 for the output and for every gradient and max|actual - expected|
  <= MAXABS x max|expected| per tensor -- the error of the kernels' own
  arithmetic;
* against the exact FP64 operator with the FP32 upstream (the reference
  tests' oracle, tests/cuda/test_fast_path.py:33-86): relative L2 <= 1e-2
  for every tensor -- the contract's roundings included.  The reference's own
  CUDA suite allows 3e-2 for gradients there (test_fast_path.py:737-742).

The complement gradient of the narrow-head and tail fixtures keeps the
reference's 1e-2 (test_fast_path.py:745-856).  Measured values are printed.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import lsso_oracle as O
from tests.golden_io import load_mixer_case, mixer_case_names
from tests.gpu_util import (max_abs, relative_l2, require_native, run_cuda, run_oracle, scaled_max_abs,
                            seeded_mixer_inputs)

pytestmark = pytest.mark.gpu

FWD = 5e-3
GRAD = 5e-3
EXACT = 1e-2  # against the exact FP64 operator
# max|actual - expected| <= MAXABS * max|expected|, per tensor: BF16 outputs
# and operands put single elements a few BF16 ulps (2^-8 relative) off.
MAXABS = 1e-2
GRAD_NAMES = ("projected", "core_base_raw", "core_drive_weight", "eta_raw")


@pytest.fixture(scope="module", autouse=True)
def native() -> None:
    require_native()


def _check(out, grads, ref_out, ref_grads, *, fwd=FWD, grad=GRAD, maxabs=MAXABS, label="", exact=None):
    """Compare with the contract oracle (``ref_*``) and, given ``exact = (out, grads)``
    of the exact FP64 operator, with that at EXACT.  Prints relL2/scaled-maxabs."""
    assert torch.isfinite(out.float()).all()
    e, m = relative_l2(out, ref_out), scaled_max_abs(out, ref_out)
    line = [f"{label} fwd={e:.2e}/{m:.2e}"]
    assert e <= fwd and m <= maxabs, line
    if grads is not None:
        for name, g, r in zip(GRAD_NAMES, grads, ref_grads):
            assert torch.isfinite(g.float()).all(), name
            ge, gm = relative_l2(g, r), scaled_max_abs(g, r)
            line.append(f"{name}={ge:.2e}/{gm:.2e}")
            assert ge <= grad and gm <= maxabs, (name, line)
    if exact is not None:
        xe = [relative_l2(out, exact[0])] + ([] if grads is None else
                                             [relative_l2(g, r) for g, r in zip(grads, exact[1])])
        line.append("exact=" + ",".join(f"{v:.2e}" for v in xe))
        assert max(xe) <= EXACT, line
    print(" ".join(line))


def _both(p, b, d, e, pos, counts, up):
    """(contract oracle) and (exact FP64 operator) on the same inputs."""
    return run_oracle(p, b, d, e, pos, counts, up), run_oracle(p, b, d, e, pos, counts, up, contract=False)


@pytest.mark.parametrize("name", mixer_case_names())
def test_golden_fixtures(name: str) -> None:
    case = load_mixer_case(name)
    t = lambda k: torch.from_numpy(case[k])  # noqa: E731
    out, grads = run_cuda(t("projected"), t("core_base_raw"), t("core_drive_weight"), t("eta_raw"),
                          case["centered_positions"], case["valid_counts"], t("upstream"))
    ref = [case["grad_projected"], case["grad_core_base_raw"], case["grad_core_drive_weight"], case["grad_eta_raw"]]
    fwd = 1e-2 if "scale64" in name else FWD
    if "narrow" in name or "tail" in name:
        assert relative_l2(grads[3], ref[3]) <= 1e-2
        if "tail" in name:
            assert torch.count_nonzero(grads[3]) == case["eta_raw"].size
    if "narrow" in name:
        # N=1 with a 10x relation: the readout cancels to ~1/1600 of its terms,
        # so only the FP32 complement gradient is pinned (as in the reference's
        # narrow-head test); the absolute output error stays at BF16 level.
        assert max_abs(out, case["out"]) < 1e-2
        print(f"{name} eta_raw={relative_l2(grads[3], ref[3]):.2e}")
        return
    # the reference's own FP64 output and gradients (FP32 upstream), at the reference's budgets
    assert relative_l2(out, case["out"]) <= fwd
    assert all(relative_l2(g, r) <= 3e-2 for g, r in zip(grads, ref))
    # the contract oracle (pinned to these fixtures by tests/test_oracle.py) at this library's budgets
    contract = run_oracle(t("projected"), t("core_base_raw"), t("core_drive_weight"), t("eta_raw"),
                          case["centered_positions"], case["valid_counts"], t("upstream"))
    _check(out, grads, *contract, label=name, exact=(case["out"], ref))
    if case["valid_mask"] is not None:
        mask = torch.from_numpy(case["valid_mask"]).cuda()
        assert torch.count_nonzero(out[~mask]) == 0


@pytest.mark.parametrize("length", (31, 32, 33, 65, 127, 128, 129, 255, 256, 257, 511, 512, 513))
def test_lengths_match_oracle(length: int) -> None:
    p, b, d, e, up = seeded_mixer_inputs(19 + length, 1, length, 2, 16, 16, core=0.1, eta=0.1)
    pos = np.arange(length, dtype=np.float32)
    pos = pos - pos.mean()
    out, grads = run_cuda(p, b, d, e, pos, None, up)
    contract, exact = _both(p, b, d, e, pos, None, up)
    _check(out, grads, *contract, label=f"N={length}", exact=exact)


EXPANDED = [
    (1, 16, 1, 1, 31), (1, 16, 1, 15, 31), (1, 16, 1, 17, 31), (1, 16, 1, 31, 33), (1, 16, 1, 32, 33),
    (1, 16, 1, 33, 33), (1, 16, 1, 257, 33), (1, 16, 1, 512, 33), (1, 32, 2, 48, 31), (2, 32, 3, 17, 35),
    (1, 48, 2, 96, 33), (1, 64, 1, 33, 33), (1, 64, 1, 257, 33), (1, 16, 1, 17, 2048), (1, 32, 1, 17, 2048),
    (1, 48, 1, 17, 2048), (1, 64, 1, 17, 2048), (1, 16, 1, 17, 2017), (1, 64, 1, 17, 2017), (1, 64, 1, 17, 4096),
    (1, 32, 8, 32, 4096), (1, 16, 4, 32, 4776), (1, 32, 1, 17, 8193), (2, 64, 2, 384, 40), (1, 48, 3, 256, 70),
    # head-group tile kernels: r = 64 with d = 32 (gradient pass per head), r = 64 / d = 64, r = 32 / d = 64
    (2, 64, 2, 32, 300), (1, 64, 2, 64, 300), (1, 32, 2, 64, 300), (1, 64, 4, 32, 1100),
    # r = 48 tiles: two heads per group (relation boxes partly owned), and one head per group at d = 64
    (2, 48, 2, 32, 300), (1, 48, 4, 32, 1100), (1, 48, 2, 64, 333), (1, 48, 8, 32, 4096),
    # r = 16 tiles: four heads per group
    (2, 16, 4, 32, 300), (1, 16, 8, 32, 2049),
]


@pytest.mark.parametrize(("batch", "rank", "heads", "head_dim", "length"), EXPANDED)
def test_expanded_shapes_match_oracle(batch, rank, heads, head_dim, length) -> None:
    p, b, d, e, up = seeded_mixer_inputs(71 + batch + rank + head_dim, batch, length, heads, rank, head_dim)
    pos = np.arange(length, dtype=np.float32)
    pos = pos - pos.mean()
    out, grads = run_cuda(p, b, d, e, pos, None, up)
    contract, exact = _both(p, b, d, e, pos, None, up)
    _check(out, grads, *contract, label=f"{(batch, rank, heads, head_dim, length)}", exact=exact)


@pytest.mark.parametrize(("rank", "head_dim", "length"),
                         [(16, 17, 35), (32, 64, 35), (48, 96, 35), (64, 257, 35), (16, 17, 2048), (64, 17, 2017),
                          (48, 32, 513), (32, 32, 513)])
def test_masked_batch_specific_positions_match_oracle(rank, head_dim, length) -> None:
    pattern = torch.tensor([True, False, True, True, False, True, True])
    first = pattern.repeat((length + 6) // 7)[:length]
    mask = torch.stack((first, torch.zeros(length, dtype=torch.bool)))
    ids = torch.stack((3 * torch.arange(length) + 7, 5 * torch.arange(length) + 101))
    from lsso import LSSO

    positions = LSSO._center_positions(ids, mask, dtype=torch.float32, all_valid=False)
    counts = mask.sum(-1).float().clamp_min(1.0)
    p, b, d, e, up = seeded_mixer_inputs(97 + rank + head_dim, 2, length, 2, rank, head_dim, mask=mask)
    out, grads = run_cuda(p, b, d, e, positions, counts, up)
    assert torch.count_nonzero(out[~mask.cuda()]) == 0
    assert torch.count_nonzero(grads[0][~mask.cuda()]) == 0
    contract, exact = _both(p, b, d, e, positions, counts, up)
    _check(out, grads, *contract, label=f"masked {(rank, head_dim, length)}", exact=exact)


@pytest.mark.parametrize(("rank", "head_dim", "length"),
                         [(16, 16, 33), (32, 64, 33), (64, 128, 33), (16, 16, 2017), (64, 128, 2049)])
def test_train_tape_and_inference_forward_agree(rank, head_dim, length) -> None:
    p, b, d, e, _ = seeded_mixer_inputs(47 + rank + head_dim, 1, length, 2, rank, head_dim, core=0.1, eta=0.1)
    args = [p.to(torch.bfloat16).cuda(), b.cuda(), d.cuda(), e.cuda()]
    with torch.inference_mode():
        inference = torch.ops.lsso_equilibrium.forward_inference(*args)
    train, tape, pivots = torch.ops.lsso_equilibrium.forward_train(*args)
    assert inference.dtype == train.dtype == torch.bfloat16
    assert tape.dtype == torch.float32 and tape.is_contiguous() and pivots.dtype == torch.int32
    assert tape.shape == (2, length * rank + 3 * rank * rank + 2 * rank * head_dim + 1)
    assert torch.equal(pivots.cpu(), torch.arange(1, rank + 1, dtype=torch.int32).repeat(2, 1))
    torch.testing.assert_close(train, inference, rtol=1e-5, atol=2e-6)


def test_contract_rejections() -> None:
    proj = torch.randn(1, 5, 32, device="cuda")
    base = torch.randn(1, 16, 16, device="cuda")
    drive = torch.randn(1, 16, 16, device="cuda")
    eta = torch.randn(1, device="cuda")
    from lsso_b200.ball import cuda

    for dtype in (torch.float16, torch.float32):
        with pytest.raises(RuntimeError, match="mixed precision CUDA contract"):
            cuda.fast_mix(proj.to(dtype), base, drive, eta)
    grads = [t.requires_grad_() for t in (base.clone(), drive.clone(), eta.clone())]
    with pytest.raises(RuntimeError, match="private tape-producing entry point"):
        torch.ops.lsso_equilibrium.forward_train(proj.bfloat16(), *grads, None)
    with pytest.raises(RuntimeError, match="inference-only entry point"):
        torch.ops.lsso_equilibrium.forward_inference(proj.bfloat16(), *grads, None)


def test_backward_requires_bf16_upstream_and_zero_upstream_gives_zero_gradients() -> None:
    projected = torch.zeros(1, 5, 32, device="cuda", dtype=torch.bfloat16)
    base = torch.zeros(1, 16, 16, device="cuda")
    drive = torch.zeros(1, 16, 16, device="cuda")
    eta = torch.zeros(1, device="cuda")
    out, tape, pivots = torch.ops.lsso_equilibrium.forward_train(projected, base, drive, eta, None)
    args = (projected, base, drive, eta, tape, pivots, None)
    with pytest.raises(RuntimeError, match="grad_output must use bfloat16"):
        torch.ops.lsso_equilibrium.backward(torch.zeros_like(out).float(), *args)
    for g in torch.ops.lsso_equilibrium.backward(torch.zeros_like(out), *args):
        assert torch.count_nonzero(g) == 0


def test_bf16_content_beyond_fp16_range() -> None:
    torch.manual_seed(101)
    projected = torch.randn(1, 33, 32)
    projected[:, :, 16:] *= 131072
    projected = projected.bfloat16().float()
    base, drive, eta = torch.zeros(1, 16, 16), torch.zeros(1, 16, 16), torch.tensor([0.7])
    upstream = torch.ones(1, 33, 16)
    out, grads = run_cuda(projected, base, drive, eta, None, None, upstream)
    assert out.float().abs().max() > torch.finfo(torch.float16).max
    contract, exact = _both(projected, base, drive, eta, None, None, upstream)
    _check(out, grads, *contract, label="bf16-range", exact=exact)


def test_results_are_deterministic() -> None:
    p, b, d, e, up = seeded_mixer_inputs(5, 2, 1500, 4, 32, 32)
    o1, g1 = run_cuda(p, b, d, e, None, None, up)
    o2, g2 = run_cuda(p, b, d, e, None, None, up)
    assert torch.equal(o1, o2)
    for x, y in zip(g1, g2):
        assert torch.equal(x, y)


def test_bench_shape_batch_slice_matches_oracle() -> None:
    """Bench shape (N=4096, H=8, r=32, d=32) on 4 samples against the FP64 oracle."""
    p, b, d, e, up = seeded_mixer_inputs(2026, 4, 4096, 8, 32, 32)
    out, grads = run_cuda(p, b, d, e, None, None, up)
    contract, exact = _both(p, b, d, e, None, None, up)
    _check(out, grads, *contract, label="bench-slice", exact=exact)


def test_full_bench_batch_is_sample_independent() -> None:
    """B=64 bench batch: every sample's output equals the output computed alone."""
    p, b, d, e, up = seeded_mixer_inputs(7, 64, 4096, 8, 32, 32)
    full, grads = run_cuda(p, b, d, e, None, None, up)
    assert all(torch.isfinite(g).all() for g in grads)
    for index in (0, 31, 63):
        alone, _ = run_cuda(p[index:index + 1], b, d, e)
        # Chunking (and so FP32 summation order) depends on the batch size; the
        # difference is a few BF16 rounding flips.
        assert relative_l2(full[index:index + 1], alone) < 2e-4


def test_device_status_is_clean() -> None:
    from lsso_b200.ball import cuda

    assert cuda.device_status(reset=False) == 0
