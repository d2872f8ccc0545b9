"""Framework drivers: the sequence shell (pre-norm residual LSSO blocks) and vision position IDs."""

from __future__ import annotations

import pytest
import torch

from lsso import LSSO, LSSOConfig
from lsso_b200.ball.shell import SequenceShell, vision_position_ids


def test_vision_position_ids_put_the_class_token_at_zero_and_center_the_patches() -> None:
    assert vision_position_ids(0).numel() == 0
    assert vision_position_ids(1).tolist() == [0.0]
    assert vision_position_ids(2).tolist() == [0.0, 0.0]
    assert vision_position_ids(5).tolist() == [0.0, -1.5, -0.5, 0.5, 1.5]
    ids = vision_position_ids(197)  # 14 x 14 patches + class token
    assert ids.dtype == torch.float32 and ids[0] == 0 and ids[1:].sum() == 0


def test_shell_blocks_are_pre_norm_residual_lsso_layers() -> None:
    torch.manual_seed(0)
    shell = SequenceShell(LSSOConfig(32, 2, 16), depth=2, vocab=8).double()
    ids = torch.randint(0, 8, (2, 11))
    mask = torch.ones(2, 11, dtype=torch.bool)
    mask[1, 7:] = False
    out = shell(ids, mask)
    x = torch.where(mask[:, :, None], shell.embedding(ids), torch.zeros(1, dtype=torch.float64))
    for block in shell.blocks:
        x = x + block.mixer(block.norm1(x), valid_mask=mask)
        x = torch.where(mask[:, :, None], x, torch.zeros_like(x))
    torch.testing.assert_close(out, x)
    assert torch.count_nonzero(out[1, 7:]) == 0
    assert shell.embedding.weight.std().item() < 0.05


@pytest.mark.gpu
def test_shell_cuda_matches_the_reference_path_in_bf16() -> None:
    from tests.gpu_util import relative_l2, require_native

    require_native()
    torch.manual_seed(0)
    shell = SequenceShell(LSSOConfig(128, 4, 48), depth=4, vocab=8).cuda()
    ids = torch.randint(0, 8, (2, 300), device="cuda")
    mask = torch.ones(2, 300, dtype=torch.bool, device="cuda")
    mask[1, 200:] = False

    def run(implementation, amp):
        for p in shell.parameters():
            p.grad = None
        with torch.autocast("cuda", dtype=torch.bfloat16, enabled=amp):
            y = shell(ids, mask, implementation=implementation)
        y.float().square().mean().backward()
        return y.detach().float(), [p.grad.detach().clone() for p in shell.parameters()]

    # BF16 CUDA blocks against the FP32 reference path of the same shell.  Four
    # BF16 layers compound their roundings, so each bound (output and every
    # gradient) is the larger of the per-layer BF16 budget (1e-2) and 1.25x the
    # error of the reference path's own BF16 (autocast) run of the same tensor.
    y_cuda, g_cuda = run("cuda", True)
    y_ref, g_ref = run("reference", False)
    y_bf16, g_bf16 = run("reference", True)
    e, e_ref = relative_l2(y_cuda, y_ref), relative_l2(y_bf16, y_ref)
    print(f"shell output rel L2: cuda {e:.2e}, reference path in BF16 {e_ref:.2e}")
    assert e <= max(1e-2, 1.25 * e_ref)
    for (name, _), a, b, c in zip(shell.named_parameters(), g_cuda, g_ref, g_bf16):
        ge, ge_ref = relative_l2(a, b), relative_l2(c, b)
        print(f"shell grad {name}: cuda {ge:.2e}, reference path in BF16 {ge_ref:.2e}")
        assert ge <= max(1e-2, 1.25 * ge_ref), (name, ge, ge_ref)
