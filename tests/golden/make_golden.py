"""Generate the golden fixtures that pin the NumPy oracle to the reference.

Run in a container where the reference project is importable (it is not
needed anywhere else):

    python tests/golden/make_golden.py /path/to/LSSO

It imports the reference's public module (``lsso.LSSO``), its math module
(``lsso.ball.reference``) and the FP64 ABI composition used by its CUDA tests
(``tests/cuda/test_fast_path.py:33-86``), evaluates seeded cases and stores
inputs, outputs and autograd gradients as ``.npz`` files beside this script.
The fixtures are small; every GPU-side parity test and the oracle tests read
them, never the reference itself.
"""

from __future__ import annotations

import copy
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def _load_reference(root: str):
    sys.path.insert(0, root)
    from lsso import LSSO, LSSOConfig  # noqa: F401
    source = (Path(root) / "tests" / "cuda" / "test_fast_path.py").read_text()
    head = source.split("def _relative_l2")[0].replace("pytestmark = pytest.mark.cuda", "")
    namespace: dict = {}
    exec(compile(head, "test_fast_path_head", "exec"), namespace)
    return namespace["_reference_fast_mix"], namespace["LSSO"], namespace["LSSOConfig"]


def _np(t):
    return None if t is None else t.detach().cpu().numpy()


def mixer_case(ref_mix, LSSO, name, *, batch, length, heads, rank, head_dim, seed,
               relscale=1.0, core=0.1, eta_values=None, masked=False, batched_positions=False):
    torch.manual_seed(seed)
    dim = heads * head_dim
    projected = torch.randn(batch, length, heads * rank + dim, dtype=torch.float32)
    projected[..., : heads * rank] *= relscale
    mask = None
    positions = None
    counts = None
    if masked:
        pattern = torch.tensor([True, False, True, True, False, True, True])
        first = pattern.repeat((length + 6) // 7)[:length]
        rows = [first] + [torch.rand(length) > 0.4 for _ in range(batch - 2)]
        rows.append(torch.zeros(length, dtype=torch.bool))
        mask = torch.stack(rows[:batch])
        projected = torch.where(mask[:, :, None], projected, torch.zeros_like(projected))
        ids = torch.stack([3 * torch.arange(length) + 7 + 2 * b for b in range(batch)])
        positions = LSSO._center_positions(ids, mask, dtype=torch.float32, all_valid=False)
        counts = mask.sum(-1).to(torch.float32).clamp_min(1.0)
    elif batched_positions:
        ids = torch.stack([5 * torch.arange(length) + 11 * b for b in range(batch)])
        positions = LSSO._center_positions(ids, torch.ones(batch, length, dtype=torch.bool),
                                           dtype=torch.float32, all_valid=False)
    projected = projected.to(torch.bfloat16)
    base = torch.randn(heads, rank, rank) * core
    drive = torch.randn(heads, head_dim, rank) * core
    eta = torch.randn(heads) * 0.1 if eta_values is None else torch.tensor(eta_values, dtype=torch.float32)
    upstream = torch.randn(batch, length, dim)
    if mask is not None:
        upstream = torch.where(mask[:, :, None], upstream, torch.zeros_like(upstream))
    inputs = [v.detach().double().requires_grad_() for v in (projected, base, drive, eta)]
    out = ref_mix(*inputs, positions, counts)
    grads = torch.autograd.grad((out * upstream.double()).sum(), inputs)
    np.savez_compressed(
        HERE / f"mixer_{name}.npz",
        projected=_np(projected.float()), core_base_raw=_np(base), core_drive_weight=_np(drive),
        eta_raw=_np(eta), upstream=_np(upstream),
        centered_positions=np.zeros(0, np.float32) if positions is None else _np(positions),
        valid_counts=np.zeros(0, np.float32) if counts is None else _np(counts),
        valid_mask=np.zeros(0, bool) if mask is None else _np(mask),
        out=_np(out), grad_projected=_np(grads[0]), grad_core_base_raw=_np(grads[1]),
        grad_core_drive_weight=_np(grads[2]), grad_eta_raw=_np(grads[3]),
        heads=heads, rank=rank,
    )


def module_case(LSSO, LSSOConfig, name, *, dim, heads, rank, bias, batch, length, seed,
                masked=False, position_ids=None, fp32_path=False, x_dtype=torch.float32):
    torch.manual_seed(seed)
    layer = LSSO(LSSOConfig(dim=dim, num_heads=heads, rank=rank, bias=bias))
    with torch.no_grad():
        layer.core_base_raw.normal_(0.0, 0.05)
        layer.core_drive_weight.normal_(0.0, 0.05)
    x = torch.randn(batch, length, dim)
    mask = None
    if masked:
        mask = torch.rand(batch, length) > 0.3
        mask[-1] = False
        x = torch.where(mask[:, :, None], x, torch.full_like(x, float("nan")))
    model = layer if fp32_path else copy.deepcopy(layer).double()
    xin = x.to(x_dtype) if fp32_path else x.double()
    xin = xin.detach().requires_grad_()
    y = model(xin, valid_mask=mask, position_ids=position_ids)
    upstream = torch.randn(batch, length, dim)
    params = list(model.named_parameters())
    grads = torch.autograd.grad((y.double() * upstream.double()).sum(), [xin] + [p for _, p in params],
                                allow_unused=True)
    record = dict(x=_np(x), y=_np(y.float() if fp32_path else y), upstream=_np(upstream),
                  grad_x=_np(grads[0]), dim=dim, heads=heads, rank=rank, bias=bias,
                  valid_mask=np.zeros(0, bool) if mask is None else _np(mask),
                  position_ids=np.zeros(0, np.int64) if position_ids is None else _np(position_ids))
    for (pname, p), g in zip(params, grads[1:]):
        key = pname.replace(".", "_")
        record[f"param_{key}"] = _np(dict(layer.named_parameters())[pname])
        record[f"grad_{key}"] = _np(g)
    np.savez_compressed(HERE / f"module_{name}.npz", **record)


def config1(LSSO, LSSOConfig):
    """LSSO(192,3,16), seed 0, x=randn(8,65,192), forward only."""
    torch.manual_seed(0)
    layer = LSSO(LSSOConfig(dim=192, num_heads=3, rank=16))
    x = torch.randn(8, 65, 192)
    with torch.no_grad():
        y = layer(x, position_ids=torch.arange(65))
    record = dict(x=_np(x), y=_np(y))
    for pname, p in layer.named_parameters():
        record[f"param_{pname.replace('.', '_')}"] = _np(p)
    np.savez_compressed(HERE / "config1_forward.npz", **record)


def checkpoint_case(LSSO, LSSOConfig, name, *, dim, heads, rank, bias, batch, length, seed, core=0.0):
    """A ``state_dict()`` written by the reference's own module (weights and the
    ``_extra_state`` configuration contract) plus an input and the reference's
    FP32 CPU output for it, saved with ``torch.save`` (plain tensors and a dict
    of str/int/bool, loadable with ``weights_only=True``)."""
    torch.manual_seed(seed)
    layer = LSSO(LSSOConfig(dim=dim, num_heads=heads, rank=rank, bias=bias))
    if core:
        with torch.no_grad():
            layer.core_base_raw.normal_(0.0, core)
            layer.core_drive_weight.normal_(0.0, core)
    x = torch.randn(batch, length, dim)
    with torch.no_grad():
        y = layer(x)
    record = {"config": dict(dim=dim, num_heads=heads, rank=rank, bias=bias),
              "state_dict": layer.state_dict(), "x": x, "y": y}
    torch.save(record, HERE / f"checkpoint_{name}.pt")


def checkpoints(LSSO, LSSOConfig) -> None:
    checkpoint_case(LSSO, LSSOConfig, "d32_h2_r16_bias", dim=32, heads=2, rank=16, bias=True, batch=2, length=33,
                    seed=2024, core=0.05)
    checkpoint_case(LSSO, LSSOConfig, "d64_h2_r32", dim=64, heads=2, rank=32, bias=False, batch=1, length=40,
                    seed=2025)


def main(root: str, only: str | None = None) -> None:
    ref_mix, LSSO, LSSOConfig = _load_reference(root)
    if only == "checkpoints":
        checkpoints(LSSO, LSSOConfig)
        return
    cases = [
        dict(name="r16_d8_n33", batch=2, length=33, heads=2, rank=16, head_dim=8, seed=1),
        dict(name="r32_d17_n65", batch=1, length=65, heads=3, rank=32, head_dim=17, seed=2),
        dict(name="r48_d24_n40", batch=2, length=40, heads=1, rank=48, head_dim=24, seed=3),
        dict(name="r64_d33_n129", batch=1, length=129, heads=1, rank=64, head_dim=33, seed=4),
        dict(name="r16_d1_n1_narrow", batch=1, length=1, heads=1, rank=16, head_dim=1, seed=190,
             relscale=10.0),
        dict(name="r16_d8_n7_tail", batch=1, length=7, heads=2, rank=16, head_dim=8, seed=191,
             core=0.0, eta_values=[-9.5, 9.5]),
        dict(name="r32_d16_n48_masked", batch=3, length=48, heads=2, rank=32, head_dim=16, seed=97,
             masked=True),
        dict(name="r16_d8_n24_batchpos", batch=2, length=24, heads=2, rank=16, head_dim=8, seed=5,
             batched_positions=True),
        dict(name="r32_d32_n64_scale64", batch=1, length=64, heads=1, rank=32, head_dim=32, seed=711,
             relscale=64.0),
    ]
    for case in cases:
        mixer_case(ref_mix, LSSO, **case)
    module_case(LSSO, LSSOConfig, "fp64_bias_pos", dim=32, heads=2, rank=16, bias=True, batch=2,
                length=33, seed=59, position_ids=3 * torch.arange(33) + 7)
    module_case(LSSO, LSSOConfig, "fp64_masked", dim=34, heads=2, rank=16, bias=True, batch=3,
                length=35, seed=109, masked=True)
    module_case(LSSO, LSSOConfig, "fp64_r64", dim=128, heads=1, rank=64, bias=False, batch=1,
                length=33, seed=123)
    module_case(LSSO, LSSOConfig, "fp32path_nobias", dim=64, heads=2, rank=32, bias=False, batch=2,
                length=40, seed=7, fp32_path=True)
    config1(LSSO, LSSOConfig)
    checkpoints(LSSO, LSSOConfig)


if __name__ == "__main__":
    if len(sys.argv) not in (2, 3):
        raise SystemExit("usage: python tests/golden/make_golden.py /path/to/LSSO [checkpoints]  "
                         "(the reference checkout; 'checkpoints' writes only the checkpoint fixtures)")
    main(sys.argv[1], sys.argv[2] if len(sys.argv) == 3 else None)
