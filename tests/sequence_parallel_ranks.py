"""Two NCCL ranks run the sequence-parallel layer; rank 0 compares with the unsplit layer.

Launched by tests/test_sequence_parallel_gpu.py through torch.distributed.run
(one process per GPU).  Prints "sequence-parallel ok" on success.
"""

from __future__ import annotations

import os
import sys
from datetime import timedelta
from pathlib import Path

import torch
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))


def main() -> int:
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
    rank, world = dist.get_rank(), dist.get_world_size()
    from lsso import LSSO, LSSOConfig
    from lsso.ball import cuda
    from lsso_b200.ball.distributed import allreduce_gradients
    from lsso_b200.ball.sequence_parallel import sequence_parallel_forward

    cuda.load(device=local)
    torch.manual_seed(0)
    layer = LSSO(LSSOConfig(256, 8, 32)).to(device)
    gen = torch.Generator(device="cpu").manual_seed(7)
    batch, length = 2, 3000
    x_full = torch.randn(batch, length, 256, generator=gen).half()
    lens = torch.tensor([length, 2100])
    mask_full = torch.arange(length)[None, :] < lens[:, None]
    cuts = [0, 1400, length]  # unequal slices
    a, b = cuts[rank], cuts[rank + 1]
    x = x_full[:, a:b].contiguous().to(device).requires_grad_()
    mask = mask_full[:, a:b].contiguous().to(device)
    with torch.autocast("cuda", dtype=torch.float16):
        y = sequence_parallel_forward(layer, x, valid_mask=mask)
    # the loss of the whole sequence is the sum of the ranks' parts
    (y.float().square().sum() / (batch * length * 256)).backward()
    params = list(layer.parameters())
    allreduce_gradients(params, average=False)
    parts = [torch.empty(batch, cuts[r + 1] - cuts[r], 256, dtype=y.dtype, device=device) for r in range(world)]
    dist.all_gather(parts, y.detach().contiguous())
    dx_parts = [torch.empty_like(p) for p in parts]
    dist.all_gather(dx_parts, x.grad.contiguous())
    ok = True
    if rank == 0:
        xf = x_full.to(device).requires_grad_()
        with torch.autocast("cuda", dtype=torch.float16):
            ref = layer(xf, valid_mask=mask_full.to(device), implementation="cuda")
        grads_sp = [q.grad.clone() for q in params]
        for q in params:
            q.grad = None
        ref.float().square().mean().backward()
        rel = lambda u, v: float((u.float() - v.float()).norm() / v.float().norm().clamp_min(1e-30))  # noqa: E731
        checks = [("y", rel(torch.cat(parts, 1), ref), 2e-3), ("dx", rel(torch.cat(dx_parts, 1), xf.grad), 5e-3)]
        names = [n for n, _ in layer.named_parameters()]
        checks += [(n, rel(g, q.grad), 5e-3) for n, g, q in zip(names, grads_sp, params)]
        for name, value, bound in checks:
            print(f"{name}: rel L2 {value:.2e} (bound {bound:g})")
            ok &= value <= bound
    flag = torch.tensor([1 if ok else 0], device=device)
    dist.broadcast(flag, 0)
    dist.destroy_process_group()
    if rank == 0 and flag.item():
        print("sequence-parallel ok")
    return 0 if flag.item() else 1


if __name__ == "__main__":
    raise SystemExit(main())
