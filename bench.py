"""Throughput of the LSSO mixer layer on B200: tokens/s forward+backward.

Workload (BASELINE config 2 at L=4096): ``LSSO(LSSOConfig(256, 8, 32))`` with
seeded default init, x ~ N(0,1) cast to FP16 of shape [64, 4096, 256] per GPU
(weak scaling: the batch grows with the number of ranks), shared positions,
one step = forward + ``loss = y.float().square().mean()`` + backward (x
carries a gradient, as in the reference's benchmarks/benchmark_ball.py) and,
with several GPUs, one NCCL all-reduce of the flat gradient buffer.

``python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]``
prints one JSON line (rank 0).  ``--impl reference`` times the CPU oracle
restatement of the reference algorithm on the host cores instead.  The shape
options (``--dim --heads --rank --batch --seq --bf16 --masked``) measure the
other BASELINE configs and ranks the same way; their lines carry no
``vs_baseline`` (the published figure is for the headline shape only).
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

METRIC = "LSSO mixer tokens/s fwd & fwd+bwd (L=4096,r=32) 1–8 B200; % HBM roofline"
DIM, HEADS, RANK = 256, 8, 32
# The reference's published fwd+bwd time at this shape (B=64, N=4096, its native CUDA path, contract 6)
# on one RTX 5070 Ti: 29.160 ms per step, i.e. 8.99 M tokens/s.
PUBLISHED_FWD_BWD = 64 * 4096 / 29.160e-3


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--batch", type=int, default=64, help="samples per GPU")
    ap.add_argument("--seq", type=int, default=4096)
    ap.add_argument("--cpu-seconds", type=float, default=12.0, help="CPU baseline sample budget")
    # Other shapes (the defaults are the headline workload; these reproduce the other BASELINE configs
    # and ranks as throughput lines, e.g. --rank 64 --batch 32 --seq 2048 --bf16 --masked for config 3).
    ap.add_argument("--dim", type=int, default=DIM)
    ap.add_argument("--heads", type=int, default=HEADS)
    ap.add_argument("--rank", type=int, default=RANK, choices=(16, 32, 48, 64))
    ap.add_argument("--bf16", action="store_true", help="BF16 activations (default FP16)")
    ap.add_argument("--masked", action="store_true",
                    help="per-sample valid prefix ~U[L/4, L], position ids arange(valid) then zeros (config 3)")
    ap.add_argument("--shell", type=int, default=0, metavar="DEPTH",
                    help="time a SequenceShell of DEPTH pre-LayerNorm residual LSSO blocks on token ids from an "
                         "embedding (vocabulary 8) instead of one layer (config 4: --shell 4 --dim 128 --heads 4 "
                         "--rank 48 --bf16)")
    return ap.parse_args()


def headline(args) -> bool:
    return (args.dim, args.heads, args.rank, args.seq, args.bf16, args.masked, args.shell) == (
        DIM, HEADS, RANK, 4096, False, False, 0)


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def workload(args, world: int) -> dict:
    name = "BASELINE config 2 (mixer bench shape)" if (args.dim, args.heads, args.rank) == (DIM, HEADS, RANK) \
        and not (args.bf16 or args.masked or args.shell) else "LSSO mixer"
    if args.shell:
        return {
            "workload": f"SequenceShell: embedding (vocabulary 8, N(0, 0.02)) + {args.shell} pre-LayerNorm residual "
                        f"blocks x + LSSO(dim={args.dim}, heads={args.heads}, rank={args.rank})(LN(x)), token ids "
                        f"~U[0, 8) [B={args.batch} per GPU, {args.seq}], {'BF16' if args.bf16 else 'FP16'} autocast, "
                        "fwd+bwd with loss=y.float().square().mean()",
            "global_batch": args.batch * world,
            "seq_len": args.seq,
            "parallelism": f"dp{world}",
            "l2": "inputs larger than L2 (per layer: packed projection "
                  f"{2 * args.batch * args.seq * (args.heads * args.rank + args.dim) / 1e6:.0f} MB)",
        }
    return {
        "workload": f"{name} at L={args.seq}: LSSO(dim={args.dim}, heads={args.heads}, "
                    f"rank={args.rank}) DYNAMIC + Rank-Rotary, x [B={args.batch} per GPU, {args.seq}, {args.dim}] "
                    f"{'BF16' if args.bf16 else 'FP16'}, "
                    f"{'per-sample valid prefixes and positions' if args.masked else 'shared positions'}, "
                    "fwd+bwd with loss=y.float().square().mean()",
        "global_batch": args.batch * world,
        "seq_len": args.seq,
        "parallelism": f"dp{world}",
        "l2": "inputs larger than L2 (x 134 MB, packed projection 268 MB per GPU at the default size)",
    }


# ---------------------------------------------------------------------------- CPU legs
def cpu_fwd_bwd_tokens_per_s(seq: int, budget_s: float, steps: int | None = None, warmup: int = 1,
                             dim: int = DIM, heads: int = HEADS, rank: int = RANK):
    """Oracle restatement (FP32 reference CPU path) on one sample of the workload."""
    import numpy as np

    from oracle import lsso_oracle as O

    params = O.init_params(dim, heads, rank, seed=0)
    x = np.random.default_rng(0).standard_normal((1, seq, dim)).astype(np.float32)

    def one():
        y, state = O.module_forward(params, x, None, None, heads=heads, rank=rank, dtype=np.float32,
                                    return_state=True)
        O.module_backward(2.0 * y / y.size, state)

    for _ in range(warmup):
        one()
    times = []
    start = time.perf_counter()
    while True:
        t = time.perf_counter()
        one()
        times.append(time.perf_counter() - t)
        if steps is not None and len(times) >= steps:
            break
        if steps is None and time.perf_counter() - start >= budget_s and len(times) >= 3:
            break
    median = statistics.median(times)
    return seq / median, len(times), median


def reference_arm(args, rank: int, world: int) -> int:
    if rank != 0:
        return 0
    cores = os.cpu_count() or 1
    value, n, median = cpu_fwd_bwd_tokens_per_s(args.seq, args.cpu_seconds, steps=args.steps, warmup=args.warmup,
                                                dim=args.dim, heads=args.heads, rank=args.rank)
    sample = f"1 sample x {args.seq} tokens per step (bench shape), median of {n} steps"
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * median, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload(args, world),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "CPU NumPy restatement of the reference algorithm (oracle/lsso_oracle.py, FP32 reference-path "
                "rounding); the reference's own PyTorch code does not travel to the GPU box",
    }
    print(json.dumps(line))
    return 0


# ---------------------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str | None) -> None:
        cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "50"]
        if gpu_id:
            cmd += ["-i", gpu_id]
        try:
            self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.3)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, smax, reasons = [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for row in out.strip().splitlines():
            cols = [c.strip() for c in row.split(",")]
            if len(cols) < 9:
                continue
            try:
                sm.append(float(cols[1]))
                smax.append(float(cols[2]))
            except ValueError:
                continue
            for name, flag in zip(names, cols[5:9]):
                if flag.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------- GPU arm
def algorithmic_bytes(kernel: str, B: int, N: int, dim: int = DIM, heads: int = HEADS,
                      rank: int = RANK) -> float | None:
    """Compulsory HBM bytes of one launch of our kernels at this workload (2-byte elements)."""
    D, W, HR = dim, heads * rank + dim, heads * rank
    T = B * N
    table = {
        "moments_fwd": 2 * W * T,            # read the packed projection once
        "readout": (2 * W + 2 * D) * T,      # read projection, write mixed coordinates
        "moments_bwd": (2 * HR + 2 * D) * T,  # read relation and the upstream gradient
        "grad": (2 * D + 4 * W) * T,         # read dY and projection, write the packed gradient
        # projection GEMMs, averaged over the launches of one step: x->projected, mixed->y,
        # dy->dmixed, dprojected->dx (4 launches) and the two weight gradients (read g and x)
        "linear": (12 * D + 4 * W) * T / 4,
        "wgrad": (2 * W + 6 * D) * T / 2,
    }
    return table.get(kernel)


def bind_near_gpu(uuid: str | None):
    """Run this thread on the host cores NVML lists as closest to the GPU (its
    NUMA node), so that the pinned host copy of x, allocated afterwards, sits
    in that node's memory and the host-to-device copies do not cross the
    sockets.  Returns the previous affinity (None if nothing changed)."""
    if uuid is None or not hasattr(os, "sched_setaffinity"):
        return None
    try:
        import pynvml

        pynvml.nvmlInit()
        handle = pynvml.nvmlDeviceGetHandleByUUID(uuid)
        words = ((os.cpu_count() or 64) + 63) // 64
        mask = pynvml.nvmlDeviceGetCpuAffinity(handle, words)
        near = {64 * w + bit for w, m in enumerate(mask) for bit in range(64) if (m >> bit) & 1}
        previous = os.sched_getaffinity(0)
        near &= previous
        if not near or near == previous:
            return None
        os.sched_setaffinity(0, near)
        return previous
    except Exception:  # noqa: BLE001  (no NVML: leave the affinity as it is)
        return None


def measured_peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.is_file():
        data = json.loads(path.read_text())
        return {"hbm_gbs": data["hbm_gbs"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


def traffic_record() -> dict:
    path = ROOT / "profiles" / "dram_traffic.json"
    return json.loads(path.read_text()) if path.is_file() else {}


def gpu_arm(args, rank: int, world: int, local: int) -> int:
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=device)
    from lsso import LSSO, LSSOConfig
    from lsso.ball import cuda
    from lsso_b200.ball import _native

    cuda.load(device=local)
    torch.manual_seed(0)
    gen = torch.Generator(device=device).manual_seed(1234 + rank)
    B, N = args.batch, args.seq
    act = torch.bfloat16 if args.bf16 else torch.float16
    if args.shell:
        from lsso_b200.ball.shell import SequenceShell

        model = SequenceShell(LSSOConfig(args.dim, args.heads, args.rank), depth=args.shell, vocab=8).to(device)
        layer = model.blocks[0].mixer
        x = torch.randint(0, 8, (B, N), device=device, generator=gen)
    else:
        model = layer = LSSO(LSSOConfig(args.dim, args.heads, args.rank)).to(device)
        x = torch.randn(B, N, args.dim, device=device, generator=gen).to(act).requires_grad_()
    params = list(model.parameters())
    mask = ids = None
    if args.masked:
        lens = torch.randint(N // 4, N + 1, (B,), device=device, generator=gen)
        pos = torch.arange(N, device=device)
        mask = pos[None, :] < lens[:, None]
        ids = torch.where(mask, pos[None, :].expand(B, N), torch.zeros_like(pos)[None, :])
    ab = lambda k: algorithmic_bytes(k, B, N, args.dim, args.heads, args.rank)  # noqa: E731
    from lsso_b200.ball.distributed import GradientExchange, layer_buckets

    # Several ranks: the gradient average is part of every step, captured with it: per bucket, on a
    # side stream under the rest of the backward -- on one host the library's one-shot all-reduce
    # kernel over NVLink peer memory, otherwise NCCL all-reduces.
    exchange = None
    exchange_note = None
    if world > 1:
        exchange = GradientExchange([params] if args.shell else layer_buckets(layer))
        exchange_note = {
            "peer": "library one-shot all-reduce kernel over NVLink peer memory (CUDA IPC regions), one launch "
                    "per bucket on a side stream under the backward, in the step's CUDA graph",
            "nccl": "NCCL all_reduce(AVG) per bucket on a side stream under the backward, in the step's CUDA graph",
        }[exchange.transport]

    def forward(xx):
        if args.shell:
            return model(xx, mask, implementation="cuda")
        return layer(xx, mask, ids, implementation="cuda")

    def fwd_bwd(xx):
        # cache_enabled=False: autocast's weight-cast cache must not outlive a graph capture.
        with torch.autocast("cuda", dtype=act, cache_enabled=False):
            loss = forward(xx).float().square().mean()
        loss.backward()
        if exchange is not None:
            exchange.finish()
        return loss.detach()

    def clear_grads(xx) -> None:
        for p in params:
            p.grad = None
        if xx.is_floating_point():
            xx.grad = None

    def train_step(xx):
        clear_grads(xx)
        return fwd_bwd(xx)

    def fwd_step(xx):
        with torch.inference_mode(), torch.autocast("cuda", dtype=act, cache_enabled=False):
            return forward(xx)

    def timed(fn, steps: int) -> float:
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(steps):
            fn()
        end.record()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        ms = torch.tensor([start.elapsed_time(end)], device=device)
        if world > 1:
            dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        return float(ms.item())

    def capture(fn, xx, train=True):
        """CUDA graph of fn(xx) (the same public-API calls, launches recorded once)."""
        side = torch.cuda.Stream(device)
        side.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(side):
            for _ in range(3):
                if train:
                    clear_grads(xx)
                fn(xx)
        torch.cuda.current_stream(device).wait_stream(side)
        if train:
            clear_grads(xx)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            out = fn(xx)
        # The gradients this graph writes.
        grads = [p.grad for p in params] if train else None
        return graph, out, grads

    def use_grads(grads) -> None:
        for p, g in zip(params, grads):
            p.grad = g

    for _ in range(args.warmup):
        train_step(x)
    for _ in range(max(3, args.warmup)):
        fwd_step(x)

    # Clocks and throttle reasons are sampled across every timed region below.
    gpu_uuid = None
    try:
        gpu_uuid = str(torch.cuda.get_device_properties(device).uuid)
        gpu_uuid = gpu_uuid if gpu_uuid.startswith("GPU-") else "GPU-" + gpu_uuid
    except Exception:  # noqa: BLE001
        gpu_uuid = None
    sampler = ClockSampler(gpu_uuid)
    time.sleep(0.3)  # let nvidia-smi start sampling

    # ---- eager pass with per-kernel CUDA events (kernel table, roofline, launch count)
    _native.profile_start()
    eager_ms = timed(lambda: train_step(x), args.steps)
    kernels = _native.profile_stop()

    # ---- device-resident fwd+bwd (the headline `value`): graph replay (gradient exchange included)
    torch.cuda.empty_cache()  # the eager pass's cached blocks: a graph allocates from its own pool
    train_graph, _, train_grads = capture(fwd_bwd, x)
    use_grads(train_grads)

    def graph_train_step():
        train_graph.replay()

    for _ in range(args.warmup):
        graph_train_step()
    train_ms = timed(graph_train_step, args.steps)
    # each graph's activations are released before the next capture (config 5 at B=256 on one GPU)
    del train_graph
    torch.cuda.empty_cache()

    fwd_eager_ms = timed(lambda: fwd_step(x), args.steps)
    with torch.inference_mode():
        x_inf = x.detach().clone()
        fwd_graph, _, _ = capture(fwd_step, x_inf, train=False)
        for _ in range(args.warmup):
            fwd_graph.replay()
        fwd_ms = timed(fwd_graph.replay, args.steps)
        del fwd_graph, x_inf
    torch.cuda.empty_cache()

    # ---- end to end through the public API: every step copies its x from pinned
    # host memory and reads its loss back.  Two input buffers, each with its own
    # graph; the copy of step i+1 runs on a copy stream while step i computes.
    previous_affinity = bind_near_gpu(gpu_uuid)
    x_host = x.detach().to("cpu").pin_memory()
    loss_host = torch.empty(args.steps, dtype=torch.float32).pin_memory()
    bufs = [torch.empty_like(x.detach()).requires_grad_(x.is_floating_point()) for _ in range(2)]
    with torch.no_grad():
        for buf in bufs:
            buf.copy_(x)
    graphs = [capture(fwd_bwd, buf) for buf in bufs]
    copy_stream = torch.cuda.Stream(device)
    compute = torch.cuda.current_stream(device)
    ready = [torch.cuda.Event() for _ in range(2)]
    free = [torch.cuda.Event() for _ in range(2)]
    # each copy bracketed by timing events on the copy stream: this rank's host->device rate
    copy_marks = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                  for _ in range(args.steps)]

    def issue_copy(i: int) -> None:
        k = i % 2
        copy_stream.wait_stream(compute) if i == 0 else copy_stream.wait_event(free[k])
        with torch.cuda.stream(copy_stream), torch.no_grad():
            copy_marks[i][0].record(copy_stream)
            bufs[k].copy_(x_host, non_blocking=True)
            copy_marks[i][1].record(copy_stream)
            ready[k].record(copy_stream)

    def e2e_run() -> None:
        issue_copy(0)
        for i in range(args.steps):
            if i + 1 < args.steps:
                issue_copy(i + 1)
            k = i % 2
            compute.wait_event(ready[k])
            graphs[k][0].replay()
            free[k].record(compute)
            loss_host[i].copy_(graphs[k][1].detach(), non_blocking=True)

    timed(e2e_run, 1)
    e2e_ms = timed(e2e_run, 1)
    copy_ms = statistics.median(a.elapsed_time(b) for a, b in copy_marks)
    h2d = torch.tensor([x_host.numel() * x_host.element_size() / (copy_ms / 1e3) / 1e9], device=device)
    h2d_slowest, h2d_fastest = h2d.clone(), h2d.clone()
    if world > 1:
        dist.all_reduce(h2d_slowest, op=dist.ReduceOp.MIN)
        dist.all_reduce(h2d_fastest, op=dist.ReduceOp.MAX)
    clocks = sampler.stop()
    if previous_affinity is not None:
        os.sched_setaffinity(0, previous_affinity)  # the CPU baseline below uses every host core
    status = cuda.device_status(reset=False)
    if world > 1:
        worst = torch.tensor([status], device=device)
        dist.all_reduce(worst, op=dist.ReduceOp.MAX)
        status = int(worst.item())
    del graphs

    tokens = B * N * world
    value = tokens * args.steps / (train_ms / 1e3)
    line = None
    if rank == 0:
        peaks = measured_peaks()
        ours = {k: v for k, v in kernels.items() if ab(k) is not None}
        dominant = max(ours, key=lambda k: ours[k][0]) if ours else None
        roofline = None
        if dominant is not None:
            total_ms, launches = ours[dominant]
            per_launch_s = total_ms / launches / 1e3
            alg = ab(dominant)
            achieved = alg / per_launch_s / 1e9
            traffic = traffic_record().get(dominant) if headline(args) and B == 64 else None
            roofline = {"bound": "hbm", "kernel": dominant, "achieved": achieved, "peak": peaks["hbm_gbs"],
                        "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"], "peak_source": peaks["source"],
                        "traffic": None if traffic is None else traffic.get("bytes_per_launch"),
                        "algorithmic_bytes_per_launch": alg, "avg_launch_ms": total_ms / launches}
        step_kernels = {k: {"ms_per_step": v[0] / args.steps, "launches_per_step": v[1] / args.steps,
                            **({} if ab(k) is None else {"gbs": ab(k) / (v[0] / v[1] / 1e3) / 1e9})}
                        for k, v in kernels.items()}
        cpu = None
        if world == 1:
            cpu_value, n, median = cpu_fwd_bwd_tokens_per_s(N, args.cpu_seconds, dim=args.dim, heads=args.heads,
                                                            rank=args.rank)
            sample = (f"1 sample x {N} tokens fwd+bwd (bench shape), median of {n} steps, NumPy oracle "
                      "(FP32 reference-path rounding) on all host threads")
            if args.shell:
                cpu_value /= args.shell
                sample += f"; one layer timed, rate divided by the {args.shell} layers (LayerNorm, embedding not counted)"
            cpu = {"value": cpu_value, "unit": "tokens/s", "cores": os.cpu_count() or 1, "kind": "port",
                   "sample": sample}
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": train_ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": value / PUBLISHED_FWD_BWD if headline(args) else None,
            "vs_baseline_note": "the reference's published fwd+bwd at N=4096 (8.99 M tokens/s, RTX 5070 Ti, one GPU)",
            "dtype": "bf16", "data": "synthetic",
            "config": dict(workload(args, world), **({"gradient_exchange": exchange_note} if exchange_note else {})),
            "fwd": {"value": tokens * args.steps / (fwd_ms / 1e3), "unit": "tokens/s",
                    "ms_per_step": fwd_ms / args.steps, "eager_ms_per_step": fwd_eager_ms / args.steps},
            "eager": {"value": tokens * args.steps / (eager_ms / 1e3), "unit": "tokens/s",
                      "ms_per_step": eager_ms / args.steps,
                      "note": "same step launched op by op (per-kernel events on); `value` replays it as a CUDA graph"},
            "e2e": {"value": tokens * args.steps / (e2e_ms / 1e3), "unit": "tokens/s",
                    "h2d_bytes_per_step": x_host.numel() * x_host.element_size(), "d2h_bytes_per_step": 4,
                    "ms_per_step": e2e_ms / args.steps,
                    "h2d_gbs_per_rank": {"slowest": float(h2d_slowest.item()), "fastest": float(h2d_fastest.item()),
                                         "note": "median duration of each rank's x copies (copy-stream events) "
                                                 "during the e2e run; all ranks copy at once"},
                    "note": "pinned host x -> device on a copy stream (double-buffered, overlapping the previous "
                            "step), graph-replayed fwd+bwd, loss -> pinned host, every step; the host thread runs "
                            "on the GPU's NUMA-local cores (NVML) while x is pinned and copied",
                    "numa_bound": previous_affinity is not None},
            "roofline": roofline, "kernels": step_kernels, "cpu_baseline": cpu, "clocks": clocks,
            "gpu_launches": sum(v[1] for v in kernels.values()), "device_status": status,
        }
    if world > 1:
        torch.cuda.synchronize()
        dist.barrier()  # no rank's exchange kernel still reads a peer's region
        if exchange is not None:
            exchange.close()
        dist.barrier()
        dist.destroy_process_group()
    if line is not None:
        print(json.dumps(line))
    return 0


def main() -> int:
    args = parse_args()
    rank, world, local = dist_env()
    if args.impl == "reference":
        return reference_arm(args, rank, world)
    return gpu_arm(args, rank, world, local)


if __name__ == "__main__":
    sys.exit(main())
