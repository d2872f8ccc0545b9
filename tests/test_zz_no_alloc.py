"""The allocation-free inference entry point, ``lsso_forward_inference_noalloc``.

It exists for callers that cannot call cudaMalloc where they run the mixer --
a host that owns all device memory through its own arena and forbids
allocation inside plugin calls, or a serving loop whose memory is fixed up
front.  Instead of a caller-allocated workspace it uses one fixed scratch
array inside the library.  This test calls it through the C ABI twice in a
row (two shapes, so the shared scratch is reused with a different layout) and
checks each result against the regular ``lsso_forward`` entry point: both run
the same plan and the same kernels, so the outputs must be bit-identical.  A
second test first leaves NaN-derived values throughout the scratch (a call on
NaN inputs at a shape whose scratch is just under the limit), then runs a
valid shape of that size and a small one, each again bit-identical to
``lsso_forward``: every call overwrites all the scratch it reads.  It also
checks that a shape too large for the fixed area is rejected with a clear
message.

The file name makes pytest collect it last, so a run that stops at the first
failure has already run every other test; it also passes on its own in a
fresh process (it binds the library with ctypes itself).
"""

from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

LSSO_ERR_WORKSPACE = 4
LIMIT = 32 << 20  # LSSO_NOALLOC_SCRATCH_BYTES


def _bind():
    from lsso_b200 import build

    lib = ctypes.CDLL(str(build.build()))
    i64, vp, sz, ci = ctypes.c_int64, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int
    lib.lsso_last_error.restype = ctypes.c_char_p
    lib.lsso_forward_workspace_size.restype = sz
    lib.lsso_forward_workspace_size.argtypes = [i64] * 5 + [ci, ci]
    lib.lsso_forward.restype = ci
    lib.lsso_forward.argtypes = [vp, vp, vp, vp, vp, ci, vp, i64, i64, i64, i64, i64, vp, vp, vp, vp, sz, vp]
    lib.lsso_forward_inference_noalloc.restype = ci
    lib.lsso_forward_inference_noalloc.argtypes = [vp, vp, vp, vp, vp, ci, vp, i64, i64, i64, i64, i64, vp, vp]
    return lib


def _inputs(seed, B, N, H, R, d, batched_positions):
    g = torch.Generator().manual_seed(seed)
    D = H * d
    projected = torch.randn(B, N, H * R + D, generator=g).to("cuda", torch.bfloat16)
    base = (0.05 * torch.randn(H, R, R, generator=g)).cuda()
    drive = (0.05 * torch.randn(H, d, R, generator=g)).cuda()
    eta = (0.1 * torch.randn(H, generator=g)).cuda()
    positions = counts = None
    if batched_positions:
        positions = (torch.randn(B, N, generator=g) * 50.0).cuda()
        counts = torch.full((B,), float(N)).cuda()
    return projected, base, drive, eta, positions, counts


def _ptr(t):
    return None if t is None else t.data_ptr()


def _run_pair(lib, seed, shape, batched, *, poison=False):
    """lsso_forward (own workspace) and lsso_forward_inference_noalloc on the same inputs."""
    B, N, H, R, d = shape
    stream = torch.cuda.current_stream().cuda_stream
    projected, base, drive, eta, positions, counts = _inputs(seed, B, N, H, R, d, batched)
    if poison:
        projected.fill_(float("nan"))
    D = H * d
    args = (_ptr(projected), _ptr(base), _ptr(drive), _ptr(eta), _ptr(positions), int(batched), _ptr(counts),
            B, N, H, D, R)
    expected = torch.empty(B, N, D, device="cuda", dtype=torch.bfloat16)
    size = lib.lsso_forward_workspace_size(B, N, H, D, R, int(batched), 0)
    workspace = torch.empty(size, device="cuda", dtype=torch.uint8)
    assert lib.lsso_forward(*args, expected.data_ptr(), None, None, workspace.data_ptr(), size, stream) == 0, \
        lib.lsso_last_error()
    actual = torch.full((B, N, D), float("nan"), device="cuda", dtype=torch.bfloat16)
    assert lib.lsso_forward_inference_noalloc(*args, actual.data_ptr(), stream) == 0, lib.lsso_last_error()
    torch.cuda.synchronize()
    return actual, expected, size


def test_noalloc_forward_matches_forward_on_two_calls_in_a_row() -> None:
    lib = _bind()
    cases = [(1, (2, 1500, 4, 32, 32), False), (2, (3, 333, 2, 48, 17), True)]
    for seed, shape, batched in cases:
        actual, expected, size = _run_pair(lib, seed, shape, batched)
        print(f"noalloc call {seed}: shape {shape}, {size} bytes of scratch")
        assert torch.isfinite(actual.float()).all()
        assert torch.equal(actual, expected)


def test_noalloc_reads_nothing_a_previous_call_left_behind() -> None:
    lib = _bind()
    # The longest sequence (B=1, H=8, r=32, d=32) whose scratch still fits the area.
    best = None
    for N in range(1024, 1 << 20, 1024):
        size = lib.lsso_forward_workspace_size(1, N, 8, 256, 32, 0, 0)
        if size <= LIMIT:
            best = (N, size) if best is None or size > best[1] else best
        elif size > 2 * LIMIT:
            break
    assert best is not None and best[1] > LIMIT // 2, best
    near = (1, best[0], 8, 32, 32)
    poisoned, _, _ = _run_pair(lib, 5, near, False, poison=True)
    assert not torch.isfinite(poisoned.float()).all()  # NaN-derived values now fill the used scratch
    for seed, shape in ((6, near), (7, (2, 257, 2, 16, 16))):
        actual, expected, size = _run_pair(lib, seed, shape, False)
        print(f"after a NaN call: shape {shape}, {size} of {LIMIT} bytes")
        assert torch.isfinite(actual.float()).all()
        assert torch.equal(actual, expected)


def test_noalloc_rejects_shapes_beyond_its_scratch() -> None:
    lib = _bind()
    projected, base, drive, eta, _, _ = _inputs(3, 1, 64, 1, 16, 16, False)
    mixed = torch.empty(1, 64, 16, device="cuda", dtype=torch.bfloat16)
    # 256 x 16384 tokens, 8 heads of rank 64: far more than the fixed area.
    B, N, H, D, R = 256, 16384, 8, 512, 64
    assert lib.lsso_forward_workspace_size(B, N, H, D, R, 0, 0) > (32 << 20)
    rc = lib.lsso_forward_inference_noalloc(projected.data_ptr(), base.data_ptr(), drive.data_ptr(), eta.data_ptr(),
                                            None, 0, None, B, N, H, D, R, mixed.data_ptr(),
                                            torch.cuda.current_stream().cuda_stream)
    assert rc == LSSO_ERR_WORKSPACE
    message = lib.lsso_last_error().decode()
    assert "scratch" in message and "lsso_forward" in message
