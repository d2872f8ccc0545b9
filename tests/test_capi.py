"""C-ABI library checks that need no GPU: it loads, exports every declared
symbol, reports its contract, and rejects invalid sizes with clear errors."""

from __future__ import annotations

import ctypes
import re
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "lsso_equilibrium.h"


@pytest.fixture(scope="module")
def library_path() -> Path:
    from lsso_b200 import build

    return build.build()


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"LSSO_API\s+[\w\s\*]+?\b(lsso_\w+)\s*\(", text)))


def test_header_declares_the_native_entry_points() -> None:
    names = declared_functions()
    assert "lsso_forward" in names and "lsso_backward" in names
    from lsso_b200.ball import _native

    assert sorted(_native.EXPORTED_SYMBOLS) == names


def test_library_exports_every_declared_symbol(library_path: Path) -> None:
    out = subprocess.run(["nm", "-D", "--defined-only", str(library_path)], capture_output=True, text=True, check=True)
    exported = set(re.findall(r"\bT (lsso_\w+)", out.stdout))
    assert set(declared_functions()) <= exported
    # Nothing but the C ABI is visible.
    assert exported == set(declared_functions())


def test_library_has_no_torch_dependency(library_path: Path) -> None:
    out = subprocess.run(["ldd", str(library_path)], capture_output=True, text=True)
    assert "torch" not in out.stdout and "c10" not in out.stdout


def test_contract_and_sizes_without_a_gpu(library_path: Path) -> None:
    lib = ctypes.CDLL(str(library_path))
    lib.lsso_last_error.restype = ctypes.c_char_p
    lib.lsso_tape_stride.restype = ctypes.c_int64
    lib.lsso_tape_stride.argtypes = [ctypes.c_int64] * 4
    lib.lsso_forward_workspace_size.restype = ctypes.c_size_t
    lib.lsso_forward_workspace_size.argtypes = [ctypes.c_int64] * 5 + [ctypes.c_int, ctypes.c_int]
    assert lib.lsso_contract_version() == 8
    assert lib.lsso_compiled_sm() == 100
    # N*R + 3R^2 + 2Rd + 1 with N=33, H=1, D=17, R=32 (reference tape-size test)
    assert lib.lsso_tape_stride(33, 1, 17, 32) == 33 * 32 + 3 * 32 * 32 + 2 * 32 * 17 + 1
    assert lib.lsso_forward_workspace_size(1, 8, 1, 16, 24, 0, 0) == 0
    assert b"rank in {16, 32, 48, 64}" in lib.lsso_last_error()
    assert lib.lsso_forward_workspace_size(1, 8, 3, 16, 16, 0, 0) == 0
    assert b"divisible by H" in lib.lsso_last_error()
    assert lib.lsso_forward_workspace_size(0, 8, 1, 16, 16, 0, 0) == 0
    assert b"must be positive" in lib.lsso_last_error()


def test_operator_registration_exposes_the_reference_schemas(library_path: Path) -> None:
    # Registration is process-wide, so it runs in a child interpreter.
    code = (
        "import torch\n"
        "from lsso_b200.ball import _native, cuda\n"
        f"_native.register({str(library_path)!r})\n"
        "assert cuda.is_available()\n"
        "assert torch.ops.lsso_equilibrium.contract_version() == 8\n"
        "print(torch.ops.lsso_equilibrium.forward_train.default._schema)\n"
        "print(torch.ops.lsso_equilibrium.backward.default._schema)\n"
    )
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, cwd=ROOT, timeout=300)
    assert out.returncode == 0, out.stderr
    assert "Tensor? centered_positions=None, Tensor? valid_counts=None) -> (Tensor, Tensor, Tensor)" in out.stdout
    assert "Tensor tape, Tensor pivots" in out.stdout


def test_every_exported_symbol_has_a_ctypes_signature(library_path: Path) -> None:
    """Without argtypes, ctypes would pass 64-bit device pointers as C int."""
    from lsso_b200.ball import _native

    lib = _native.open_library(library_path).lib
    for name in _native.EXPORTED_SYMBOLS:
        fn = getattr(lib, name)
        assert fn.argtypes is not None, name
        assert fn.restype is not None or name.endswith("_start"), name
