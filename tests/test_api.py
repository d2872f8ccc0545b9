"""Public API, checkpoint contract and loader boundary on CPU.

Mirrors the CPU-side contract tests of the reference (tests/core/test_model.py
and the fake-backend half of tests/cuda/test_fast_path.py): the CUDA boundary
is explicit, dispatch picks the train/inference entry points, the loader binds
one architecture under a lock and rejects stale or misnamed libraries.
"""

from __future__ import annotations

from pathlib import Path
from threading import Event, Thread
from types import SimpleNamespace

import numpy as np
import pytest
import torch

import lsso
from lsso import CoreMode, LSSO, LSSOConfig
from lsso.ball import cuda
from oracle import lsso_oracle as O
from tests.golden_io import load_module_case, module_case_names


# ------------------------------------------------------------------ configuration
def test_public_api_names() -> None:
    assert lsso.__version__ == "0.6.3"
    assert set(lsso.__all__) == {"CoreMode", "LSSO", "LSSOConfig", "__version__"}
    assert lsso.LSSO is LSSO


@pytest.mark.parametrize(("kwargs", "error"), [
    (dict(dim=32, num_heads=3), ValueError),
    (dict(dim=32, num_heads=2, rank=15), ValueError),
    (dict(dim=32, num_heads=2, rank=0), ValueError),
    (dict(dim=32.0, num_heads=2), TypeError),
    (dict(dim=True, num_heads=2), TypeError),
    (dict(dim=32, num_heads=2, bias=1), TypeError),
    (dict(dim=32, num_heads=2, rank_rotary="yes"), TypeError),
    (dict(dim=32, num_heads=2, core_mode="bogus"), ValueError),
])
def test_configuration_validation(kwargs, error) -> None:
    with pytest.raises(error):
        LSSOConfig(**kwargs)


def test_core_mode_accepts_strings_and_exposes_head_dim() -> None:
    config = LSSOConfig(dim=48, num_heads=3, rank=16, core_mode="static")
    assert config.core_mode is CoreMode.STATIC
    assert config.head_dim == 16
    layer = LSSO(config)
    assert layer.core_drive_weight is None and layer.core_base_raw is not None


# ------------------------------------------------------------------ checkpoint contract 12
def test_checkpoint_contract_round_trips_and_rejects_mismatch() -> None:
    layer = LSSO(LSSOConfig(32, 2, 16))
    state = layer.state_dict()
    assert state["_extra_state"]["version"] == 12
    assert state["_extra_state"]["numerics"] == "tf32-wbc-ieee-fgram-tc16-v6"
    LSSO(LSSOConfig(32, 2, 16)).load_state_dict(state)
    with pytest.raises(RuntimeError, match="incompatible LSSO checkpoint contract"):
        LSSO(LSSOConfig(32, 2, 32)).load_state_dict(state, strict=False)
    missing = {k: v for k, v in state.items() if k != "_extra_state"}
    with pytest.raises(RuntimeError, match="missing its configuration contract"):
        LSSO(LSSOConfig(32, 2, 16)).load_state_dict(missing, strict=False)


def test_checkpoint_contract_holds_inside_a_parent_module() -> None:
    parent = torch.nn.Sequential(LSSO(LSSOConfig(32, 2, 16)))
    state = parent.state_dict()
    state["0._extra_state"] = dict(state["0._extra_state"], bias=True)
    with pytest.raises(RuntimeError, match="bias"):
        torch.nn.Sequential(LSSO(LSSOConfig(32, 2, 16))).load_state_dict(state)


CHECKPOINTS = sorted(p.name for p in (Path(__file__).resolve().parent / "golden").glob("checkpoint_*.pt"))


def _reference_checkpoint(name: str) -> dict:
    return torch.load(Path(__file__).resolve().parent / "golden" / name, weights_only=True)


def test_reference_checkpoint_fixtures_exist() -> None:
    assert len(CHECKPOINTS) == 2


@pytest.mark.parametrize("name", CHECKPOINTS)
def test_reference_written_checkpoint_loads_strictly_and_reproduces_its_output(name: str) -> None:
    """A state_dict written by the reference's own module (tests/golden/make_golden.py,
    reference model.py:79-140) loads strictly here and gives the reference's y."""
    record = _reference_checkpoint(name)
    layer = LSSO(LSSOConfig(**record["config"]))
    result = layer.load_state_dict(record["state_dict"], strict=True)
    assert not result.missing_keys and not result.unexpected_keys
    for key, value in layer.state_dict().items():
        if key != "_extra_state":
            assert torch.equal(value, record["state_dict"][key]), key
    with torch.no_grad():
        y = layer(record["x"])
    assert y.dtype == record["y"].dtype and y.shape == record["y"].shape
    assert torch.equal(y, record["y"])


@pytest.mark.parametrize("name", CHECKPOINTS)
def test_state_dict_matches_the_reference_key_by_key(name: str) -> None:
    """This module's state_dict has the reference's keys in the reference's order,
    with the same shapes and dtypes and an equal configuration contract, so
    checkpoints written here load into the reference and vice versa."""
    record = _reference_checkpoint(name)
    ours = LSSO(LSSOConfig(**record["config"])).state_dict()
    theirs = record["state_dict"]
    assert list(ours) == list(theirs)
    for key in theirs:
        if key == "_extra_state":
            assert ours[key] == theirs[key]
            assert [type(v) for v in ours[key].values()] == [type(v) for v in theirs[key].values()]
        else:
            assert (ours[key].shape, ours[key].dtype) == (theirs[key].shape, theirs[key].dtype), key


@pytest.mark.parametrize("name", CHECKPOINTS)
def test_reference_checkpoint_is_rejected_by_a_different_configuration(name: str) -> None:
    record = _reference_checkpoint(name)
    config = dict(record["config"])
    config["rank"] = 48 if config["rank"] != 48 else 16
    with pytest.raises(RuntimeError, match="incompatible LSSO checkpoint contract"):
        LSSO(LSSOConfig(**config)).load_state_dict(record["state_dict"], strict=False)


# ------------------------------------------------------------------ reference path vs golden fixtures
@pytest.mark.parametrize("name", [n for n in module_case_names() if n.startswith("fp64")])
def test_reference_path_matches_golden_fp64(name: str) -> None:
    case = load_module_case(name)
    config = LSSOConfig(dim=case["dim"], num_heads=case["heads"], rank=case["rank"], bias=case["bias"])
    layer = LSSO(config).double()
    names = {"w_bc": "w_bc.weight", "b_bc": "w_bc.bias", "w_o": "w_o.weight", "b_o": "w_o.bias",
             "core_base_raw": "core_base_raw", "core_drive_weight": "core_drive_weight", "eta_raw": "eta_raw"}
    params = dict(layer.named_parameters())
    with torch.no_grad():
        for key, value in case["params"].items():
            if value is not None:
                params[names[key]].copy_(torch.from_numpy(value))
    x = torch.from_numpy(case["x"]).double().requires_grad_()
    mask = None if case["valid_mask"] is None else torch.from_numpy(case["valid_mask"])
    pos = None if case["position_ids"] is None else torch.from_numpy(case["position_ids"])
    y = layer(x, valid_mask=mask, position_ids=pos)
    assert O.relative_l2(y.detach().numpy(), case["y"]) < 1e-12
    grads = torch.autograd.grad((y * torch.from_numpy(case["upstream"]).double()).sum(), [x, *params.values()])
    assert O.relative_l2(np.nan_to_num(grads[0].numpy()), np.nan_to_num(case["grad_x"])) < 1e-10


def test_masked_nan_padding_matches_cropped_sequence() -> None:
    torch.manual_seed(3)
    layer = LSSO(LSSOConfig(32, 2, 16)).double()
    x = torch.randn(1, 9, 32, dtype=torch.float64)
    mask = torch.zeros(1, 9, dtype=torch.bool)
    mask[0, 2:7] = True
    padded = torch.where(mask[:, :, None], x, torch.full_like(x, float("nan")))
    full = layer(padded, valid_mask=mask)
    cropped = layer(x[:, 2:7])
    torch.testing.assert_close(full[:, 2:7], cropped)
    assert torch.count_nonzero(full[~mask]) == 0


def test_integer_positions_are_shift_invariant() -> None:
    torch.manual_seed(4)
    layer = LSSO(LSSOConfig(32, 2, 16)).double()
    x = torch.randn(2, 7, 32, dtype=torch.float64)
    a = layer(x, position_ids=torch.arange(7))
    b = layer(x, position_ids=torch.arange(7) + 10 ** 9)
    torch.testing.assert_close(a, b)


# ------------------------------------------------------------------ CUDA dispatch contract (CPU side)
def test_cuda_boundary_is_explicit() -> None:
    if cuda.is_available():
        cuda.require_available()
    else:
        with pytest.raises(RuntimeError, match="extension is not loaded"):
            cuda.require_available()


def test_fast_mix_rejects_position_gradients_before_loading() -> None:
    positions = torch.arange(4, dtype=torch.float32, requires_grad=True)
    with pytest.raises(ValueError, match="does not support gradients"):
        cuda.fast_mix(torch.empty(0), torch.empty(0), torch.empty(0), torch.empty(0), positions)


def test_fast_mix_selects_train_and_inference_entry_points(monkeypatch: pytest.MonkeyPatch) -> None:
    calls: list[str] = []

    def inference(*args):
        calls.append("forward_inference")
        assert args[0].dtype == torch.bfloat16
        return args[0].detach().clone()

    def train(*args):
        calls.append("forward_train")
        return args[0].clone(), torch.empty(1, dtype=torch.float32), torch.empty(1, dtype=torch.int32)

    def backward(*args):
        calls.append("backward")
        assert len(args) == 9 and args[0].dtype == torch.bfloat16
        torch.testing.assert_close(args[7], torch.tensor([0.0, 1.0]))
        torch.testing.assert_close(args[8], torch.tensor([2.0]))
        return tuple(torch.ones_like(a) for a in args[1:5])

    namespace = SimpleNamespace(contract_version=lambda: 8, forward_inference=inference, forward_train=train,
                                backward=backward)
    monkeypatch.setattr(cuda, "torch", SimpleNamespace(ops=SimpleNamespace(lsso_equilibrium=namespace),
                                                       is_grad_enabled=torch.is_grad_enabled))
    monkeypatch.setattr(cuda, "require_available", lambda: None)
    projected = torch.randn(1, 2, 3, dtype=torch.bfloat16, requires_grad=True)
    base = torch.randn(1, 16, 16, requires_grad=True)
    drive = torch.randn(1, 16, 16, requires_grad=True)
    eta = torch.randn(1, requires_grad=True)
    positions, counts = torch.tensor([0.0, 1.0]), torch.tensor([2.0])
    cuda.fast_mix(projected, base, drive, eta, positions, counts).sum().backward()
    assert calls == ["forward_train", "backward"]
    calls.clear()
    with torch.inference_mode():
        out = cuda.fast_mix(projected, base, drive, eta, positions, counts)
    assert not out.requires_grad and calls == ["forward_inference"]


def test_probe_rejects_incomplete_or_stale_abi(monkeypatch: pytest.MonkeyPatch) -> None:
    partial = SimpleNamespace(forward_train=object(), backward=object())
    monkeypatch.setattr(cuda, "torch", SimpleNamespace(ops=SimpleNamespace(lsso_equilibrium=partial)))
    assert not cuda.is_available()
    stale = SimpleNamespace(contract_version=lambda: 7, forward_inference=object(), forward_train=object(),
                            backward=object())
    monkeypatch.setattr(cuda, "torch", SimpleNamespace(ops=SimpleNamespace(lsso_equilibrium=stale)))
    monkeypatch.setattr(cuda, "_LOADED_ARCHITECTURE", None)
    assert not cuda.is_available()
    with pytest.raises(RuntimeError, match="native contract version"):
        cuda.require_available()


def test_loader_rejects_misnamed_missing_and_foreign_architecture(tmp_path: Path,
                                                                  monkeypatch: pytest.MonkeyPatch) -> None:
    monkeypatch.setattr(cuda, "_device_architecture", lambda device=None: 100)
    monkeypatch.setattr(cuda, "is_available", lambda: False)
    monkeypatch.setattr(cuda, "_LOADED_ARCHITECTURE", None)
    wrong = tmp_path / "lsso_equilibrium.so"
    wrong.touch()
    with pytest.raises(RuntimeError, match="requires lsso_equilibrium_sm100.so"):
        cuda.load(path=wrong)
    with pytest.raises(RuntimeError, match="was not found"):
        cuda.load(path=tmp_path / "lsso_equilibrium_sm100.so")
    monkeypatch.setattr(cuda, "is_available", lambda: True)
    monkeypatch.setattr(cuda, "_LOADED_ARCHITECTURE", 90)
    with pytest.raises(RuntimeError, match="targets SM90, not requested SM100"):
        cuda.load()


def test_loader_rejects_a_stale_library_contract(tmp_path: Path, monkeypatch: pytest.MonkeyPatch) -> None:
    library = tmp_path / "lsso_equilibrium_sm100.so"
    library.touch()
    namespace = SimpleNamespace()

    def register(path):
        assert path == library.resolve()
        namespace.contract_version = lambda: 7
        namespace.forward_inference = namespace.forward_train = namespace.backward = object()

    monkeypatch.setattr(cuda, "_device_architecture", lambda device=None: 100)
    monkeypatch.setattr(cuda, "_LOADED_ARCHITECTURE", None)
    monkeypatch.setattr(cuda, "_register_library", register)
    monkeypatch.setattr(cuda, "torch", SimpleNamespace(ops=SimpleNamespace(lsso_equilibrium=namespace)))
    with pytest.raises(RuntimeError, match="native contract version"):
        cuda.load(path=library)


def test_loader_serializes_a_mixed_architecture_race(monkeypatch: pytest.MonkeyPatch) -> None:
    monkeypatch.setattr(cuda, "_device_architecture", lambda device=None: 100)
    monkeypatch.setattr(cuda, "_LOADED_ARCHITECTURE", None)
    monkeypatch.setattr(cuda, "is_available", lambda: True)
    started, finished = Event(), Event()
    errors: list[RuntimeError] = []

    def second() -> None:
        started.set()
        try:
            cuda.load(device=0)
        except RuntimeError as error:
            errors.append(error)
        finally:
            finished.set()

    with cuda._LOAD_LOCK:
        thread = Thread(target=second)
        thread.start()
        assert started.wait(timeout=1.0)
        assert not finished.wait(timeout=0.1)
        monkeypatch.setattr(cuda, "_LOADED_ARCHITECTURE", 90)
    thread.join(timeout=1.0)
    assert finished.is_set() and len(errors) == 1
    assert "targets SM90, not requested SM100" in str(errors[0])


def test_architecture_check_accepts_only_sm100(monkeypatch: pytest.MonkeyPatch) -> None:
    monkeypatch.setattr(cuda.torch.cuda, "is_available", lambda: True)
    monkeypatch.setattr(cuda.torch.cuda, "current_device", lambda: 0)
    monkeypatch.setattr(cuda.torch.cuda, "get_device_capability", lambda device: (10, 0))
    assert cuda._device_architecture() == 100
    monkeypatch.setattr(cuda.torch.cuda, "get_device_capability", lambda device: (9, 0))
    with pytest.raises(RuntimeError, match="supports SM100"):
        cuda._device_architecture()


def test_default_library_path_honours_override(monkeypatch: pytest.MonkeyPatch, tmp_path: Path) -> None:
    monkeypatch.setenv("LSSO_CUDA_LIBRARY", str(tmp_path / "x.so"))
    assert cuda._default_library_path() == tmp_path / "x.so"
    monkeypatch.delenv("LSSO_CUDA_LIBRARY")
    monkeypatch.setattr(cuda, "_device_architecture", lambda device=None: 100)
    assert cuda._default_library_path().name == "lsso_equilibrium_sm100.so"


@pytest.mark.parametrize("config", [
    LSSOConfig(32, 2, rank=16, core_mode=CoreMode.STATIC),
    LSSOConfig(32, 2, rank=16, rank_rotary=False),
    LSSOConfig(32, 2, rank=24),
])
def test_cuda_dispatch_rejects_unsupported_contracts(config: LSSOConfig) -> None:
    with pytest.raises(ValueError, match="implementation='cuda'"):
        LSSO(config)(torch.randn(1, 4, config.dim), implementation="cuda")


@pytest.mark.parametrize(("rank", "head_dim"), [(16, 1), (32, 17), (48, 256), (64, 384)])
def test_cuda_dispatch_accepts_supported_ranks_and_any_head_dim(rank: int, head_dim: int) -> None:
    layer = LSSO(LSSOConfig(dim=2 * head_dim, num_heads=2, rank=rank))
    with pytest.raises(ValueError, match="CUDA tensor"):
        layer(torch.randn(1, 4, 2 * head_dim).half(), implementation="cuda")


def test_reference_is_default_and_implementation_is_validated(monkeypatch: pytest.MonkeyPatch) -> None:
    layer = LSSO(LSSOConfig(32, 2, 16)).eval()
    monkeypatch.setattr(cuda, "fast_mix", lambda *a, **k: pytest.fail("reference dispatch called CUDA"))
    x = torch.randn(2, 5, 32).half()
    assert layer(x).shape == x.shape
    with pytest.raises(ValueError, match="'reference' or 'cuda'"):
        layer(x, implementation="automatic")


def test_input_validation_messages() -> None:
    layer = LSSO(LSSOConfig(32, 2, 16))
    with pytest.raises(ValueError, match="batch size must be positive"):
        layer(torch.randn(0, 4, 32))
    with pytest.raises(ValueError, match="sequence length must be positive"):
        layer(torch.randn(1, 0, 32))
    with pytest.raises(TypeError, match="valid_mask must have dtype torch.bool"):
        layer(torch.randn(1, 4, 32), valid_mask=torch.ones(1, 4))
    with pytest.raises(TypeError, match="floating position_ids"):
        layer(torch.randn(1, 4, 32), position_ids=torch.arange(4).half())
