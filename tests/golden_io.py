"""Loading helpers for the golden fixtures in ``tests/golden``."""

from __future__ import annotations

from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"

_MIXER_KEYS = ("projected", "core_base_raw", "core_drive_weight", "eta_raw", "upstream", "out",
               "grad_projected", "grad_core_base_raw", "grad_core_drive_weight", "grad_eta_raw")

_PARAM_NAMES = {
    "w_bc_weight": "w_bc", "w_bc_bias": "b_bc", "w_o_weight": "w_o", "w_o_bias": "b_o",
    "core_base_raw": "core_base_raw", "core_drive_weight": "core_drive_weight", "eta_raw": "eta_raw",
}


def mixer_case_names() -> list[str]:
    return sorted(p.stem[len("mixer_"):] for p in GOLDEN.glob("mixer_*.npz"))


def module_case_names() -> list[str]:
    return sorted(p.stem[len("module_"):] for p in GOLDEN.glob("module_*.npz"))


def _optional(array: np.ndarray):
    return None if array.size == 0 else array


def load_mixer_case(name: str) -> dict:
    data = np.load(GOLDEN / f"mixer_{name}.npz")
    case = {key: data[key] for key in _MIXER_KEYS}
    case["centered_positions"] = _optional(data["centered_positions"])
    case["valid_counts"] = _optional(data["valid_counts"])
    case["valid_mask"] = _optional(data["valid_mask"])
    case["heads"] = int(data["heads"])
    case["rank"] = int(data["rank"])
    return case


def load_module_case(name: str) -> dict:
    data = np.load(GOLDEN / f"module_{name}.npz")
    params = {"b_bc": None, "b_o": None}
    grads = {}
    for key in data.files:
        if key.startswith("param_"):
            params[_PARAM_NAMES[key[len("param_"):]]] = data[key]
        elif key.startswith("grad_") and key != "grad_x":
            grads[_PARAM_NAMES[key[len("grad_"):]]] = data[key]
    return dict(
        x=data["x"], y=data["y"], upstream=data["upstream"], grad_x=data["grad_x"],
        heads=int(data["heads"]), rank=int(data["rank"]), dim=int(data["dim"]), bias=bool(data["bias"]),
        valid_mask=_optional(data["valid_mask"]), position_ids=_optional(data["position_ids"]),
        params=params, grads=grads,
    )
