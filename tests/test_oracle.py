"""Pin the NumPy oracle against the reference's golden fixtures (CPU only).

The fixtures in ``tests/golden`` hold outputs and autograd gradients of the
reference's own PyTorch implementation; the oracle must reproduce them before
any CUDA result is compared with it.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import lsso_oracle as O
from tests.golden_io import GOLDEN, load_mixer_case, load_module_case, mixer_case_names, module_case_names


@pytest.mark.parametrize("name", mixer_case_names())
def test_oracle_mixer_matches_reference_fp64(name: str) -> None:
    case = load_mixer_case(name)
    out, state = O.mixer_forward(case["projected"], case["core_base_raw"], case["core_drive_weight"],
                                 case["eta_raw"], case["centered_positions"], case["valid_counts"],
                                 return_state=True)
    assert O.relative_l2(out, case["out"]) < 1e-12
    grads = O.mixer_backward(case["upstream"], state)
    for got, key in zip(grads, ("grad_projected", "grad_core_base_raw", "grad_core_drive_weight", "grad_eta_raw")):
        assert O.relative_l2(got, case[key]) < 1e-10, key


@pytest.mark.parametrize("name", module_case_names())
def test_oracle_module_matches_reference(name: str) -> None:
    case = load_module_case(name)
    dtype = np.float32 if name.startswith("fp32path") else np.float64
    y, state = O.module_forward(case["params"], case["x"], case["valid_mask"], case["position_ids"],
                                heads=case["heads"], rank=case["rank"], dtype=dtype, return_state=True)
    if dtype == np.float64:
        assert O.relative_l2(y, case["y"]) < 1e-12
        grads = O.module_backward(case["upstream"], state)
        assert O.relative_l2(grads["x"], np.nan_to_num(case["grad_x"])) < 1e-10
        for key, expected in case["grads"].items():
            assert O.relative_l2(grads[key], expected) < 1e-10, key
    else:
        # The reference FP32 CPU path rounds the packed projection and the mixer
        # output to BF16; the restatement rounds at the same points, so only
        # FP32 summation order and rare BF16 tie flips separate them.
        assert O.relative_l2(y, case["y"]) < 2e-3


def test_oracle_config1_forward_matches_reference() -> None:
    data = np.load(GOLDEN / "config1_forward.npz")
    params = dict(w_bc=data["param_w_bc_weight"], b_bc=None, w_o=data["param_w_o_weight"], b_o=None,
                  core_base_raw=data["param_core_base_raw"], core_drive_weight=data["param_core_drive_weight"],
                  eta_raw=data["param_eta_raw"])
    y = O.module_forward(params, data["x"], None, np.arange(65), heads=3, rank=16, dtype=np.float32)
    assert y.shape == (8, 65, 192)
    assert O.relative_l2(y, data["y"]) < 2e-3
    # Published oracle check of this configuration (norm and max of y).
    assert abs(np.linalg.norm(data["y"]) - 88.4024) < 1e-3
    assert abs(np.abs(data["y"]).max() - 1.4346) < 1e-3


def test_round_bf16_is_round_to_nearest_even() -> None:
    values = np.array([1.0, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, -2.5, 3.0e38, 1e-40], dtype=np.float32)
    rounded = O.round_bf16(values)
    assert rounded[0] == 1.0
    assert rounded[1] == 1.0  # tie rounds to even mantissa
    assert rounded[2] == 1.0 + 2 ** -6
    assert rounded[3] == -2.5
    assert np.isfinite(rounded[4]) or rounded[4] == np.inf
    bits = rounded.view(np.uint32)
    assert np.all(bits & 0xFFFF == 0)


def test_cholesky_frame_identity_equals_qr_frame() -> None:
    rng = np.random.default_rng(0)
    A = rng.standard_normal((3, 41, 16)) * 3.0
    P = O.qr_soft_frame(A)
    L = np.linalg.cholesky(np.swapaxes(A, -1, -2) @ A + np.eye(16))
    P2 = np.swapaxes(np.linalg.solve(L, np.swapaxes(A, -1, -2)), -1, -2)
    assert O.relative_l2(P2, P) < 1e-12


def test_backward_matches_finite_differences() -> None:
    rng = np.random.default_rng(3)
    heads, rank, head_dim, length = 1, 16, 4, 9
    projected = rng.standard_normal((1, length, heads * (rank + head_dim)))
    base = 0.1 * rng.standard_normal((heads, rank, rank))
    drive = 0.1 * rng.standard_normal((heads, head_dim, rank))
    eta = np.array([0.3])
    upstream = rng.standard_normal((1, length, heads * head_dim))
    _, state = O.mixer_forward(projected, base, drive, eta, return_state=True)
    grads = O.mixer_backward(upstream, state)

    def loss(p, b, dr, e):
        return float((O.mixer_forward(p, b, dr, e) * upstream).sum())

    args = [projected, base, drive, eta]
    for index in range(4):
        flat = args[index].reshape(-1)
        for position in rng.choice(flat.size, size=min(5, flat.size), replace=False):
            step = 1e-6
            plus = [a.copy() for a in args]
            minus = [a.copy() for a in args]
            plus[index].reshape(-1)[position] += step
            minus[index].reshape(-1)[position] -= step
            numeric = (loss(*plus) - loss(*minus)) / (2 * step)
            assert abs(numeric - grads[index].reshape(-1)[position]) < 1e-6 * max(1.0, abs(numeric))


def test_contract_mode_rounds_only_at_the_contract_boundaries() -> None:
    """``contract=True`` is the FP64 operator with the CUDA contract's roundings.
    With FP16-exact phases (every position 0) its forward stays within BF16
    rounding of the exact operator, its BF16 boundaries hold BF16 values, and
    its mixer backward is the exact VJP of the BF16-rounded gradient."""
    rng = np.random.default_rng(12)
    params = O.init_params(32, 2, 16, bias=True, seed=4, core_scale=0.05)
    x = rng.standard_normal((2, 17, 32))
    zeros = np.zeros((2, 17), np.int64)
    y_c, st_c = O.module_forward(params, x, None, zeros, heads=2, rank=16, return_state=True, contract=True)
    y_e, st_e = O.module_forward(params, x, None, zeros, heads=2, rank=16, return_state=True)
    assert 1e-5 < O.relative_l2(y_c, y_e) < 1e-2
    # the BF16 boundaries: packed projection and mixer output are BF16 values
    for value in (st_c["mixed"], st_c["x"]):
        assert np.array_equal(O.round_bf16(value), value.astype(np.float32))
    upstream = rng.standard_normal(y_c.shape)
    g_c = O.module_backward(upstream, st_c)
    g_e = O.module_backward(upstream, st_e)
    for key in ("x", "w_bc", "w_o", "core_base_raw", "core_drive_weight"):
        assert O.relative_l2(g_c[key], g_e[key]) < 2e-2, key
    # the mixer part of the contract backward is the exact VJP of the rounded gradient
    go = O.round_bf16(upstream.reshape(-1, 32)).astype(np.float64)
    grad_mixed = O.round_bf16(go @ st_c["w_o"]).astype(np.float64).reshape(2, 17, 32)
    _, base, _, _ = O.mixer_backward(grad_mixed, st_c["mixer"])
    assert np.array_equal(base, g_c["core_base_raw"])
