"""CPU tests of the tensor-core prefill's numerics (tests/chunk_model.py mirrors the kernel):
the algorithm is exact without operand rounding, and with the kernel's bf16 operand rounding it
stays inside the north-star bf16 bound (2e-2) with margin, up to the BASELINE length T = 4096."""
import numpy as np
import pytest

from chunk_model import blocked_unit_lower_inverse, prefill_model
from fixtures import TOL_BF16, baseline_inputs, bf16_round, rel_err
from oracle import oracle as O


def test_blocked_inverse():
    rng = np.random.default_rng(0)
    A = np.tril(rng.standard_normal((64, 64)) * 0.3, -1)
    T = blocked_unit_lower_inverse(A)
    np.testing.assert_allclose(T @ (np.eye(64) + A), np.eye(64), atol=1e-12)


@pytest.mark.parametrize("masks", [False, True])
def test_chunk_algorithm_exact_without_rounding(masks):
    B, T, H, D = 1, 200, 2, 128
    q, k, v, al, be = baseline_inputs(1, B, T, H, D, D)
    rng = np.random.default_rng(5)
    valid = rng.random((B, T)) > 0.1 if masks else None
    reset = rng.random((B, T)) > 0.97 if masks else None
    init = (0.02 * rng.standard_normal((B, H, D, D))).astype(np.float32) if masks else None
    ro, rf, _ = O.scan_scalar(q, k, v, al, be, valid, reset, init)
    mo, mf = prefill_model(q, k, v, al, be, 1 / np.sqrt(D), valid, reset, init, rounding=False)
    assert rel_err(mo, ro) < 2e-5 and rel_err(mf, rf) < 2e-5


def test_kernel_rounding_budget_at_baseline_length():
    B, T, H, D = 1, 4096, 1, 128
    q, k, v, al, be = baseline_inputs(2, B, T, H, D, D)
    q, k, v = bf16_round(q), bf16_round(k), bf16_round(v)
    ro, rf, _ = O.scan_scalar(q, k, v, al, be)
    mo, mf = prefill_model(q, k, v, al, be, 1 / np.sqrt(D))
    assert rel_err(mo, ro) < 0.6 * TOL_BF16
    assert rel_err(mf, rf) < 0.6 * TOL_BF16
