"""Shared helpers for the GPU parity tests: device transfer, bf16 rounding and the
reference's comparison rules (tests/test_utils.hpp:70-190 of Cu-Vit)."""

from __future__ import annotations

import numpy as np


def to_device(array, dtype=None):
    import torch

    tensor = torch.from_numpy(np.ascontiguousarray(array, dtype=np.float32))
    if dtype is not None:
        tensor = tensor.to(dtype)
    return tensor.cuda()


def to_host(tensor) -> np.ndarray:
    import torch

    return tensor.detach().to(torch.float32).cpu().numpy()


def bf16_round(array) -> np.ndarray:
    """Round-to-nearest-even to bfloat16, returned as float32 values."""
    import torch

    tensor = torch.from_numpy(np.ascontiguousarray(array, dtype=np.float32))
    return tensor.to(torch.bfloat16).to(torch.float32).numpy()


def assert_close(actual, expected, rtol, atol, context=""):
    """NumPy-style mixed tolerance: |a - e| <= atol + rtol * |e| (compare_close)."""
    actual = np.asarray(actual, np.float64).reshape(-1)
    expected = np.asarray(expected, np.float64).reshape(-1)
    assert actual.shape == expected.shape, context
    assert np.isfinite(actual).all(), f"{context}: non-finite output"
    diff = np.abs(actual - expected)
    bound = atol + rtol * np.abs(expected)
    bad = np.flatnonzero(diff > bound)
    if bad.size:
        i = bad[0]
        raise AssertionError(f"{context}: {bad.size} mismatches; first at {i}: actual "
                             f"{actual[i]!r} expected {expected[i]!r} (|diff| {diff[i]:.3g})")


def assert_close_scaled(actual, expected, scale, rtol, atol, context=""):
    """Reduction tolerance against the summed term magnitudes (compare_close_scaled)."""
    actual = np.asarray(actual, np.float64).reshape(-1)
    expected = np.asarray(expected, np.float64).reshape(-1)
    scale = np.abs(np.asarray(scale, np.float64).reshape(-1))
    assert np.isfinite(actual).all(), f"{context}: non-finite output"
    diff = np.abs(actual - expected)
    bad = np.flatnonzero(diff > atol + rtol * scale)
    if bad.size:
        i = bad[0]
        raise AssertionError(f"{context}: {bad.size} mismatches; first at {i}: actual "
                             f"{actual[i]!r} expected {expected[i]!r} scale {scale[i]!r} "
                             f"(worst term-relative {np.max(diff / np.maximum(scale, 1e-30)):.3g})")


def worst_scaled(actual, expected, scale) -> float:
    actual = np.asarray(actual, np.float64).reshape(-1)
    expected = np.asarray(expected, np.float64).reshape(-1)
    scale = np.abs(np.asarray(scale, np.float64).reshape(-1))
    return float(np.max(np.abs(actual - expected) / np.maximum(scale, 1e-30)))
