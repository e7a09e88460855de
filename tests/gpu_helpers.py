"""Helpers for the GPU parity tests: CUDA path vs the CPU oracle.

Bar (from the operator's specification): latest-k values, masks and gathered
payloads bit-exact; segmented sums and gradients within a relative tolerance
of the float64 oracle -- 1e-5 for float32, 1e-2 for bfloat16 (float32
accumulation), 5e-3 for float16, 1e-10 for float64 -- applied as
|actual - expected| <= tol * (|expected| + max|expected|).
"""
from __future__ import annotations

import numpy as np
import torch

SUM_TOL = {torch.float32: 1e-5, torch.bfloat16: 1e-2, torch.float16: 5e-3, torch.float64: 1e-10}
CODE = {torch.float32: None, torch.bfloat16: "bf16", torch.float16: "f16", torch.float64: None}


def to_np_bits(t: torch.Tensor) -> np.ndarray:
    """Raw element bits of a tensor as an unsigned numpy array."""
    t = t.detach().contiguous().cpu()
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.view(torch.int16).numpy().view(np.uint16)
    if t.dtype == torch.float32:
        return t.numpy().view(np.uint32)
    if t.dtype == torch.float64:
        return t.numpy().view(np.uint64)
    return t.numpy()


def payload_np(p: torch.Tensor) -> np.ndarray:
    """Payload in the form the oracle takes (bits for 16-bit floats)."""
    p = p.detach().contiguous().cpu()
    if p.dtype == torch.bfloat16:
        return p.view(torch.int16).numpy().view(np.uint16)
    if p.dtype == torch.float16:
        return p.numpy()
    return p.numpy()


def to_f64(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().double().numpy()


def assert_close(actual: np.ndarray, expected: np.ndarray, tol: float, what: str = "") -> None:
    scale = float(np.max(np.abs(expected))) if expected.size else 0.0
    err = np.abs(actual - expected)
    bound = tol * (np.abs(expected) + max(scale, 1e-30))
    bad = err > bound
    if bad.any():
        i = np.unravel_index(np.argmax(err - bound), err.shape)
        raise AssertionError(f"{what}: {int(bad.sum())} of {err.size} elements beyond tol {tol}; worst at {i}: "
                             f"actual {actual[i]!r} expected {expected[i]!r} (max|expected| {scale:.3g})")


def assert_bits_equal(actual: torch.Tensor, expected_bits: np.ndarray, what: str = "") -> None:
    """Bitwise equality; a float ``expected_bits`` array is compared through its raw bits."""
    if expected_bits.dtype.kind == "f":
        expected_bits = expected_bits.view({2: np.uint16, 4: np.uint32, 8: np.uint64}[expected_bits.itemsize])
    a = to_np_bits(actual)
    if a.shape != expected_bits.shape:
        raise AssertionError(f"{what}: shape {a.shape} != {expected_bits.shape}")
    if not np.array_equal(a, expected_bits):
        diff = a != expected_bits
        n = int(diff.sum())
        idx = np.argwhere(diff)
        width = a.dtype.itemsize * 8
        sign = np.uint64(1) << np.uint64(width - 1)
        only_sign = int(((a.astype(np.uint64) ^ expected_bits.astype(np.uint64)) == sign)[diff].sum())
        first = ", ".join(f"{tuple(int(x) for x in i)}: {int(a[tuple(i)]):#x} vs {int(expected_bits[tuple(i)]):#x}"
                          for i in idx[:6])
        raise AssertionError(f"{what}: {n} of {a.size} elements differ bitwise ({only_sign} only in the sign "
                             f"bit); first: {first}")
