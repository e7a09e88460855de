"""The CPU oracle against golden vectors produced by the reference itself.

Pins ``oracle/`` to ``ravel_lm/ravel_memory.py`` of the reference: the
fixtures in ``tests/golden`` hold the reference's own outputs
(``tests/golden/make_golden.py``).  Latest-k values and all masks must match
bit for bit (including the sign of zero in invalid slots); sums and gradients
(reference run on float64 payloads) to 1e-10 relative.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import golden_cases, load_golden, payload_as_float64, payload_code


def _bits(a: np.ndarray) -> np.ndarray:
    return a.view({2: np.uint16, 4: np.uint32, 8: np.uint64}[a.dtype.itemsize])


def _close(actual, expected, rel=1e-10):
    scale = max(1.0, float(np.max(np.abs(expected))) if expected.size else 1.0)
    np.testing.assert_allclose(actual, expected, rtol=rel, atol=rel * scale)


@pytest.mark.parametrize("name", golden_cases())
def test_oracle_matches_reference_golden(oracle_mod, name):
    case = load_golden(name)
    A, k = int(case["A"]), int(case["k"])
    w = case["waddr"]
    r = case.get("raddr")
    m = case.get("wmask")
    code = payload_code(case)
    vals, mask, src, tape = oracle_mod.latestk_fwd(w, case["payload"], r, address_space=A, k=k,
                                                   write_mask=m, dtype=code)
    assert vals.shape == case["lk_vals"].shape
    assert np.array_equal(_bits(vals), _bits(case["lk_vals"])), "latest-k values differ bitwise"
    assert np.array_equal(mask, case["lk_mask"].astype(bool))

    B, T, C = w.shape
    D = case["payload"].shape[-1]
    grad = oracle_mod.latestk_bwd(mask, src, case["g_lk"].astype(np.float64), B * T * C).reshape(B, T, C, D)
    _close(grad, case["lk_grad64"])

    sums, smask, _ = oracle_mod.segsum_fwd(w, payload_as_float64(case), r, address_space=A, write_mask=m,
                                           tape=tape)
    assert np.array_equal(smask, case["ss_mask"].astype(bool))
    _close(sums, case["ss_sums64"])
    sgrad = oracle_mod.segsum_bwd(tape, smask, case["g_ss"].astype(np.float64))
    _close(sgrad, case["ss_grad64"])


def test_oracle_key_dtype_threshold(oracle_mod):
    """tests/test_memory.py:11-13 of the reference, plus the benchmark configurations."""
    z = load_golden("key_dtype")
    for (B, T, C, A), is32 in zip(z["cases"], z["is_int32"]):
        assert oracle_mod.key_is_int32(int(B), int(T), int(C), int(A)) == bool(is32)


def test_oracle_kat_values(oracle_mod):
    """tests/test_memory.py:16-23 and :61-67, restated as literal checks."""
    addr = np.array([[[1], [2], [1], [3], [1]]], np.int64)
    payload = np.arange(5, dtype=np.float32).reshape(1, 5, 1, 1)
    vals, mask, _, _ = oracle_mod.latestk_fwd(addr, payload, address_space=8, k=2)
    assert not mask[0, 0, 0, 0]
    assert vals[0, 2, 0, 0, 0] == 0.0 and vals[0, 4, 0, 0, 0] == 2.0 and vals[0, 4, 0, 1, 0] == 0.0
    addr = np.array([[[1], [2], [1], [1]]], np.int64)
    sums, _, _ = oracle_mod.segsum_fwd(addr, np.array([1.0, 10.0, 3.0, 7.0]).reshape(1, 4, 1, 1), address_space=8)
    assert sums[0, 0, 0, 0] == 0.0 and sums[0, 2, 0, 0] == 1.0 and sums[0, 3, 0, 0] == 4.0


def test_oracle_history_brute_force(oracle_mod):
    """Seeded brute-force history check (the pattern of tests/test_memory.py:26-58)."""
    rng = np.random.default_rng(3)
    B, T, C, D, A, k = 2, 40, 3, 2, 5, 3
    w = rng.integers(0, A, (B, T, C))
    r = rng.integers(0, A, (B, T, C))
    m = rng.random((B, T)) < 0.7
    p = rng.normal(size=(B, T, C, D)).astype(np.float32)
    vals, mask, _, _ = oracle_mod.latestk_fwd(w, p, r, address_space=A, k=k, write_mask=m)
    sums, smask, _ = oracle_mod.segsum_fwd(w, p.astype(np.float64), r, address_space=A, write_mask=m)
    for b in range(B):
        for c in range(C):
            hist: dict[int, list[int]] = {}
            for t in range(T):
                prior = hist.get(int(r[b, t, c]), [])
                for j in range(k):
                    if j < len(prior):
                        assert mask[b, t, c, j]
                        assert np.array_equal(vals[b, t, c, j], p[b, prior[-1 - j], c])
                    else:
                        assert not mask[b, t, c, j]
                        assert np.all(vals[b, t, c, j] == 0)
                expect = sum((p[b, s, c].astype(np.float64) for s in prior), np.zeros(D))
                assert smask[b, t, c] == bool(prior)
                np.testing.assert_allclose(sums[b, t, c], expect, rtol=1e-12, atol=1e-12)
                if m[b, t]:
                    hist.setdefault(int(w[b, t, c]), []).append(t)


def test_oracle_cache_sequence(oracle_mod):
    """RavelLayerCache read/write sequence (tests/test_memory.py:70-79 extended)."""
    z = load_golden("cache_sequence")
    B, C, A, D = (int(z[x]) for x in ("B", "C", "A", "D"))
    values = np.zeros((B, C, A, D), np.float32)
    filled = np.zeros((B, C, A), bool)
    for s in range(z["raddr"].shape[0]):
        v, m = oracle_mod.cache_read(values, filled, z["raddr"][s])
        assert np.array_equal(v.view(np.uint32), z["vals"][s].view(np.uint32))
        assert np.array_equal(m, z["mask"][s].astype(bool))
        oracle_mod.cache_write(values, filled, z["waddr"][s], z["payload"][s])
    assert np.array_equal(values, z["final_values"])
    assert np.array_equal(filled, z["final_filled"].astype(bool))
