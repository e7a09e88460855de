"""CPU-only checks of the C ABI library and the Python boundary (no GPU calls)."""
from __future__ import annotations

import re
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]


def _declared_symbols() -> list[str]:
    text = (ROOT / "include" / "ravel_b200.h").read_text()
    return sorted(set(re.findall(r"^\s*(?:[\w\s\*]+?)\b(ravel_\w+)\s*\(", text, flags=re.M)))


def test_library_exports_every_declared_symbol():
    import ravel_lm_b200._lib as L
    lib = L.load()
    names = _declared_symbols()
    assert len(names) >= 16
    for n in names:
        assert hasattr(lib, n), f"{n} declared in include/ravel_b200.h but not exported"
    assert set(names) == set(L.SIGNATURES), "ctypes signature table out of sync with the header"


def test_version_and_status_strings():
    import ravel_lm_b200._lib as L
    lib = L.load()
    assert b"sm_100a" in lib.ravel_version()
    assert lib.ravel_status_string(0) == b"ok"
    assert b"invalid" in lib.ravel_status_string(1)


def test_tape_and_scratch_sizes():
    import ravel_lm_b200._lib as L
    lib = L.load()
    # config 3: 32-bit keys, T fits one key per event -> 64 streams x 32768 x 4 bytes
    t3 = lib.ravel_tape_bytes(4, 32768, 16, 65536, 0)
    assert 64 * 32768 * 4 <= t3 < 64 * 32768 * 4 + 4096
    # general reads add one int32 per read
    t3g = lib.ravel_tape_bytes(4, 32768, 16, 65536, L.RAVEL_TAPE_GENERAL_READS)
    assert t3g - t3 >= 4 * 32768 * 16 * 4
    # 64-bit keys when address + time bits exceed 32
    assert lib.ravel_tape_bytes(1, 4096, 1, 2**31, 0) >= 4096 * 8
    assert lib.ravel_tape_bytes(1, 4, 1, 0, 0) == 0  # A must be positive
    s = lib.ravel_scratch_bytes(4, 32768, 16, 64, 65536, 8, L.RAVEL_BF16, 0)
    assert s > 0


def test_entry_points_reject_bad_arguments_without_touching_a_gpu():
    import ravel_lm_b200._lib as L
    lib = L.load()
    # k <= 0, A <= 0, null pointers: rejected during validation, before any CUDA call
    assert lib.ravel_latestk_fwd_tape(None, 0, None, 1, None, 0, 1, 4, 1, 2, 8, 0, None, None, None) == 1
    assert lib.ravel_latestk_fwd_tape(None, 0, None, 1, None, 0, 1, 4, 1, 2, 0, 1, None, None, None) == 1
    assert lib.ravel_cache_read(None, None, None, 1, 0, 1, 1, 4, 2, None, None, None) == 1
    assert lib.ravel_latestk_fwd_tape(None, 0, None, 1, None, 9, 1, 4, 1, 2, 8, 1, None, None, None) == 1
    assert lib.ravel_latestk_fwd_tape(None, 0, None, 1, None, 0, 1, 4, 1, 2, 8, 1000, None, None, None) == 4


def test_python_api_validation_matches_reference_messages():
    from ravel_lm_b200 import causal_last_k_lookup, causal_sum_lookup
    a = torch.zeros(1, 4, 2, dtype=torch.long)
    p = torch.zeros(1, 4, 2, 3)
    with pytest.raises(ValueError, match="same shape"):
        causal_last_k_lookup(a, p, torch.zeros(1, 5, 2, dtype=torch.long), address_space=8)
    with pytest.raises(ValueError, match=r"addresses must have shape \[B, T, C\]"):
        causal_last_k_lookup(a[0], p, address_space=8)
    with pytest.raises(ValueError, match=r"payloads must have shape \[B, T, C, D\]"):
        causal_last_k_lookup(a, p[0], address_space=8)
    with pytest.raises(ValueError, match="leading dimensions"):
        causal_last_k_lookup(a, torch.zeros(1, 3, 2, 3), address_space=8)
    with pytest.raises(ValueError, match="k must be positive"):
        causal_last_k_lookup(a, p, address_space=8, k=0)
    with pytest.raises(ValueError, match=r"write_mask must have shape \[B, T\]"):
        causal_last_k_lookup(a, p, address_space=8, write_mask=torch.ones(1, 3, dtype=torch.bool))
    with pytest.raises(ValueError, match="expected write_addresses"):
        causal_sum_lookup(a[0], p, address_space=8)
    # valid shapes on CPU tensors: no fallback, a loud error
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        causal_last_k_lookup(a, p, address_space=8)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        causal_sum_lookup(a, p, address_space=8)


def test_cache_validation_and_no_cpu_path():
    from ravel_lm_b200 import RavelLayerCache
    c = RavelLayerCache.empty(2, 3, 16, 4, device="cpu", dtype=torch.float32)
    assert c.values.shape == (2, 3, 16, 4) and c.filled.dtype == torch.bool and not c.filled.any()
    with pytest.raises(ValueError, match="does not match"):
        c.read(torch.zeros(2, 2, dtype=torch.long))
    with pytest.raises(ValueError, match="do not match"):
        c.write(torch.zeros(2, 3, dtype=torch.long), torch.zeros(2, 3, 5))
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        c.read(torch.zeros(2, 3, dtype=torch.long))
    with pytest.raises(ValueError, match="shape"):
        c.prefill(torch.zeros(2, 3, dtype=torch.long), torch.zeros(2, 3, 4))
    with pytest.raises(ValueError, match="do not match"):
        c.prefill(torch.zeros(2, 5, 3, dtype=torch.long), torch.zeros(2, 4, 3, 4))
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        c.prefill(torch.zeros(2, 5, 3, dtype=torch.long), torch.zeros(2, 5, 3, 4))
    # step: the C++ fast path declines CPU tensors and the checked path raises
    a = torch.zeros(2, 3, dtype=torch.long)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        c.step(a, a, torch.zeros(2, 3, 4))
    with pytest.raises(ValueError, match="do not match"):
        c.step(a, a, torch.zeros(2, 2, 4))


def test_host_extension_loads_and_timing_api_without_a_gpu():
    import ravel_lm_b200._lib as L
    h = L.host()
    for name in ("cache_step", "tape_build", "latestk_fwd", "segsum_fwd", "segsum_bwd", "latestk_bwd"):
        assert callable(getattr(h, name)), name
    # the extension links to the very library ctypes loaded (one copy of its counters)
    lib = L.load()
    assert lib.ravel_timing_start(0) == L.RAVEL_ERR_INVALID_ARG
    assert lib.ravel_timing_stop() == L.RAVEL_OK
    assert lib.ravel_timing_count() == 0
    assert L.timing_stop() == []


def test_composite_key_dtype_matches_reference_golden():
    from conftest import load_golden
    from ravel_lm_b200 import _composite_key_dtype
    z = load_golden("key_dtype")
    for (B, T, C, A), is32 in zip(z["cases"], z["is_int32"]):
        assert (_composite_key_dtype(int(B), int(T), int(C), int(A)) == torch.int32) == bool(is32)


def test_fake_tensor_shapes_for_compile():
    """The custom ops' fake implementations give the right output shapes."""
    from torch._subclasses.fake_tensor import FakeTensorMode
    import ravel_lm_b200.ravel_memory as rm
    with FakeTensorMode():
        w = torch.empty(2, 8, 3, dtype=torch.long, device="cuda")
        p = torch.empty(2, 8, 3, 5, dtype=torch.bfloat16, device="cuda")
        v, m, t = rm._latestk_fwd(w, p, None, None, 16, 4)
        assert v.shape == (2, 8, 3, 4, 5) and v.dtype == torch.bfloat16 and m.dtype == torch.bool
        s, sm, _ = rm._segsum_fwd(w, p, None, None, 16)
        assert s.shape == (2, 8, 3, 5) and sm.shape == (2, 8, 3)


def test_workload_generator_is_seeded():
    from ravel_lm_b200.workloads import CONFIGS, make_inputs, zipf_ranks
    x1 = make_inputs(CONFIGS[1])
    x2 = make_inputs(CONFIGS[1])
    assert torch.equal(x1["write"], x2["write"]) and torch.equal(x1["payload"], x2["payload"])
    assert x1["write"].shape == (8, 256, 4) and x1["write"].max() < 256
    g = torch.Generator().manual_seed(0)
    z = zipf_ranks(1000, 1.1, (200000,), g)
    counts = np.bincount(z.numpy(), minlength=1000)
    assert counts[0] > counts[1] > counts[10] > counts[500]
    x5 = make_inputs(CONFIGS[5])
    assert torch.equal(x5["write"][..., :4], x5["read"][..., :4])
    assert not torch.equal(x5["write"][..., 4:], x5["read"][..., 4:])
