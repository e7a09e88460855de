"""Failure detection on the GPU without faulting it.

Every wait on another block is bounded: after the poll limit
(``ravel_set_wait_limit``) it gives up, sets ``RAVEL_DEVERR_SPIN`` in the device
error word and returns, so the context stays usable.  The self-test entry point
runs that same wait on a device word nothing sets; the look-back of the real
scan, at a one-poll limit, must either finish exactly or report the give-up --
never return a wrong sum silently.
"""
from __future__ import annotations

import time

import pytest
import torch

pytestmark = pytest.mark.gpu

DEFAULT_LIMIT = 1 << 22


@pytest.fixture()
def lib():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import ravel_lm_b200._lib as L
    L.load()
    st = torch.cuda.current_stream().cuda_stream
    L.clear_device_error(st)
    yield L, st
    L.call("ravel_set_wait_limit", DEFAULT_LIMIT)
    L.clear_device_error(st)


def test_a_wait_nothing_answers_gives_up_and_reports(lib):
    L, st = lib
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    L.call("ravel_set_wait_limit", 20000)
    t0 = time.perf_counter()
    L.call("ravel_wait_selftest", flag.data_ptr(), st)
    err = L.device_error(st)
    assert err & L.RAVEL_DEVERR_SPIN
    assert time.perf_counter() - t0 < 10.0
    # the context is still usable: clear, restore the limit, run a lookup
    L.clear_device_error(st)
    L.call("ravel_set_wait_limit", DEFAULT_LIMIT)
    from ravel_lm_b200 import causal_last_k_lookup
    w = torch.tensor([[[1], [2], [1], [3], [1]]], device="cuda")
    p = torch.arange(5, dtype=torch.float32, device="cuda").view(1, 5, 1, 1)
    vals, mask = causal_last_k_lookup(w, p, address_space=8, k=2)
    assert vals[0, 4, 0, :, 0].tolist() == [2.0, 0.0] and mask[0, 4, 0].tolist() == [True, True]
    assert L.device_error(st) == 0


def test_a_set_flag_passes(lib):
    L, st = lib
    flag = torch.ones(1, dtype=torch.int32, device="cuda")
    L.call("ravel_wait_selftest", flag.data_ptr(), st)
    assert L.device_error(st) == 0


def test_wait_limit_argument_checks(lib):
    L, _ = lib
    with pytest.raises(ValueError):
        L.call("ravel_set_wait_limit", 0)
    with pytest.raises(ValueError):
        L.call("ravel_set_wait_limit", 1 << 29)


@pytest.mark.parametrize("D", [64, 24])  # the range scan and the look-back fallback scan
def test_one_poll_scans_are_exact_or_report(lib, D):
    L, st = lib
    from ravel_lm_b200 import causal_sum_lookup
    from ravel_lm_b200.ravel_memory import clear_tape_cache
    g = torch.Generator(device="cuda").manual_seed(D)
    w = torch.randint(0, 3, (2, 30000, 4), generator=g, device="cuda")  # long segments: carries cross blocks
    p = torch.randn(2, 30000, 4, D, generator=g, device="cuda")
    want, _ = causal_sum_lookup(w, p, address_space=3)
    torch.cuda.synchronize()
    L.call("ravel_set_wait_limit", 1)
    reported = 0
    for _ in range(20):
        clear_tape_cache()
        got, _ = causal_sum_lookup(w, p, address_space=3)
        err = L.device_error(st)
        if err & L.RAVEL_DEVERR_SPIN:
            reported += 1
            L.clear_device_error(st)
        else:
            assert torch.equal(got, want), "a scan that reported nothing must be exact"
    L.call("ravel_set_wait_limit", DEFAULT_LIMIT)
    clear_tape_cache()
    again, _ = causal_sum_lookup(w, p, address_space=3)
    assert torch.equal(again, want) and L.device_error(st) == 0


@pytest.mark.parametrize("D,dtype", [(64, torch.bfloat16), (24, torch.float32)])
def test_scans_are_reproducible_bit_for_bit(lib, D, dtype):
    """Long segments spanning many blocks: the forward and backward sums of repeated calls
    are the same bits (no timing-dependent association in the look-back)."""
    from ravel_lm_b200 import causal_sum_lookup
    from ravel_lm_b200.ravel_memory import clear_tape_cache
    g = torch.Generator(device="cuda").manual_seed(5)
    w = torch.randint(0, 2, (2, 30000, 8), generator=g, device="cuda")
    p0 = torch.randn(2, 30000, 8, D, generator=g, device="cuda").to(dtype)
    gs = torch.randn(2, 30000, 8, D, generator=g, device="cuda").to(dtype)
    outs = []
    for _ in range(6):
        clear_tape_cache()
        p = p0.clone().requires_grad_(True)
        sums, _ = causal_sum_lookup(w, p, address_space=2)
        sums.backward(gs)
        outs.append((sums.detach(), p.grad))
    for s2, g2 in outs[1:]:
        assert torch.equal(s2, outs[0][0]) and torch.equal(g2, outs[0][1])
