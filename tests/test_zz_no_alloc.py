"""The no-allocation entry point ``ravel_segsum_fwd_noalloc`` (GPU).

Some hosts of this library cannot hand it device scratch: a plugin whose
enqueue callback is not allowed to allocate, or a caller in another language
that has no CUDA allocator.  ``ravel_segsum_fwd_noalloc`` serves them by keeping its tape and
scratch in a fixed-size device array inside the library.  This test calls it
through the C ABI and checks it against the allocating ``ravel_segsum_fwd`` on
two calls in a row with different sizes, flags and inputs (the array keeps the
previous call's contents, so the second call also checks that everything that
must start from zero is cleared), and that a call too large for the array is
refused without launching anything.

The file is named so that pytest collects it last.
"""
from __future__ import annotations

import pytest
import torch

from gpu_helpers import SUM_TOL

pytestmark = pytest.mark.gpu


def _case(seed, B, T, C, D, A, dtype, general, masked):
    g = torch.Generator().manual_seed(seed)
    w = torch.randint(-A, 2 * A, (B, T, C), generator=g).cuda()
    r = torch.randint(-A, 2 * A, (B, T, C), generator=g).cuda() if general else None
    m = (torch.rand(B, T, generator=g) < 0.7).cuda() if masked else None
    p = torch.randn(B, T, C, D, generator=g).to(dtype).cuda()
    return w, r, m, p


def _ptr(t):
    return None if t is None else t.data_ptr()


def _flags(L, r, m):
    return (L.RAVEL_TAPE_GENERAL_READS if r is not None else 0) | (L.RAVEL_TAPE_WRITE_MASK if m is not None else 0)


def _code(dtype):
    import ravel_lm_b200._lib as L
    return {torch.float32: L.RAVEL_F32, torch.bfloat16: L.RAVEL_BF16}[dtype]


def _allocating(L, w, r, m, p, A):
    lib = L.load()
    B, T, C, D = p.shape
    fl = _flags(L, r, m)
    tape = torch.empty(lib.ravel_tape_bytes(B, T, C, A, fl), dtype=torch.uint8, device="cuda")
    scratch = torch.empty(lib.ravel_scratch_bytes(B, T, C, D, A, 1, _code(p.dtype), fl), dtype=torch.uint8, device="cuda")
    sums = torch.empty_like(p)
    mask = torch.empty(B, T, C, dtype=torch.bool, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    rc = lib.ravel_segsum_fwd(w.data_ptr(), _ptr(r), L.RAVEL_I64, _ptr(m), p.data_ptr(), _code(p.dtype), B, T, C, D,
                              A, sums.data_ptr(), mask.data_ptr(), tape.data_ptr(), tape.numel(),
                              scratch.data_ptr(), scratch.numel(), st)
    assert rc == 0
    return sums, mask


def _no_alloc(L, w, r, m, p, A):
    lib = L.load()
    B, T, C, D = p.shape
    sums = torch.full_like(p, float("nan"))
    mask = torch.ones(B, T, C, dtype=torch.bool, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    rc = lib.ravel_segsum_fwd_noalloc(w.data_ptr(), _ptr(r), L.RAVEL_I64, _ptr(m), p.data_ptr(), _code(p.dtype),
                                      B, T, C, D, A, sums.data_ptr(), mask.data_ptr(), st)
    return rc, sums, mask


def test_no_alloc_matches_allocating_entry_point_twice():
    import ravel_lm_b200._lib as L
    assert torch.cuda.is_available()
    cases = [
        # multi-tile streams (sort ping-pong in scratch), general reads, write mask
        dict(seed=1, B=2, T=12000, C=3, D=32, A=700, dtype=torch.float32, general=True, masked=True),
        # a different, smaller aliased case in the same array
        dict(seed=2, B=3, T=2048, C=4, D=64, A=65536, dtype=torch.bfloat16, general=False, masked=False),
    ]
    for c in cases:
        w, r, m, p = _case(c["seed"], c["B"], c["T"], c["C"], c["D"], c["A"], c["dtype"], c["general"], c["masked"])
        ref_sums, ref_mask = _allocating(L, w, r, m, p, c["A"])
        rc, sums, mask = _no_alloc(L, w, r, m, p, c["A"])
        torch.cuda.synchronize()
        assert rc == 0, L.load().ravel_status_string(rc)
        assert torch.equal(mask, ref_mask)
        tol = SUM_TOL[c["dtype"]]
        torch.testing.assert_close(sums.float(), ref_sums.float(), rtol=tol, atol=tol)
    assert L.device_error(torch.cuda.current_stream().cuda_stream) == 0


def test_no_alloc_refuses_sizes_beyond_its_array():
    import ravel_lm_b200._lib as L
    lib = L.load()
    B, T, C, D, A = 4, 32768, 16, 256, 65536  # tape + scratch well above the array
    need = lib.ravel_tape_bytes(B, T, C, A, 0) + lib.ravel_scratch_bytes(B, T, C, D, A, 1, L.RAVEL_F32, 0)
    assert need > L.RAVEL_NOALLOC_SCRATCH_BYTES
    w = torch.zeros(1, dtype=torch.int64, device="cuda")  # never read: the call is refused first
    out = torch.zeros(1, device="cuda")
    launches = L.kernel_launches()
    rc = lib.ravel_segsum_fwd_noalloc(w.data_ptr(), None, L.RAVEL_I64, None, out.data_ptr(), L.RAVEL_F32,
                                      B, T, C, D, A, out.data_ptr(), out.data_ptr(),
                                      torch.cuda.current_stream().cuda_stream)
    assert rc == L.RAVEL_ERR_WORKSPACE
    assert L.kernel_launches() == launches
