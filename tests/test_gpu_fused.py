"""The memory layer's read-out on the tensor cores (``memory_read_linear``).

The fused kernel must equal ``fuse(cat(latest-k values, sums))`` (and the gate
residual on top, ``ravel_lm/model.py:367-388``) computed from the unfused
pieces in float64, within the TF32 tolerance of its inputs (the reference's own
CUDA ``fast_linear`` is a TF32 Triton dot): |error| <= 5e-3 * max|expected|.
Its backward (cuBLAS float32 GEMMs plus the operator's own backward kernels)
must match float64 autograd of the unfused composition within 1e-4 of the
largest gradient (the gate's gradient, a product with the forward's TF32
result, within the forward's tolerance).  Cases cover aliased and general reads, a write mask, k of
1-3, with and without the sum read, N below, at and above one tile (64, 128,
256 columns), token counts that are not a multiple of 128, and a K of 24 (one
partial 32-float chunk).
"""
from __future__ import annotations

import zlib

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import ravel_lm_b200._lib as L
    L.load()
    yield
    torch.cuda.synchronize()
    assert L.device_error(torch.cuda.current_stream().cuda_stream) == 0


def _case(B, T, C, D, A, k, N, general, masked, use_sum, gated, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    K = C * k * D + (C * D if use_sum else 0)
    c = dict(B=B, T=T, C=C, D=D, A=A, k=k, N=N, use_sum=use_sum)
    c["w"] = torch.randint(0, A, (B, T, C), generator=g, device="cuda")
    c["r"] = torch.randint(0, A, (B, T, C), generator=g, device="cuda") if general else None
    c["m"] = (torch.rand(B, T, generator=g, device="cuda") < 0.8) if masked else None
    c["p"] = torch.randn(B, T, C, D, generator=g, device="cuda")
    c["W"] = torch.randn(N, K, generator=g, device="cuda") * K ** -0.5
    c["x"] = torch.randn(B, T, N, generator=g, device="cuda") if gated else None
    c["gate"] = torch.randn(B, T, N, generator=g, device="cuda") if gated else None
    c["gy"] = torch.randn(B, T, N, generator=g, device="cuda")
    return c


def _composed(c, p, W, x, gate):
    """The unfused layer read-out (ravel_lm/model.py:367-388) with this package's lookups."""
    from ravel_lm_b200 import causal_last_k_lookup, causal_sum_lookup
    from ravel_lm_b200.ravel_memory import clear_tape_cache
    clear_tape_cache()
    B, T = c["B"], c["T"]
    vals, _ = causal_last_k_lookup(c["w"], p, c["r"], address_space=c["A"], k=c["k"], write_mask=c["m"])
    pieces = [vals.reshape(B, T, -1)]
    if c["use_sum"]:
        sums, _ = causal_sum_lookup(c["w"], p, c["r"], address_space=c["A"], write_mask=c["m"])
        pieces.append(sums.reshape(B, T, -1))
    out = torch.nn.functional.linear(torch.cat(pieces, -1), W)
    if x is not None:
        out = x + torch.sigmoid(gate) * out
    return out


def _check(c, tol_fwd=5e-3, tol_bwd=1e-4):
    from ravel_lm_b200.fused import memory_read_linear
    from ravel_lm_b200.ravel_memory import clear_tape_cache
    leaves = {n: (c[n].clone().requires_grad_(True) if c[n] is not None else None) for n in ("p", "W", "x", "gate")}
    clear_tape_cache()
    out = memory_read_linear(c["w"], leaves["p"], c["r"], leaves["W"], address_space=c["A"], k=c["k"],
                             use_sum_read=c["use_sum"], write_mask=c["m"], x=leaves["x"], gate_lin=leaves["gate"])
    out.backward(c["gy"])
    ref = {n: (c[n].double().requires_grad_(True) if c[n] is not None else None) for n in ("p", "W", "x", "gate")}
    want = _composed(c, ref["p"], ref["W"], ref["x"], ref["gate"])
    want.backward(c["gy"].double())
    want = want.detach()
    scale = float(want.abs().max())
    err = float((out.double() - want).abs().max())
    assert err <= tol_fwd * scale, f"forward: max error {err:.3g} vs {tol_fwd} * {scale:.3g}"
    for n in ("p", "W", "x", "gate"):
        if ref[n] is None:
            continue
        # d gate = gy * (A W^T) * s * (1 - s) carries the forward's TF32 error; the
        # others come from float32 GEMMs of exact rows
        tol = tol_fwd if n == "gate" else tol_bwd
        g, gw = leaves[n].grad.double(), ref[n].grad
        e, s = float((g - gw).abs().max()), float(gw.abs().max())
        assert e <= tol * s, f"grad {n}: max error {e:.3g} vs {tol} * {s:.3g}"


def test_small_aliased_with_sums():
    _check(_case(B=2, T=200, C=4, D=32, A=50, k=2, N=128, general=False, masked=False, use_sum=True, gated=False,
                 seed=1))


@pytest.mark.parametrize("name,kw", [
    ("general_mask_k3_N80", dict(B=3, T=333, C=3, D=16, A=40, k=3, N=80, general=True, masked=True, use_sum=False,
                                 gated=False)),
    ("gated_N64_K24", dict(B=2, T=100, C=2, D=4, A=9, k=2, N=64, general=False, masked=False, use_sum=True,
                           gated=True)),
    ("cfg5_layer", dict(B=8, T=1024, C=8, D=32, A=1024, k=2, N=256, general=True, masked=False, use_sum=True,
                        gated=True)),
    ("N256_tiles", dict(B=20, T=1024, C=4, D=32, A=512, k=2, N=256, general=False, masked=False, use_sum=True,
                        gated=False)),
    ("N300", dict(B=1, T=300, C=2, D=8, A=30, k=1, N=300, general=True, masked=False, use_sum=False, gated=True)),
])
def test_read_linear_cases(name, kw):
    _check(_case(seed=zlib.crc32(name.encode()) % 1000, **kw))


def test_token_addressed_equals_address_tensors():
    from ravel_lm_b200 import literal_addresses_from_tokens
    from ravel_lm_b200.fused import memory_read_linear, memory_read_linear_tokens
    g = torch.Generator(device="cuda").manual_seed(3)
    B, T, L, Ll, D, A, k, N = 4, 512, 4, 4, 32, 1024, 2, 256
    toks = torch.randint(0, 1024, (B, T), generator=g, device="cuda")
    lw = torch.randint(0, A, (B, T, Ll), generator=g, device="cuda")
    lr = torch.randint(0, A, (B, T, Ll), generator=g, device="cuda")
    p = torch.randn(B, T, L + Ll, D, generator=g, device="cuda")
    W = torch.randn(N, (L + Ll) * (k + 1) * D, generator=g, device="cuda") * 0.02
    a = memory_read_linear_tokens(toks, p, lw, lr, W, address_space=A, n_literal_heads=L, bos_token_id=257, k=k,
                                  use_sum_read=True)
    lit = literal_addresses_from_tokens(toks, address_space=A, n_heads=L, bos_token_id=257)
    b = memory_read_linear(torch.cat([lit, lw], -1), p, torch.cat([lit, lr], -1), W, address_space=A, k=k,
                           use_sum_read=True)
    assert torch.equal(a, b)


def test_two_calls_in_a_row_and_graph_capture():
    """Repeated launches reuse nothing stale; a captured call replays to the eager result."""
    from ravel_lm_b200.fused import memory_read_linear
    c = _case(B=2, T=256, C=4, D=32, A=64, k=2, N=128, general=True, masked=False, use_sum=True, gated=True, seed=8)
    args = (c["w"], c["p"], c["r"], c["W"])
    kw = dict(address_space=c["A"], k=c["k"], use_sum_read=True, x=c["x"], gate_lin=c["gate"])
    e1 = memory_read_linear(*args, **kw)
    e2 = memory_read_linear(*args, **kw)
    assert torch.equal(e1, e2)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(side):
        memory_read_linear(*args, **kw)
        with torch.cuda.graph(graph, stream=side):
            cap = memory_read_linear(*args, **kw)
    torch.cuda.current_stream().wait_stream(side)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(cap, e1)
    del graph
