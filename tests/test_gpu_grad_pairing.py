"""The two lookups of one payload share one gradient buffer in a single backward pass.

When ``causal_sum_lookup`` reuses the tape of a ``causal_last_k_lookup`` call
on the same payload, one backward pass through both writes the payload
gradient once: the sum's backward fills it and the latest-k backward adds its
part in its own kernel (``ravel_latestk_bwd_accumulate``) instead of autograd
adding two tensors.  These tests check the total against the float64 oracle
and check that every other way of taking gradients still gives each lookup's
own gradient.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from gpu_helpers import SUM_TOL, assert_close, payload_np, to_f64

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import ravel_lm_b200._lib as L
    L.load()
    yield
    L.set_call_hook(None)
    torch.cuda.synchronize()
    assert L.device_error(torch.cuda.current_stream().cuda_stream) == 0


class Calls:
    """Names of the C-ABI entry points called inside the block."""

    def __enter__(self):
        import ravel_lm_b200._lib as L
        self.names = []
        L.set_call_hook(lambda name, thunk: (self.names.append(name), thunk())[1])
        return self

    def __exit__(self, *exc):
        import ravel_lm_b200._lib as L
        L.set_call_hook(None)


def _case(general, masked, dtype, seed=3):
    g = torch.Generator().manual_seed(seed)
    B, T, C, D, A, k = 2, 1500, 3, 32, 90, 3
    w = torch.randint(0, A, (B, T, C), generator=g)
    r = torch.randint(0, A, (B, T, C), generator=g) if general else None
    m = (torch.rand(B, T, generator=g) < 0.7) if masked else None
    p = torch.randn(B, T, C, D, generator=g).to(dtype)
    gv = torch.randn(B, T, C, k, D, generator=g).to(dtype)
    gs = torch.randn(B, T, C, D, generator=g).to(dtype)
    return dict(w=w, r=r, m=m, p=p, gv=gv, gs=gs, A=A, k=k)


def _expected(oracle, c):
    """float64 payload gradients of each lookup (oracle)."""
    code = {torch.bfloat16: "bf16", torch.float16: "f16"}.get(c["p"].dtype)
    w, p = c["w"].numpy(), payload_np(c["p"])
    r = None if c["r"] is None else c["r"].numpy()
    m = None if c["m"] is None else c["m"].numpy()
    vals, mask, src, tape = oracle.latestk_fwd(w, p, r, address_space=c["A"], k=c["k"], write_mask=m, dtype=code)
    _, smask, _ = oracle.segsum_fwd(w, to_f64(c["p"]), r, address_space=c["A"], write_mask=m, tape=tape)
    B, T, C, D = c["p"].shape
    glk = oracle.latestk_bwd(mask, src, to_f64(c["gv"]), B * T * C).reshape(B, T, C, D)
    gss = oracle.segsum_bwd(tape, smask, to_f64(c["gs"]))
    return glk, gss


def _lookups(c, p):
    from ravel_lm_b200 import causal_last_k_lookup, causal_sum_lookup
    w = c["w"].cuda()
    r = None if c["r"] is None else c["r"].cuda()
    m = None if c["m"] is None else c["m"].cuda()
    vals, _ = causal_last_k_lookup(w, p, r, address_space=c["A"], k=c["k"], write_mask=m)
    sums, _ = causal_sum_lookup(w, p, r, address_space=c["A"], write_mask=m)
    return vals, sums


@pytest.mark.parametrize("general,masked", [(False, False), (True, False), (True, True), (False, True)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_one_pass_writes_the_total_once(oracle_mod, general, masked, dtype):
    c = _case(general, masked, dtype)
    glk, gss = _expected(oracle_mod, c)
    p = c["p"].cuda().requires_grad_(True)
    with Calls() as calls:
        vals, sums = _lookups(c, p)
        torch.autograd.backward([vals, sums], [c["gv"].cuda(), c["gs"].cuda()])
        torch.cuda.synchronize()
    assert calls.names.count("ravel_latestk_bwd_accumulate") == 1, calls.names
    assert "ravel_latestk_bwd" not in calls.names
    assert_close(to_f64(p.grad), glk + gss, SUM_TOL[dtype], "summed payload gradient")


def test_other_uses_keep_their_own_gradients(oracle_mod):
    c = _case(True, True, torch.float32)
    glk, gss = _expected(oracle_mod, c)
    tol = SUM_TOL[torch.float32]
    gv, gs = c["gv"].cuda(), c["gs"].cuda()
    # only one of the two outputs in the pass
    for which, want in ((0, glk), (1, gss)):
        p = c["p"].cuda().requires_grad_(True)
        outs = _lookups(c, p)
        with Calls() as calls:
            torch.autograd.backward([outs[which]], [(gv, gs)[which]])
        assert "ravel_latestk_bwd_accumulate" not in calls.names
        assert_close(to_f64(p.grad), want, tol, f"output {which} alone")
    # two separate passes over a retained graph
    p = c["p"].cuda().requires_grad_(True)
    vals, sums = _lookups(c, p)
    with Calls() as calls:
        a = torch.autograd.grad(sums, p, gs, retain_graph=True)[0]
        b = torch.autograd.grad(vals, p, gv)[0]
    assert "ravel_latestk_bwd_accumulate" not in calls.names
    assert_close(to_f64(a), gss, tol, "sum pass")
    assert_close(to_f64(b), glk, tol, "latest-k pass")
    # a third consumer of the payload in the same pass
    p = c["p"].cuda().requires_grad_(True)
    vals, sums = _lookups(c, p)
    extra = (p * 2.0).sum()
    with Calls() as calls:
        torch.autograd.backward([vals, sums, extra], [gv, gs, None])
    assert calls.names.count("ravel_latestk_bwd_accumulate") == 1
    assert_close(to_f64(p.grad), glk + gss + 2.0, tol, "with a third consumer")
    # the sum lookup first: the latest-k backward runs first and nothing is handed over
    from ravel_lm_b200 import causal_last_k_lookup, causal_sum_lookup
    p = c["p"].cuda().requires_grad_(True)
    w, r, m = c["w"].cuda(), c["r"].cuda(), c["m"].cuda()
    sums, _ = causal_sum_lookup(w, p, r, address_space=c["A"], write_mask=m)
    vals, _ = causal_last_k_lookup(w, p, r, address_space=c["A"], k=c["k"], write_mask=m)
    with Calls() as calls:
        torch.autograd.backward([vals, sums], [gv, gs])
    assert "ravel_latestk_bwd_accumulate" not in calls.names
    assert_close(to_f64(p.grad), glk + gss, tol, "sum lookup first")


def test_a_payload_changed_in_place_is_not_paired(oracle_mod):
    c = _case(False, False, torch.float32)
    from ravel_lm_b200 import causal_last_k_lookup, causal_sum_lookup
    leaf = c["p"].cuda().requires_grad_(True)
    p = leaf * 1.0
    w = c["w"].cuda()
    vals, _ = causal_last_k_lookup(w, p, address_space=c["A"], k=c["k"])
    p.mul_(1.0)  # same values, new version: the sum lookup sees another tensor state
    sums, _ = causal_sum_lookup(w, p, address_space=c["A"])
    with Calls() as calls:
        torch.autograd.backward([vals, sums], [c["gv"].cuda(), c["gs"].cuda()])
    assert "ravel_latestk_bwd_accumulate" not in calls.names
    glk, gss = _expected(oracle_mod, c)
    assert_close(to_f64(leaf.grad), glk + gss, SUM_TOL[torch.float32], "in-place case")


def test_layer_shaped_use_concat_and_linear(oracle_mod):
    """The memory layer's own pattern (model.py:367-386): both outputs concatenated and fed
    to a Linear; the pairing happens and the gradient matches the same graph in float64."""
    c = _case(True, False, torch.float32, seed=11)
    B, T, C, D = c["p"].shape
    torch.manual_seed(0)
    lin = torch.nn.Linear(C * (c["k"] + 1) * D, 16, bias=False).cuda()
    p = c["p"].cuda().requires_grad_(True)
    with Calls() as calls:
        vals, sums = _lookups(c, p)
        out = lin(torch.cat([vals.reshape(B, T, -1), sums.reshape(B, T, -1)], -1))
        out.square().sum().backward()
    assert calls.names.count("ravel_latestk_bwd_accumulate") == 1
    # reference: the same graph with the gradients split out by hand
    p2 = c["p"].cuda().requires_grad_(True)
    vals2, sums2 = _lookups(c, p2)
    out2 = lin(torch.cat([vals2.reshape(B, T, -1), sums2.reshape(B, T, -1)], -1))
    gv2, gs2 = torch.autograd.grad(out2.square().sum(), [vals2, sums2])
    a = torch.autograd.grad(vals2, p2, gv2, retain_graph=True)[0]
    b = torch.autograd.grad(sums2, p2, gs2)[0]
    torch.testing.assert_close(p.grad, a + b, rtol=1e-5, atol=1e-5)
    assert np.isfinite(to_f64(p.grad)).all()
