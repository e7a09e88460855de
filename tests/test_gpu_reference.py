"""CUDA path vs the reference's own PyTorch code on the same B200, at full sizes.

The reference (``ravel_lm/ravel_memory.py``) is pure Python over torch ops, so
its functions run on CUDA tensors too.  These tests import an installed copy of
it from ``baseline/_ref`` (``pip install --no-deps --target baseline/_ref
<ravel-lm>``; skipped when absent) and run both implementations on identical
seeded inputs of the benchmark configurations:

* latest-k values and masks: bit for bit against the reference's torch path
  (``ravel_memory.py:126-176``).  Configuration 1 is also compared with the
  kernel the reference's dispatch picks for it on CUDA (Triton v2,
  ``triton_latest1.py:86-154``), which writes +0.0 into invalid slots where
  the torch path writes ``candidate * 0``: equal as values;
* segmented sums and every gradient: within the operator's tolerance
  (1e-5 float32, 1e-2 bfloat16 with float32 accumulation) of the reference
  run on ``payloads.double()``;
* the decode cache at configuration 4 (256 x 16 streams, A = 4096, D = 64
  bf16): a 4096-step prefill and 1024 read + write steps, every read and the
  final cache bit for bit against the reference's ``RavelLayerCache``;
* ``torch.compile(fullgraph=True)`` of both lookups, forward and backward:
  bit for bit equal to eager.
"""
from __future__ import annotations

import contextlib
import sys
from pathlib import Path

import pytest
import torch

from gpu_helpers import SUM_TOL

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
REF = ROOT / "baseline" / "_ref"


@pytest.fixture(scope="module")
def ref():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    if not (REF / "ravel_lm" / "ravel_memory.py").exists():
        pytest.skip("no installed reference under baseline/_ref")
    if str(REF) not in sys.path:
        sys.path.insert(0, str(REF))
    import ravel_lm.ravel_memory as mem
    import ravel_lm.triton_latest1 as tl1
    import ravel_lm_b200._lib as L
    L.load()
    yield mem, tl1
    torch.cuda.synchronize()
    assert L.device_error(torch.cuda.current_stream().cuda_stream) == 0


@contextlib.contextmanager
def _torch_path(tl1):
    """Make the reference's dispatch skip its Triton v2 kernel (its torch path runs)."""
    old = tl1._HAS_TRITON
    tl1._HAS_TRITON = False
    try:
        yield
    finally:
        tl1._HAS_TRITON = old


def _bits(t: torch.Tensor) -> torch.Tensor:
    t = t.detach().contiguous()
    return t.view({2: torch.int16, 4: torch.int32, 8: torch.int64}[t.element_size()]) if t.is_floating_point() else t


def _assert_bits(a: torch.Tensor, b: torch.Tensor, what: str) -> None:
    assert a.shape == b.shape and a.dtype == b.dtype, f"{what}: {a.shape}/{a.dtype} vs {b.shape}/{b.dtype}"
    diff = _bits(a) != _bits(b)
    n = int(diff.sum())
    if n:
        idx = diff.nonzero()[:4].tolist()
        raise AssertionError(f"{what}: {n} of {a.numel()} elements differ bitwise; first at {idx}")


def _assert_close(actual: torch.Tensor, expected: torch.Tensor, tol: float, what: str) -> None:
    a, e = actual.detach().double(), expected.detach().double()
    scale = float(e.abs().max()) if e.numel() else 0.0
    bound = tol * (e.abs() + max(scale, 1e-30))
    bad = (a - e).abs() > bound
    n = int(bad.sum())
    if n:
        i = int(((a - e).abs() - bound).flatten().argmax())
        raise AssertionError(f"{what}: {n} of {a.numel()} beyond tol {tol}; worst: {a.flatten()[i].item()!r} vs "
                             f"{e.flatten()[i].item()!r} (max|expected| {scale:.3g})")


def _inputs(cfg, seed):
    from ravel_lm_b200.workloads import make_inputs
    x = make_inputs(cfg, seed=seed, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(seed + 1)
    B, T, C, D, k = cfg.B, cfg.T, cfg.C, cfg.D, cfg.k
    if "g_vals" not in x:
        x["g_vals"] = torch.randn(B, T, C, k, D, generator=g, device="cuda").to(cfg.dtype)
        x["g_sums"] = torch.randn(B, T, C, D, generator=g, device="cuda").to(cfg.dtype)
    return x


def _both_lookups(lk, ss, w, p, r, A, k, gv, gs):
    """Values, masks and the two payload gradients (each on its own) of one implementation."""
    p = p.detach().clone().requires_grad_(True)
    vals, mask = lk(w, p, r, address_space=A, k=k)
    sums, smask = ss(w, p, r, address_space=A)
    glk = torch.autograd.grad(vals, p, gv.to(p.dtype), retain_graph=True)[0]
    gss = torch.autograd.grad(sums, p, gs.to(p.dtype))[0]
    return vals.detach(), mask, sums.detach(), smask, glk, gss


def _compare_config(ref, cfg, seed):
    from ravel_lm_b200 import causal_last_k_lookup, causal_sum_lookup
    mem, tl1 = ref
    x = _inputs(cfg, seed)
    w, r, p, A, k = x["write"], x["read"], x["payload"], cfg.A, cfg.k
    ov, om, os_, osm, oglk, ogss = _both_lookups(causal_last_k_lookup, causal_sum_lookup, w, p, r, A, k,
                                                 x["g_vals"], x["g_sums"])
    with _torch_path(tl1), torch.no_grad():
        rv, rm = mem.causal_last_k_lookup(w, p, r, address_space=A, k=k)
    _assert_bits(ov, rv, f"cfg{cfg.cfg} latest-k values vs the reference's torch path")
    assert torch.equal(om, rm), f"cfg{cfg.cfg} latest-k mask"
    del rv, rm
    # sums and gradients: the reference on float64 payloads
    with _torch_path(tl1):
        rv64, rm64, rs64, rsm64, rglk64, rgss64 = _both_lookups(mem.causal_last_k_lookup, mem.causal_sum_lookup, w,
                                                                p.double(), r, A, k, x["g_vals"], x["g_sums"])
    assert torch.equal(om, rm64) and torch.equal(osm, rsm64), f"cfg{cfg.cfg} masks (float64 run)"
    tol = SUM_TOL[p.dtype]
    _assert_close(os_, rs64, tol, f"cfg{cfg.cfg} sums")
    _assert_close(oglk, rglk64, tol, f"cfg{cfg.cfg} latest-k payload gradient")
    _assert_close(ogss, rgss64, tol, f"cfg{cfg.cfg} sum payload gradient")
    return x, ov, om


@pytest.mark.parametrize("c", [1, 2, 5])
def test_fp32_configs_against_the_reference(ref, c):
    """Configurations 1, 2 and the op shapes of 5 (learned read heads: reads differ from writes), fp32."""
    from ravel_lm_b200.workloads import CONFIGS
    cfg = CONFIGS[c]
    x, ov, om = _compare_config(ref, cfg, seed=31000 + c)
    if c == 1:
        mem, tl1 = ref
        assert tl1.can_use_triton_latest1_v2(x["write"], x["payload"], x["read"], address_space=cfg.A, k=cfg.k,
                                             write_mask=None)
        with torch.no_grad():
            tv, tm = mem.causal_last_k_lookup(x["write"], x["payload"], x["read"], address_space=cfg.A, k=cfg.k)
        assert torch.equal(tm, om), "cfg1 mask vs the reference's Triton v2 kernel"
        assert torch.equal(tv, ov), "cfg1 values vs the reference's Triton v2 kernel"


def test_config3_full_against_the_reference(ref):
    """Configuration 3 at full size (B4 T32768 H16 D64 bf16, k = 8, Zipf(1.05) over 65536)."""
    from ravel_lm_b200.workloads import CONFIGS
    _compare_config(ref, CONFIGS[3], seed=33003)
    torch.cuda.empty_cache()


def test_masked_general_reads_against_the_reference(ref):
    """Reads apart from the writes plus a write mask, int32 addresses with negatives, bf16, k = 3."""
    from ravel_lm_b200 import causal_last_k_lookup, causal_sum_lookup
    mem, tl1 = ref
    g = torch.Generator(device="cuda").manual_seed(909)
    B, T, C, D, A, k = 3, 3000, 5, 24, 700, 3
    w = torch.randint(-2 * A, 2 * A, (B, T, C), generator=g, device="cuda", dtype=torch.int32)
    r = torch.randint(-2 * A, 2 * A, (B, T, C), generator=g, device="cuda", dtype=torch.int32)
    m = torch.rand(B, T, generator=g, device="cuda") < 0.7
    p = torch.randn(B, T, C, D, generator=g, device="cuda").to(torch.bfloat16)
    gv = torch.randn(B, T, C, k, D, generator=g, device="cuda")
    gs = torch.randn(B, T, C, D, generator=g, device="cuda")
    pp = p.clone().requires_grad_(True)
    ov, om = causal_last_k_lookup(w, pp, r, address_space=A, k=k, write_mask=m)
    os_, osm = causal_sum_lookup(w, pp, r, address_space=A, write_mask=m)
    oglk = torch.autograd.grad(ov, pp, gv.to(p.dtype), retain_graph=True)[0]
    ogss = torch.autograd.grad(os_, pp, gs.to(p.dtype))[0]
    rv, rm = mem.causal_last_k_lookup(w, p, r, address_space=A, k=k, write_mask=m)
    _assert_bits(ov.detach(), rv, "latest-k values")
    assert torch.equal(om, rm)
    p64 = p.double().requires_grad_(True)
    rv64, _ = mem.causal_last_k_lookup(w, p64, r, address_space=A, k=k, write_mask=m)
    rs64, rsm = mem.causal_sum_lookup(w, p64, r, address_space=A, write_mask=m)
    rglk = torch.autograd.grad(rv64, p64, gv.double(), retain_graph=True)[0]
    rgss = torch.autograd.grad(rs64, p64, gs.double())[0]
    assert torch.equal(osm, rsm)
    _assert_close(os_, rs64, SUM_TOL[torch.bfloat16], "sums")
    _assert_close(oglk, rglk, SUM_TOL[torch.bfloat16], "latest-k gradient")
    _assert_close(ogss, rgss, SUM_TOL[torch.bfloat16], "sum gradient")


@pytest.mark.parametrize("independent", [False, True])
def test_config4_decode_against_the_reference(ref, independent):
    """Configuration 4: prefill by 4096 writes, then 1024 steps of read then write per head.

    ``independent`` draws the read addresses apart from the write addresses (the
    learned heads of ``model.py:406-424``); otherwise a step reads and writes the
    same address (literal heads).  Our prefill runs both token by token and in
    bulk (``RavelLayerCache.prefill``); our steps use the one-launch ``step``.
    """
    from ravel_lm_b200 import RavelLayerCache
    from ravel_lm_b200.workloads import DECODE
    mem, _ = ref
    S, H, A, D, dt, P, steps = (DECODE[k] for k in ("streams", "H", "A", "D", "dtype", "prefill", "steps"))
    g = torch.Generator(device="cuda").manual_seed(4444 + independent)
    pa = torch.randint(0, A, (S, P, H), generator=g, device="cuda")
    pp = torch.randn(S, P, H, D, generator=g, device="cuda").to(dt)
    rc = mem.RavelLayerCache.empty(S, H, A, D, device="cuda", dtype=dt)
    oc = RavelLayerCache.empty(S, H, A, D, device="cuda", dtype=dt)
    bulk = RavelLayerCache.empty(S, H, A, D, device="cuda", dtype=dt)
    for t in range(P):
        rc.write(pa[:, t], pp[:, t])
        oc.write(pa[:, t], pp[:, t])
    bulk.prefill(pa, pp)
    for c in (oc, bulk):
        assert torch.equal(c.filled, rc.filled)
        _assert_bits(c.values, rc.values, "prefilled cache")
    del pa, pp, bulk
    wa = torch.randint(-5, A + 5, (steps, S, H), generator=g, device="cuda")  # clamped, as in the reference
    ra = torch.randint(-5, A + 5, (steps, S, H), generator=g, device="cuda") if independent else wa
    pay = torch.randn(steps, S, H, D, generator=g, device="cuda").to(dt)
    out_o = torch.empty(steps, S, H, D, device="cuda", dtype=dt)
    out_r = torch.empty_like(out_o)
    mask_o = torch.empty(steps, S, H, device="cuda", dtype=torch.bool)
    mask_r = torch.empty_like(mask_o)
    for i in range(steps):
        v, m = rc.read(ra[i])
        rc.write(wa[i], pay[i])
        out_r[i], mask_r[i] = v, m
        v, m = oc.step(ra[i], wa[i], pay[i])
        out_o[i], mask_o[i] = v, m
    assert torch.equal(mask_o, mask_r)
    _assert_bits(out_o, out_r, "decode reads")
    assert torch.equal(oc.filled, rc.filled)
    _assert_bits(oc.values, rc.values, "cache after the decode steps")


def test_torch_compile_fullgraph_matches_eager(ref):
    """Both lookups under torch.compile(fullgraph=True) (the custom ops with their fake
    and autograd registrations), forward and backward, bit for bit equal to eager."""
    from ravel_lm_b200 import causal_last_k_lookup, causal_sum_lookup
    from ravel_lm_b200.ravel_memory import clear_tape_cache
    g = torch.Generator(device="cuda").manual_seed(77)
    B, T, C, D, A, k = 2, 4096, 4, 32, 300, 3
    w = torch.randint(0, A, (B, T, C), generator=g, device="cuda")
    r = torch.randint(0, A, (B, T, C), generator=g, device="cuda")
    m = torch.rand(B, T, generator=g, device="cuda") < 0.8
    p0 = torch.randn(B, T, C, D, generator=g, device="cuda")
    gv = torch.randn(B, T, C, k, D, generator=g, device="cuda")
    gs = torch.randn(B, T, C, D, generator=g, device="cuda")

    def f(w, p, r, m):
        vals, mask = causal_last_k_lookup(w, p, r, address_space=A, k=k, write_mask=m)
        sums, smask = causal_sum_lookup(w, p, r, address_space=A, write_mask=m)
        return vals, mask, sums, smask

    results = []
    for fn in (f, torch.compile(f, fullgraph=True)):
        for reads in (None, r):
            clear_tape_cache()
            p = p0.clone().requires_grad_(True)
            vals, mask, sums, smask = fn(w, p, reads, m)
            # each lookup's gradient on its own (two backward passes), then both in one pass;
            # the compiled graph adds the two gradients with one elementwise add, as eager
            # autograd does when they come from separate passes
            g_lk = torch.autograd.grad(vals, p, gv, retain_graph=True)[0]
            g_ss = torch.autograd.grad(sums, p, gs, retain_graph=True)[0]
            torch.autograd.backward([vals, sums], [gv, gs])
            results.append((vals.detach(), mask, sums.detach(), smask, g_lk, g_ss, g_lk + g_ss, p.grad))
    names = ("values", "mask", "sums", "sum mask", "latest-k gradient", "sum gradient", "summed gradients")
    for eager, compiled in zip(results[:2], results[2:]):
        for a, b, what in zip(eager, compiled, names):
            _assert_bits(b, a, f"compiled {what}")
        _assert_bits(compiled[7], eager[6], "compiled one-pass gradient vs the eager sum of the two")
        # eager's one pass adds the latest-k gradient inside its kernel: one rounding fewer
        _assert_close(eager[7], eager[6], 1e-6, "eager one-pass gradient")
