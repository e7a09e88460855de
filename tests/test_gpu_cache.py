"""Decode cache (RavelLayerCache) on the GPU vs the reference and vs prefill."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_golden
from gpu_helpers import assert_bits_equal

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    yield
    import ravel_lm_b200._lib as L
    torch.cuda.synchronize()
    assert L.device_error(torch.cuda.current_stream().cuda_stream) == 0


def test_cache_sequence_golden():
    """Reference read/write sequence with out-of-range addresses (clamped)."""
    from ravel_lm_b200 import RavelLayerCache
    z = load_golden("cache_sequence")
    B, C, A, D = (int(z[x]) for x in ("B", "C", "A", "D"))
    cache = RavelLayerCache.empty(B, C, A, D, device="cuda", dtype=torch.float32)
    for s in range(z["raddr"].shape[0]):
        v, m = cache.read(torch.from_numpy(z["raddr"][s]).cuda())
        assert_bits_equal(v, z["vals"][s].view(np.uint32), f"read {s}")
        assert np.array_equal(m.cpu().numpy(), z["mask"][s].astype(bool))
        cache.write(torch.from_numpy(z["waddr"][s]).cuda(), torch.from_numpy(z["payload"][s]).cuda())
    assert np.array_equal(cache.values.cpu().numpy(), z["final_values"])
    assert np.array_equal(cache.filled.cpu().numpy(), z["final_filled"].astype(bool))


def test_kat_write_then_read():
    """tests/test_memory.py:70-79 of the reference."""
    from ravel_lm_b200 import RavelLayerCache
    cache = RavelLayerCache.empty(1, 2, 16, 3, device="cuda", dtype=torch.float32)
    addrs = torch.tensor([[5, 7]], device="cuda")
    _, mask = cache.read(addrs)
    assert not mask.any()
    payload = torch.tensor([[[1.0, 2.0, 3.0], [4.0, 5.0, 6.0]]], device="cuda")
    cache.write(addrs, payload)
    vals, mask = cache.read(addrs)
    assert mask.all()
    assert torch.equal(vals, payload)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32, torch.float16, torch.float64])
def test_step_equals_read_then_write(oracle_mod, dtype):
    from ravel_lm_b200 import RavelLayerCache
    g = torch.Generator().manual_seed(11)
    B, C, A, D = 5, 4, 64, 12
    c1 = RavelLayerCache.empty(B, C, A, D, device="cuda", dtype=dtype)
    c2 = RavelLayerCache.empty(B, C, A, D, device="cuda", dtype=dtype)
    vals_np = np.zeros((B, C, A, D), np.float64)
    filled_np = np.zeros((B, C, A), bool)
    for _ in range(40):
        ra = torch.randint(-4, A + 4, (B, C), generator=g)
        wa = torch.randint(-4, A + 4, (B, C), generator=g)
        p = torch.randn(B, C, D, generator=g).to(dtype)
        v1, m1 = c1.read(ra.cuda())
        c1.write(wa.cuda(), p.cuda())
        v2, m2 = c2.step(ra.cuda(), wa.cuda(), p.cuda())
        assert torch.equal(v1, v2) and torch.equal(m1, m2)
        ov, om = oracle_mod.cache_read(vals_np, filled_np, ra.numpy())
        assert np.array_equal(m1.cpu().numpy(), om)
        assert np.array_equal(v1.double().cpu().numpy(), ov)
        oracle_mod.cache_write(vals_np, filled_np, wa.numpy(), p.double().numpy())
    assert torch.equal(c1.values, c2.values) and torch.equal(c1.filled, c2.filled)


def test_decode_matches_prefill_latest1():
    """Token-by-token cache steps == latest-1 prefill over the same tape
    (the property behind tests/test_model.py:78-91 of the reference)."""
    from ravel_lm_b200 import RavelLayerCache, causal_last_k_lookup
    g = torch.Generator().manual_seed(3)
    B, T, C, A, D = 6, 300, 4, 50, 16
    addr = torch.randint(0, A, (B, T, C), generator=g).cuda()
    pay = torch.randn(B, T, C, D, generator=g).to(torch.bfloat16).cuda()
    vals, mask = causal_last_k_lookup(addr, pay, address_space=A, k=1)
    cache = RavelLayerCache.empty(B, C, A, D, device="cuda", dtype=torch.bfloat16)
    for t in range(T):
        v, m = cache.step(addr[:, t], addr[:, t], pay[:, t])
        assert torch.equal(m, mask[:, t, :, 0])
        assert torch.equal(v, vals[:, t, :, 0])  # value equality (+0 == -0)


def test_decode_cuda_graph_replay():
    """Steps captured once in a CUDA graph and replayed give the eager result."""
    from ravel_lm_b200 import RavelLayerCache
    g = torch.Generator().manual_seed(9)
    S, H, A, D, steps = 16, 4, 128, 64, 12
    ra = torch.randint(0, A, (steps, S, H), generator=g).cuda()
    wa = torch.randint(0, A, (steps, S, H), generator=g).cuda()
    pay = torch.randn(steps, S, H, D, generator=g).to(torch.bfloat16).cuda()
    eager = RavelLayerCache.empty(S, H, A, D, device="cuda", dtype=torch.bfloat16)
    ev = [eager.step(ra[i], wa[i], pay[i]) for i in range(steps)]
    graphed = RavelLayerCache.empty(S, H, A, D, device="cuda", dtype=torch.bfloat16)
    outs = []
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(graph, stream=stream):
            for i in range(steps):
                outs.append(graphed.step(ra[i], wa[i], pay[i]))
    torch.cuda.current_stream().wait_stream(stream)
    graphed.values.zero_()
    graphed.filled.zero_()
    graph.replay()
    torch.cuda.synchronize()
    for (v1, m1), (v2, m2) in zip(ev, outs):
        assert torch.equal(v1, v2) and torch.equal(m1, m2)
    assert torch.equal(eager.values, graphed.values)
    del graph


PREFILL_CASES = [
    # name, B, T, C, A, D, dtype, address dtype, address range (lo, hi)
    ("bf16_clamped", 3, 500, 4, 64, 16, torch.bfloat16, torch.int64, (-8, 72)),
    ("f32_one_tile", 2, 4096, 3, 4096, 8, torch.float32, torch.int32, (0, 4096)),
    ("f16_cluster", 1, 20000, 2, 300, 24, torch.float16, torch.int64, (-5, 310)),
    ("f64_merge", 1, 70000, 2, 1000, 4, torch.float64, torch.int64, (0, 1000)),
    ("bf16_hot", 2, 9000, 2, 5, 64, torch.bfloat16, torch.int64, (0, 5)),
]


@pytest.mark.parametrize("case", PREFILL_CASES, ids=[c[0] for c in PREFILL_CASES])
def test_bulk_prefill_equals_token_by_token_writes(oracle_mod, case):
    """RavelLayerCache.prefill leaves the state of T sequential writes (ravel_lm/model.py:600-602 prefill),
    bit for bit, on a cache that already holds data; checked against the oracle on the smallest case."""
    from ravel_lm_b200 import RavelLayerCache
    name, B, T, C, A, D, dtype, adt, (lo, hi) = case
    g = torch.Generator().manual_seed(len(name) * 1009 + T)
    addr = torch.randint(lo, hi, (B, T, C), generator=g).to(adt)
    pay = torch.randn(B, T, C, D, generator=g).to(dtype)
    prior_v = torch.randn(B, C, A, D, generator=g).to(dtype)
    prior_f = torch.rand(B, C, A, generator=g) < 0.3
    bulk = RavelLayerCache(prior_v.clone().cuda(), prior_f.clone().cuda())
    bulk.prefill(addr.cuda(), pay.cuda())
    seq = RavelLayerCache(prior_v.clone().cuda(), prior_f.clone().cuda())
    ad, pd = addr.cuda(), pay.cuda()
    for t in range(T):
        seq.write(ad[:, t], pd[:, t])
    torch.cuda.synchronize()
    assert torch.equal(bulk.filled, seq.filled), name
    assert torch.equal(bulk.values.view(torch.uint8), seq.values.view(torch.uint8)), name
    if B * T * C <= 6000:
        vals_np = prior_v.double().numpy().copy()
        filled_np = prior_f.numpy().copy()
        for t in range(T):
            oracle_mod.cache_write(vals_np, filled_np, addr[:, t].numpy(), pay[:, t].double().numpy())
        assert np.array_equal(bulk.filled.cpu().numpy(), filled_np)
        assert np.array_equal(bulk.values.double().cpu().numpy(), vals_np)


def test_bulk_prefill_then_decode_matches_latest1():
    """Prefill in bulk, then decode step by step: every read equals latest-1 over the whole tape."""
    from ravel_lm_b200 import RavelLayerCache, causal_last_k_lookup
    g = torch.Generator().manual_seed(21)
    B, T0, T1, C, A, D = 4, 700, 60, 3, 40, 32
    addr = torch.randint(0, A, (B, T0 + T1, C), generator=g).cuda()
    pay = torch.randn(B, T0 + T1, C, D, generator=g).to(torch.bfloat16).cuda()
    vals, mask = causal_last_k_lookup(addr, pay, address_space=A, k=1)
    cache = RavelLayerCache.empty(B, C, A, D, device="cuda", dtype=torch.bfloat16)
    cache.prefill(addr[:, :T0], pay[:, :T0])
    for t in range(T0, T0 + T1):
        v, m = cache.step(addr[:, t], addr[:, t], pay[:, t])
        assert torch.equal(m, mask[:, t, :, 0])
        assert torch.equal(v, vals[:, t, :, 0])


def test_step_into_reused_outputs():
    """``step(..., out=...)`` writes the read into the given buffers, equal to a fresh step."""
    import torch
    from ravel_lm_b200 import RavelLayerCache
    g = torch.Generator(device="cuda").manual_seed(12)
    B, C, A, D = 3, 4, 50, 8
    c1 = RavelLayerCache.empty(B, C, A, D, device="cuda", dtype=torch.float32)
    c2 = RavelLayerCache.empty(B, C, A, D, device="cuda", dtype=torch.float32)
    buf = (torch.empty(B, C, D, device="cuda"), torch.empty(B, C, dtype=torch.bool, device="cuda"))
    for _ in range(20):
        ra = torch.randint(0, A, (B, C), generator=g, device="cuda")
        wa = torch.randint(0, A, (B, C), generator=g, device="cuda")
        p = torch.randn(B, C, D, generator=g, device="cuda")
        v1, m1 = c1.step(ra, wa, p)
        v2, m2 = c2.step(ra, wa, p, out=buf)
        assert v2 is buf[0] and m2 is buf[1]
        assert torch.equal(v1, v2) and torch.equal(m1, m2)
    with pytest.raises(ValueError):
        c2.step(ra, wa, p, out=(buf[0][:, :2], buf[1]))
