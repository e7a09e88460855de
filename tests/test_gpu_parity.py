"""CUDA path vs the reference: golden vectors and the CPU oracle.

Every test calls the public drop-in API (which runs ``libravel_b200.so``
through its C ABI) on ``cuda:0`` and checks it against either the committed
golden outputs of the reference itself or the C oracle on identical seeded
inputs.
"""
from __future__ import annotations

import zlib

import numpy as np
import pytest
import torch

from conftest import golden_cases, load_golden, payload_as_float64, payload_code
from gpu_helpers import SUM_TOL, assert_bits_equal, assert_close, payload_np, to_f64

pytestmark = pytest.mark.gpu

DT = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16, "float64": torch.float64}


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import ravel_lm_b200._lib as L
    L.load()
    yield
    torch.cuda.synchronize()
    assert L.device_error(torch.cuda.current_stream().cuda_stream) == 0


def _payload_tensor(case) -> torch.Tensor:
    p = case["payload"]
    dt = DT[str(case["dtype"])]
    if dt == torch.bfloat16:
        return torch.from_numpy(p.view(np.int16).copy()).view(torch.bfloat16)
    if dt == torch.float16:
        return torch.from_numpy(p.view(np.int16).copy()).view(torch.float16)
    return torch.from_numpy(p.copy())


def _run(w, p, r, m, A, k, g_lk, g_ss, dev="cuda"):
    from ravel_lm_b200 import causal_last_k_lookup, causal_sum_lookup
    pw = p.to(dev).requires_grad_(True)
    wd = w.to(dev)
    rd = None if r is None else r.to(dev)
    md = None if m is None else m.to(dev)
    vals, mask = causal_last_k_lookup(wd, pw, rd, address_space=A, k=k, write_mask=md)
    sums, smask = causal_sum_lookup(wd, pw, rd, address_space=A, write_mask=md)
    glk = torch.autograd.grad(vals, pw, g_lk.to(dev).to(p.dtype), retain_graph=True, allow_unused=True)[0]
    gss = torch.autograd.grad(sums, pw, g_ss.to(dev).to(p.dtype), allow_unused=True)[0]
    torch.cuda.synchronize()
    return vals, mask, sums, smask, glk, gss


@pytest.mark.parametrize("name", golden_cases())
def test_golden_vectors(name):
    """Reference outputs on its own known-answer and seeded cases."""
    case = load_golden(name)
    A, k = int(case["A"]), int(case["k"])
    w = torch.from_numpy(case["waddr"])
    r = torch.from_numpy(case["raddr"]) if "raddr" in case else None
    m = torch.from_numpy(case["wmask"]).bool() if "wmask" in case else None
    p = _payload_tensor(case)
    vals, mask, sums, smask, glk, gss = _run(w, p, r, m, A, k, torch.from_numpy(case["g_lk"]),
                                             torch.from_numpy(case["g_ss"]))
    assert_bits_equal(vals, case["lk_vals"], f"{name} latest-k values")
    assert np.array_equal(mask.cpu().numpy(), case["lk_mask"].astype(bool)), f"{name} latest-k mask"
    assert np.array_equal(smask.cpu().numpy(), case["ss_mask"].astype(bool)), f"{name} sum mask"
    tol = SUM_TOL[p.dtype]
    assert_close(to_f64(sums), case["ss_sums64"], tol, f"{name} sums")
    if glk is not None:
        assert_close(to_f64(glk), case["lk_grad64"], tol, f"{name} latest-k grad")
    if gss is not None:
        assert_close(to_f64(gss), case["ss_grad64"], tol, f"{name} sum grad")


def _oracle_check(oracle, w, p, r, m, A, k, g_lk, g_ss, *, check_grads=True):
    vals, mask, sums, smask, glk, gss = _run(w, p, r, m, A, k, g_lk, g_ss)
    code = {torch.bfloat16: "bf16", torch.float16: "f16"}.get(p.dtype)
    wn = w.numpy()
    rn = None if r is None else r.numpy()
    mn = None if m is None else m.numpy()
    ov, om, osrc, tape = oracle.latestk_fwd(wn, payload_np(p), rn, address_space=A, k=k, write_mask=mn, dtype=code)
    assert_bits_equal(vals, ov.view({2: np.uint16, 4: np.uint32, 8: np.uint64}[ov.dtype.itemsize]), "values")
    assert np.array_equal(mask.cpu().numpy(), om), "latest-k mask"
    p64 = to_f64(p)
    osum, osm, _ = oracle.segsum_fwd(wn, p64, rn, address_space=A, write_mask=mn, tape=tape)
    assert np.array_equal(smask.cpu().numpy(), osm), "sum mask"
    tol = SUM_TOL[p.dtype]
    assert_close(to_f64(sums), osum, tol, "sums")
    if check_grads:
        B, T, C, D = p.shape
        olk = oracle.latestk_bwd(om, osrc, to_f64(g_lk), B * T * C).reshape(B, T, C, D)
        oss = oracle.segsum_bwd(tape, osm, to_f64(g_ss))
        assert_close(to_f64(glk), olk, tol, "latest-k grad")
        assert_close(to_f64(gss), oss, tol, "sum grad")


CASES = [
    # name, B, T, C, D, A, k, dtype, reads, mask, address dist
    ("cfg1", 8, 256, 4, 16, 256, 1, torch.float32, False, False, "zipf1.1"),
    ("cfg2_fast", 16, 2048, 8, 32, 4096, 4, torch.float32, False, False, "product"),
    ("multitile_bf16", 1, 20000, 3, 64, 65536, 8, torch.bfloat16, False, False, "zipf1.05"),
    ("long_t32k_bf16", 1, 32768, 2, 64, 65536, 8, torch.bfloat16, False, False, "zipf1.05"),
    ("hot_segments", 2, 9000, 2, 16, 3, 6, torch.float32, False, False, "uniform"),
    ("general_reads", 4, 700, 5, 24, 97, 3, torch.float32, True, False, "uniform"),
    ("general_mask", 3, 1500, 4, 8, 40, 2, torch.float32, True, True, "uniform"),
    ("mask_aliased", 3, 900, 3, 16, 30, 4, torch.bfloat16, False, True, "uniform"),
    ("general_long_multitile", 1, 17000, 2, 32, 500, 3, torch.float32, True, True, "uniform"),
    ("odd_d_f16", 2, 300, 3, 5, 11, 3, torch.float16, True, False, "uniform"),
    ("f64_fast", 2, 513, 3, 7, 17, 2, torch.float64, False, False, "uniform"),
    ("d1_k_gt_t", 3, 5, 2, 1, 3, 8, torch.float32, False, False, "uniform"),
    ("key64", 2, 4096, 2, 8, 2**31, 2, torch.float32, False, False, "huge"),
    ("key64_general", 2, 3000, 2, 8, 2**31, 2, torch.float32, True, True, "huge"),
    ("wide_d300_fallback", 2, 700, 2, 300, 60, 2, torch.float32, True, True, "uniform"),
    ("d33_fallback_bf16", 2, 900, 3, 33, 70, 3, torch.bfloat16, False, False, "uniform"),
    ("d256_bf16_el8", 1, 3000, 2, 256, 90, 2, torch.bfloat16, False, False, "uniform"),
    ("d128_f32_el4", 1, 2500, 2, 128, 40, 2, torch.float32, True, False, "uniform"),
    ("d48_f64_el2", 1, 1700, 2, 48, 30, 2, torch.float64, False, True, "uniform"),
    ("general_bf16_d64_vec", 2, 3000, 4, 64, 500, 4, torch.bfloat16, True, True, "zipf1.05"),
    ("general_f16_d32_vec", 2, 2000, 3, 32, 300, 3, torch.float16, True, False, "uniform"),
    # a mask keeping 3% of the positions: the bucket starts past the last valid write fill
    # most of each stream's tail
    ("general_sparse_mask", 2, 33000, 2, 16, 300, 3, torch.float32, True, 0.03, "uniform"),
    # 1 KB rows: the range scan's two-vectors-per-lane form (payload rows, or float accumulator rows
    # of the general path)
    ("d256_f32_1kb_rows", 1, 3000, 2, 256, 50, 2, torch.float32, False, False, "uniform"),
    ("d512_bf16_1kb_rows_mask", 1, 1200, 2, 512, 30, 2, torch.bfloat16, False, True, "uniform"),
    ("d128_f64_1kb_general", 1, 1500, 2, 128, 40, 2, torch.float64, True, True, "uniform"),
    ("d256_bf16_general_acc_1kb", 1, 2000, 2, 256, 60, 2, torch.bfloat16, True, False, "uniform"),
    # short streams of 128-byte rows: the one-CTA-per-stream scan (aliased and merged, masks,
    # 16-bit and 64-bit keys, a single step)
    ("short_general_mask_f32", 3, 1500, 4, 32, 40, 3, torch.float32, True, True, "uniform"),
    ("short_aliased_bf16", 2, 1800, 3, 64, 50, 2, torch.bfloat16, False, False, "zipf1.05"),
    ("short_aliased_mask_bf16", 2, 1800, 3, 64, 50, 2, torch.bfloat16, False, True, "uniform"),
    ("short_general_f16_d64", 2, 1000, 3, 64, 30, 2, torch.float16, True, False, "uniform"),
    ("short_key64_general_mask", 2, 1500, 2, 32, 2**31, 2, torch.float32, True, True, "huge"),
    ("short_t1_f32", 4, 1, 3, 32, 5, 2, torch.float32, True, False, "uniform"),
    ("short_t4096_aliased_f32", 1, 4096, 2, 32, 300, 2, torch.float32, False, False, "uniform"),
]


def _gen_addresses(gen, dist, shape, A):
    if dist.startswith("zipf"):
        from ravel_lm_b200.workloads import zipf_ranks
        return zipf_ranks(A, float(dist[4:]), shape, gen)
    if dist == "product":
        return torch.randint(0, 64, shape, generator=gen) * 64 + torch.randint(0, 64, shape, generator=gen)
    if dist == "huge":
        pool = torch.randint(0, 2**31 - 1, (64,), generator=gen)
        return pool[torch.randint(0, 64, shape, generator=gen)]
    return torch.randint(-A, 2 * A, shape, generator=gen)


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_seeded_vs_oracle(oracle_mod, case):
    name, B, T, C, D, A, k, dt, reads, mask, dist = case
    gen = torch.Generator().manual_seed(zlib.crc32(name.encode()))
    w = _gen_addresses(gen, dist, (B, T, C), A)
    r = _gen_addresses(gen, dist, (B, T, C), A) if reads else None
    m = (torch.rand(B, T, generator=gen) < (0.7 if mask is True else mask)) if mask else None
    if m is not None and B > 1:
        m[1] = False  # an all-masked batch row: empty streams inside the tape
    p = torch.randn(B, T, C, D, generator=gen).to(dt)
    g_lk = torch.randn(B, T, C, k, D, generator=gen).to(dt)
    g_ss = torch.randn(B, T, C, D, generator=gen).to(dt)
    _oracle_check(oracle_mod, w, p, r, m, A, k, g_lk, g_ss)


def test_int32_addresses_match_int64(oracle_mod):
    gen = torch.Generator().manual_seed(5)
    w = torch.randint(-50, 50, (2, 400, 3), generator=gen)
    r = torch.randint(-50, 50, (2, 400, 3), generator=gen)
    p = torch.randn(2, 400, 3, 8, generator=gen)
    g1 = torch.randn(2, 400, 3, 2, 8, generator=gen)
    g2 = torch.randn(2, 400, 3, 8, generator=gen)
    a = _run(w, p, r, None, 37, 2, g1, g2)
    b = _run(w.int(), p, r.int(), None, 37, 2, g1, g2)
    for x, y in zip(a[:4], b[:4]):
        assert torch.equal(x, y)
    for x, y in zip(a[4:], b[4:]):  # the backward is deterministic: same keys, same bits
        assert torch.equal(x, y)


@pytest.mark.parametrize("D,dt", [(5, torch.float16), (300, torch.float32), (256, torch.float32), (33, torch.bfloat16)])
def test_general_backward_bits_repeat_for_any_row_shape(D, dt):
    """Rows that are not 2^m <= 32 vectors take the element-wise gathers: two runs, same bits."""
    gen = torch.Generator().manual_seed(D)
    B, T, C, A, k = 2, 700, 3, 23, 3
    w = torch.randint(-A, 2 * A, (B, T, C), generator=gen)
    r = torch.randint(-A, 2 * A, (B, T, C), generator=gen)
    m = torch.rand(B, T, generator=gen) < 0.7
    p = torch.randn(B, T, C, D, generator=gen).to(dt)
    g1 = torch.randn(B, T, C, k, D, generator=gen)
    g2 = torch.randn(B, T, C, D, generator=gen)
    a = _run(w, p, r, m, A, k, g1, g2)
    b = _run(w, p, r, m, A, k, g1, g2)
    for x, y in zip(a[4:], b[4:]):
        assert torch.equal(x.view(torch.uint8), y.view(torch.uint8))


def test_model_config5_op_shapes(oracle_mod):
    """Config 5 (literal + learned heads, read != write) at its per-GPU size."""
    from ravel_lm_b200.workloads import CONFIGS, make_inputs
    cfg = CONFIGS[5]
    x = make_inputs(cfg)
    _oracle_check(oracle_mod, x["write"], x["payload"], x["read"], None, cfg.A, cfg.k, x["g_vals"], x["g_sums"])


def test_config2_full(oracle_mod):
    from ravel_lm_b200.workloads import CONFIGS, make_inputs
    cfg = CONFIGS[2]
    x = make_inputs(cfg)
    _oracle_check(oracle_mod, x["write"], x["payload"], None, None, cfg.A, cfg.k, x["g_vals"], x["g_sums"])


def test_config3_full(oracle_mod):
    """The long-context configuration at full size (B4 T32768 H16 D64 bf16 k8)."""
    from ravel_lm_b200.workloads import CONFIGS, make_inputs
    cfg = CONFIGS[3]
    x = make_inputs(cfg)
    _oracle_check(oracle_mod, x["write"], x["payload"], None, None, cfg.A, cfg.k, x["g_vals"], x["g_sums"])


@pytest.mark.parametrize("T,A,mask", [(256, 256, False), (300, 50, False), (20000, 65536, False),
                                      (1500, 40, True), (5, 3, False), (65536, 4096, False),
                                      (70000, 1000, True), (16385, 2**20, True)])
def test_tape_sort_order(oracle_mod, T, A, mask):
    """The per-stream sorted keys of the tape equal the reference's sort order."""
    import ravel_lm_b200.ravel_memory as rm
    gen = torch.Generator().manual_seed(T + A)
    B, C = 2, 3
    w = torch.randint(-A, 2 * A, (B, T, C), generator=gen)
    m = (torch.rand(B, T, generator=gen) < 0.6) if mask else None
    p = torch.randn(B, T, C, 4, generator=gen)
    _, _, tape = rm._latestk_fwd(w.cuda(), p.cuda(), None, None if m is None else m.cuda(), A, 1)
    torch.cuda.synchronize()
    ot = oracle_mod.Tape(w.numpy(), None, None if m is None else m.numpy(), A)
    tbits = max(1, (T - 1).bit_length())
    abits = (A - 1).bit_length()
    key64 = tbits + abits + (1 if mask else 0) > 32
    keys = tape.cpu().numpy().view(np.uint64 if key64 else np.uint32)[: B * C * T].reshape(B * C, T)
    # oracle: global sorted keys -> per-stream (addr, t)
    sk = ot.sorted_keys[: ot.nw]
    base = sk // (T + 1)
    stream = base // A
    addr = base % A
    t = sk % (T + 1)
    pos = 0
    for s in range(B * C):
        n = int((stream == s).sum())
        got = keys[s, :n].astype(np.int64)
        exp = (addr[pos:pos + n].astype(np.int64) << tbits) | t[pos:pos + n]
        assert np.array_equal(got, exp), f"stream {s}: sorted keys differ at {np.argwhere(got != exp)[:5].ravel()}"
        pos += n


def test_tape_cache_reuse_and_invalidation():
    """causal_sum_lookup after causal_last_k_lookup on the same tensors reuses the
    sorted tape; an in-place change of the addresses must not."""
    import ravel_lm_b200.ravel_memory as rm
    from ravel_lm_b200 import causal_last_k_lookup, causal_sum_lookup
    g = torch.Generator().manual_seed(21)
    B, T, C, D, A = 2, 3000, 3, 16, 50
    w = torch.randint(0, A, (B, T, C), generator=g).cuda()
    p = torch.randn(B, T, C, D, generator=g).cuda()
    rm.clear_tape_cache()
    causal_last_k_lookup(w, p, address_space=A, k=2)
    hit = rm._tape_cache.get(w, None, None, A, torch.cuda.current_stream().cuda_stream)
    assert hit is not None
    s_cached, m_cached = causal_sum_lookup(w, p, address_space=A)
    rm.clear_tape_cache()
    s_fresh, m_fresh = causal_sum_lookup(w, p, address_space=A)
    assert torch.equal(s_cached, s_fresh) and torch.equal(m_cached, m_fresh)
    # in-place edit after the latest-k call: the sum must see the new addresses
    causal_last_k_lookup(w, p, address_space=A, k=2)
    w[:, ::2] = (w[:, ::2] + 7) % A
    assert rm._tape_cache.get(w, None, None, A, torch.cuda.current_stream().cuda_stream) is None
    s_new, _ = causal_sum_lookup(w, p, address_space=A)
    rm.clear_tape_cache()
    s_ref, _ = causal_sum_lookup(w, p, address_space=A)
    assert torch.equal(s_new, s_ref)
    assert not torch.equal(s_new, s_fresh)


SPECIAL_BITS = {
    # +Inf, -Inf, quiet NaN, NaN with payload and sign, -0, +0, smallest subnormal, -subnormal, max finite
    torch.bfloat16: [0x7F80, 0xFF80, 0x7FC0, 0xFFA1, 0x8000, 0x0000, 0x0001, 0x8001, 0x7F7F],
    torch.float16: [0x7C00, 0xFC00, 0x7E00, 0xFE01, 0x8000, 0x0000, 0x0001, 0x8001, 0x7BFF],
    torch.float32: [0x7F800000, 0xFF800000, 0x7FC00000, 0xFFC12345, 0x80000000, 0x0, 0x1, 0x80000001, 0x7F7FFFFF],
    torch.float64: [0x7FF0000000000000, 0xFFF0000000000000, 0x7FF8000000000000, 0xFFF8000000000ABC,
                    0x8000000000000000, 0x0, 0x1, 0x8000000000000001, 0x7FEFFFFFFFFFFFFF],
}

NONFINITE_CASES = [
    # name, B, T, C, D, k, dtype, reads (each case lands on a different output loop of the fast kernel)
    ("bf16_d64_k8", 2, 600, 3, 64, 8, torch.bfloat16, False),
    ("f16_d16_k4", 2, 500, 3, 16, 4, torch.float16, False),
    ("f32_d64_k4", 2, 400, 2, 64, 4, torch.float32, False),
    ("f32_d32_k4", 2, 400, 2, 32, 4, torch.float32, False),
    ("f64_d32_k4", 1, 300, 2, 32, 4, torch.float64, False),
    ("bf16_d24_k16", 1, 700, 2, 24, 16, torch.bfloat16, False),
    ("bf16_d64_k8_general", 2, 500, 3, 64, 8, torch.bfloat16, True),
]


@pytest.mark.parametrize("case", NONFINITE_CASES, ids=[c[0] for c in NONFINITE_CASES])
def test_latestk_nonfinite_payload_bits(oracle_mod, case):
    """Invalid slots hold candidate * 0: +-0 for finite candidates (sign kept) and the canonical
    quiet NaN for Inf/NaN; valid slots copy the candidate's bits, NaN payloads included."""
    from ravel_lm_b200 import causal_last_k_lookup
    name, B, T, C, D, k, dt, reads = case
    gen = torch.Generator().manual_seed(zlib.crc32(name.encode()))
    A = 37
    w = torch.randint(0, A, (B, T, C), generator=gen)
    r = torch.randint(0, A, (B, T, C), generator=gen) if reads else None
    p = torch.randn(B, T, C, D, generator=gen).to(dt)
    ibits = {2: torch.int16, 4: torch.int32, 8: torch.int64}[p.element_size()]
    bits = p.view(ibits)
    width = 8 * p.element_size()
    signed = [v - 2 ** width if v >= 2 ** (width - 1) else v for v in SPECIAL_BITS[dt]]
    special = torch.tensor(signed, dtype=ibits)
    pick = torch.rand(bits.shape, generator=gen) < 0.15
    choice = special[torch.randint(0, len(special), bits.shape, generator=gen)]
    bits[pick] = choice[pick]
    vals, mask = causal_last_k_lookup(w.cuda(), p.cuda(), None if r is None else r.cuda(), address_space=A, k=k)
    torch.cuda.synchronize()
    code = {torch.bfloat16: "bf16", torch.float16: "f16"}.get(dt)
    ov, om, _, _ = oracle_mod.latestk_fwd(w.numpy(), payload_np(p), None if r is None else r.numpy(),
                                          address_space=A, k=k, dtype=code)
    assert np.array_equal(mask.cpu().numpy(), om), "latest-k mask"
    assert_bits_equal(vals, ov.view({2: np.uint16, 4: np.uint32, 8: np.uint64}[ov.dtype.itemsize]), name)
    assert (~om).any() and om.any(), "the case must hold both valid and invalid slots"


@pytest.mark.parametrize("general", [False, True], ids=["aliased", "general_mask"])
def test_training_step_captured_in_cuda_graph(general):
    """Forward and backward of both lookups captured once in a CUDA graph, then replayed on new
    inputs copied into the captured buffers: bit-identical to the eager step on those inputs."""
    from ravel_lm_b200 import causal_last_k_lookup, causal_sum_lookup
    g = torch.Generator().manual_seed(33 + int(general))
    B, T, C, D, A, k = 2, 2048, 4, 32, 300, 3

    def fresh():
        w = torch.randint(0, A, (B, T, C), generator=g)
        r = torch.randint(0, A, (B, T, C), generator=g) if general else None
        m = (torch.rand(B, T, generator=g) < 0.8) if general else None
        p = torch.randn(B, T, C, D, generator=g).to(torch.bfloat16)
        gv = torch.randn(B, T, C, k, D, generator=g).to(torch.bfloat16)
        gs = torch.randn(B, T, C, D, generator=g).to(torch.bfloat16)
        return [w, r, m, p, gv, gs]

    def step(w, r, m, p, gv, gs):
        vals, vm = causal_last_k_lookup(w, p, r, address_space=A, k=k, write_mask=m)
        sums, sm = causal_sum_lookup(w, p, r, address_space=A, write_mask=m)
        (gp,) = torch.autograd.grad([vals, sums], [p], [gv, gs])
        return vals, vm, sums, sm, gp

    static = [None if t is None else t.cuda() for t in fresh()]
    static[3].requires_grad_(True)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(2):
            step(*static)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        captured = step(*static)
    for _ in range(2):
        new = fresh()
        with torch.no_grad():
            for dst, src in zip(static, new):
                if dst is not None:
                    dst.copy_(src.cuda())
        graph.replay()
        torch.cuda.synchronize()
        eager_in = [None if t is None else t.cuda() for t in new]
        eager_in[3].requires_grad_(True)
        eager = step(*eager_in)
        torch.cuda.synchronize()
        for name, a, b in zip(("values", "mask", "sums", "sum mask", "payload grad"), captured, eager):
            assert torch.equal(a.view(torch.uint8) if a.dtype != torch.bool else a,
                               b.view(torch.uint8) if b.dtype != torch.bool else b), name
    del graph
