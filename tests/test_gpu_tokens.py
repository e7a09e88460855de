"""Memory-layer addresses from token ids: the literal hashes and the fused tape build.

* ``literal_addresses_from_tokens`` equals the reference's function of that name
  (``ravel_lm/model.py:195-231``, imported from ``baseline/_ref``) bit for bit,
  including token ids whose products overflow 64 bits and negative ids.
* ``memory_lookups`` (literal heads hashed inside the sort's key build) equals the
  composition it replaces -- literal hashes, ``torch.cat`` with the learned heads,
  ``causal_last_k_lookup`` and ``causal_sum_lookup`` -- bit for bit in values,
  masks, sums and the payload gradient, and the reference's own functions on the
  concatenated addresses for values and masks.
"""
from __future__ import annotations

import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

REF = Path(__file__).resolve().parents[1] / "baseline" / "_ref"


@pytest.fixture(scope="module")
def ref_model():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import ravel_lm_b200._lib as L
    L.load()
    if not (REF / "ravel_lm" / "model.py").exists():
        pytest.skip("no installed reference under baseline/_ref")
    if str(REF) not in sys.path:
        sys.path.insert(0, str(REF))
    import ravel_lm.model as model
    import ravel_lm.ravel_memory as mem
    yield model, mem
    torch.cuda.synchronize()
    assert L.device_error(torch.cuda.current_stream().cuda_stream) == 0


def _bits(t):
    return t.detach().view({2: torch.int16, 4: torch.int32, 8: torch.int64}[t.element_size()])


@pytest.mark.parametrize("n_heads", [0, 1, 2, 3, 4, 8])
@pytest.mark.parametrize("T", [1, 2, 3, 1000])
def test_literal_addresses_equal_the_reference(ref_model, n_heads, T):
    model, _ = ref_model
    from ravel_lm_b200 import literal_addresses_from_tokens
    if T == 1 and n_heads >= 3:
        pytest.skip("the reference's trigram head needs T >= 2 (its prev2 has two columns)")
    g = torch.Generator(device="cuda").manual_seed(T * 10 + n_heads)
    toks = torch.randint(0, 1024, (3, T), generator=g, device="cuda")
    toks[0, ::3] = torch.randint(-(1 << 62), 1 << 62, toks[0, ::3].shape, generator=g, device="cuda")  # wraps
    toks[1, ::5] = -toks[1, ::5] - 1
    for A, bos in ((1024, 257), (1000003, 0), (7, 5)):
        want = model.literal_addresses_from_tokens(toks, address_space=A, n_heads=n_heads, bos_token_id=bos)
        got = literal_addresses_from_tokens(toks, address_space=A, n_heads=n_heads, bos_token_id=bos)
        assert got.dtype == torch.int64 and torch.equal(got, want), (A, bos)


def _layer_case(B, T, L, Ll, D, A, seed, dtype, masked, separate_reads):
    g = torch.Generator(device="cuda").manual_seed(seed)
    toks = torch.randint(0, 300, (B, T), generator=g, device="cuda")
    lw = torch.randint(0, A, (B, T, Ll), generator=g, device="cuda") if Ll else None
    lr = torch.randint(0, A, (B, T, Ll), generator=g, device="cuda") if (Ll and separate_reads) else lw
    m = (torch.rand(B, T, generator=g, device="cuda") < 0.8) if masked else None
    p = torch.randn(B, T, L + Ll, D, generator=g, device="cuda").to(dtype)
    return toks, lw, lr, m, p


@pytest.mark.parametrize("L,Ll,separate_reads,masked", [(4, 4, True, False), (4, 4, True, True), (3, 0, False, False),
                                                        (2, 2, False, True), (0, 3, True, False)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_memory_lookups_equal_the_composition(ref_model, L, Ll, separate_reads, masked, dtype):
    model, mem = ref_model
    from ravel_lm_b200 import causal_last_k_lookup, causal_sum_lookup, literal_addresses_from_tokens, memory_lookups
    from ravel_lm_b200.ravel_memory import clear_tape_cache
    B, T, D, A, k, bos = 3, 1500, 16, 1024, 2, 257
    toks, lw, lr, m, p0 = _layer_case(B, T, L, Ll, D, A, seed=L * 7 + Ll, dtype=dtype, masked=masked,
                                      separate_reads=separate_reads)
    gv = torch.randn(B, T, L + Ll, k, D, device="cuda").to(dtype)
    gs = torch.randn(B, T, L + Ll, D, device="cuda").to(dtype)
    # fused
    clear_tape_cache()
    p = p0.clone().requires_grad_(True)
    v1, m1, s1, sm1 = memory_lookups(toks, p, lw, lr, address_space=A, n_literal_heads=L, bos_token_id=bos, k=k,
                                     use_sum_read=True, write_mask=m)
    torch.autograd.backward([v1, s1], [gv, gs])
    g1 = p.grad
    # composed (model.py:333-384 with this package's functions)
    clear_tape_cache()
    lit = literal_addresses_from_tokens(toks, address_space=A, n_heads=L, bos_token_id=bos)
    write = lit if lw is None else torch.cat([lit, lw], -1)
    read = write if lr is lw else torch.cat([lit, lr], -1)  # reads that alias writes stay one tensor
    p = p0.clone().requires_grad_(True)
    v2, m2 = causal_last_k_lookup(write, p, read, address_space=A, k=k, write_mask=m)
    s2, sm2 = causal_sum_lookup(write, p, read, address_space=A, write_mask=m)
    torch.autograd.backward([v2, s2], [gv, gs])
    for a, b, what in ((v1, v2, "values"), (s1, s2, "sums"), (g1, p.grad, "payload gradient")):
        assert torch.equal(_bits(a), _bits(b)), what
    assert torch.equal(m1, m2) and torch.equal(sm1, sm2)
    # the reference on the concatenated addresses
    ref_lit = model.literal_addresses_from_tokens(toks, address_space=A, n_heads=L, bos_token_id=bos)
    rw = ref_lit if lw is None else torch.cat([ref_lit, lw], -1)
    rr = ref_lit if lr is None else torch.cat([ref_lit, lr], -1)
    with torch.no_grad():
        rv, rm = mem.causal_last_k_lookup(rw, p0, rr, address_space=A, k=k, write_mask=m)
    assert torch.equal(_bits(v1), _bits(rv)) and torch.equal(m1, rm)


def test_memory_lookups_without_sums_and_argument_checks(ref_model):
    from ravel_lm_b200 import memory_lookups
    toks, lw, lr, m, p = _layer_case(2, 64, 2, 2, 8, 100, seed=1, dtype=torch.float32, masked=False,
                                     separate_reads=True)
    v, vm, s, sm = memory_lookups(toks, p, lw, lr, address_space=100, n_literal_heads=2, bos_token_id=0, k=3)
    assert v.shape == (2, 64, 4, 3, 8) and s is None and sm is None
    with pytest.raises(ValueError):
        memory_lookups(toks, p, None, None, address_space=100, n_literal_heads=2, bos_token_id=0)
    with pytest.raises(ValueError):
        memory_lookups(toks, p, lw[..., :1], lr, address_space=100, n_literal_heads=2, bos_token_id=0)
