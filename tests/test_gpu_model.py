"""The reference's own RAVEL language model with this operator dropped in.

``ravel_lm/model.py`` takes the three names of the operator from
``.ravel_memory`` (``model.py:11``).  These tests import the stock model from
the installed reference under ``baseline/_ref`` (skipped when absent), rebind
those three names in ``ravel_lm.model`` to this package -- the one-line import
change a maintainer makes -- and compare the model against itself with the
stock operator on the same weights and tokens:

* float64, six layers at the widths of benchmark configuration 5 (vocab 1024,
  d_model 256, 4 literal + 4 learned heads, 2 x 32 product codes, A = 1024,
  payload 32, last_k = 2, sum read): logits, loss and every parameter gradient
  within 1e-9 (float64 makes the learned argmax addresses of later layers
  identical in both runs);
* float32, six layers, latest-k only: logits bit for bit equal (the reference's
  CUDA glue is used unchanged in both runs), gradients within 1e-4; the same
  with this package's ``gate_residual`` kernel in place of ``model.py:12``'s;
* float32, one layer with the sum read at B = 4, T = 1024: logits and gradients
  within float32 tolerance (the reference's glue runs IEEE float32 dots here in
  both runs, not its default TF32);
* decode (float64): ``forward_step`` over a prompt equals the full forward
  (the reference's ``tests/test_model.py:78-91``) and equals the stock model's
  ``forward_step`` bit for bit; ``generate`` (float32) with greedy sampling
  gives the same tokens.
"""
from __future__ import annotations

import contextlib
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
REF = ROOT / "baseline" / "_ref"
NAMES = ("causal_last_k_lookup", "causal_sum_lookup", "RavelLayerCache")


@pytest.fixture(scope="module")
def ref():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    if not (REF / "ravel_lm" / "model.py").exists():
        pytest.skip("no installed reference under baseline/_ref")
    if str(REF) not in sys.path:
        sys.path.insert(0, str(REF))
    import triton
    # The reference's CUDA glue multiplies float32 with Triton dots, TF32 by default.
    # TF32 rounds the GEMM inputs to 10 mantissa bits, which turns last-bit
    # differences of the operator's float32 sums into 1e-3 relative differences
    # downstream; both runs of every comparison use IEEE float32 dots instead.
    old_fp32 = triton.knobs.language.fp32_default
    triton.knobs.language.fp32_default = "ieee"
    import ravel_lm.config as config
    import ravel_lm.deferred as deferred
    import ravel_lm.model as model
    import ravel_lm_b200._lib as L
    L.load()
    yield model, config.RavelConfig, deferred
    triton.knobs.language.fp32_default = old_fp32
    torch.cuda.synchronize()
    assert L.device_error(torch.cuda.current_stream().cuda_stream) == 0


@contextlib.contextmanager
def ours(model_mod, glue=False):
    """``from ravel_lm_b200.ravel_memory import ...`` in place of ``model.py:11`` (and, with
    ``glue``, ``gate_residual`` from ``ravel_lm_b200.glue`` in place of ``model.py:12``'s)."""
    import ravel_lm_b200.glue as glue_mod
    import ravel_lm_b200.ravel_memory as mine
    from ravel_lm_b200.ravel_memory import clear_tape_cache
    names = NAMES + (("gate_residual",) if glue else ())
    saved = {n: getattr(model_mod, n) for n in names}
    for n in names:
        setattr(model_mod, n, getattr(glue_mod if n == "gate_residual" else mine, n))
    clear_tape_cache()
    try:
        yield
    finally:
        for n, v in saved.items():
            setattr(model_mod, n, v)
        clear_tape_cache()


def cfg5(RavelConfig, **kw):
    base = dict(vocab_size=1024, block_size=1024, d_model=256, n_layers=6, address_space=1024, n_literal_heads=4,
                n_learned_heads=4, n_codebooks=2, codebook_size=32, payload_dim=32, last_k=2, use_sum_read=True,
                memory_every=1, dropout=0.0)
    base.update(kw)
    return RavelConfig(**base)


def _tokens(B, T, vocab, seed):
    from ravel_lm_b200.workloads import zipf_ranks
    g = torch.Generator(device="cuda").manual_seed(seed)
    return zipf_ranks(vocab, 1.1, (B, T), g), zipf_ranks(vocab, 1.1, (B, T), g)


def _step(model, deferred, x, y):
    """Forward + backward; returns logits, loss and {name: grad}."""
    model.zero_grad(set_to_none=True)
    out = model(x, y)
    out["loss"].backward()
    deferred.flush_deferred()
    grads = {n: p.grad.detach().clone() for n, p in model.named_parameters() if p.grad is not None}
    return out["logits"].detach(), out["loss"].detach(), grads


def _close(a, b, tol, what):
    a, b = a.double(), b.double()
    scale = float(b.abs().max()) if b.numel() else 0.0
    err = float((a - b).abs().max()) if b.numel() else 0.0
    assert err <= tol * max(scale, 1e-30), f"{what}: max abs err {err:.3g} vs tol {tol} * {scale:.3g}"


def _compare(model_mod, model, deferred, x, y, tol_logits, tol_grads, exact_logits=False, glue=False):
    ref_logits, ref_loss, ref_grads = _step(model, deferred, x, y)
    with ours(model_mod, glue=glue):
        logits, loss, grads = _step(model, deferred, x, y)
    if exact_logits:
        assert torch.equal(logits, ref_logits), "logits differ bitwise"
    else:
        _close(logits, ref_logits, tol_logits, "logits")
    _close(loss, ref_loss, tol_logits, "loss")
    assert grads.keys() == ref_grads.keys()
    memory_grads = 0
    for n, g in ref_grads.items():
        _close(grads[n], g, tol_grads, f"grad of {n}")
        memory_grads += ".memory.payload." in n and bool(g.abs().max() > 0)
    assert memory_grads == model.cfg.n_layers, "every memory layer's payload projection gets a gradient"


def test_config5_model_float64_fwd_bwd(ref):
    model_mod, RavelConfig, deferred = ref
    torch.manual_seed(0)
    model = model_mod.RavelLM(cfg5(RavelConfig)).cuda().double()
    x, y = _tokens(2, 512, 1024, seed=5)
    _compare(model_mod, model, deferred, x, y, 1e-9, 1e-9)


@pytest.mark.parametrize("glue", [False, True], ids=["operator", "operator+gate_residual"])
def test_config5_model_float32_latest_k(ref, glue):
    model_mod, RavelConfig, deferred = ref
    torch.manual_seed(1)
    model = model_mod.RavelLM(cfg5(RavelConfig, use_sum_read=False)).cuda()
    x, y = _tokens(4, 1024, 1024, seed=6)
    _compare(model_mod, model, deferred, x, y, 0.0, 1e-4, exact_logits=True, glue=glue)


def test_config5_layer_float32_with_sum_read(ref):
    model_mod, RavelConfig, deferred = ref
    torch.manual_seed(2)
    model = model_mod.RavelLM(cfg5(RavelConfig, n_layers=1)).cuda()
    x, y = _tokens(4, 1024, 1024, seed=7)
    _compare(model_mod, model, deferred, x, y, 1e-4, 1e-3)


def test_decode_equals_prefill_and_stock_decode(ref):
    """forward_step supports last_k = 1 without the sum read (model.py:402-403)."""
    model_mod, RavelConfig, _ = ref
    torch.manual_seed(123)
    cfg = cfg5(RavelConfig, n_layers=3, last_k=1, use_sum_read=False, block_size=256)
    # float64: the full forward's CUDA GEMMs in float32 are Triton dots in TF32, the
    # step's are cuBLAS float32, so only float64 leaves the two paths comparable
    model = model_mod.RavelLM(cfg).cuda().double().eval()
    x, _ = _tokens(4, 96, 1024, seed=8)
    with torch.no_grad():
        stock_steps = []
        cache = model.init_cache(batch_size=4, device="cuda", dtype=torch.float64)
        for t in range(x.shape[1]):
            stock_steps.append(model.forward_step(x[:, t], cache))
        with ours(model_mod):
            full = model(x)["logits"]
            cache = model.init_cache(batch_size=4, device="cuda", dtype=torch.float64)
            import ravel_lm_b200
            assert isinstance(cache.block_caches[0].memory_cache, ravel_lm_b200.RavelLayerCache)
            steps = [model.forward_step(x[:, t], cache) for t in range(x.shape[1])]
    stepped, stock = torch.stack(steps, 1), torch.stack(stock_steps, 1)
    assert torch.equal(stepped, stock), "decode logits differ from the stock cache's"
    # the reference's own tolerance for decode == prefill (tests/test_model.py:91)
    assert torch.allclose(full, stepped, atol=1e-5, rtol=1e-4)


def test_generate_greedy_matches_stock(ref):
    model_mod, RavelConfig, _ = ref
    torch.manual_seed(9)
    cfg = cfg5(RavelConfig, n_layers=2, last_k=1, use_sum_read=False, block_size=128)
    model = model_mod.RavelLM(cfg).cuda().eval()
    prompt, _ = _tokens(2, 12, 1024, seed=9)
    stock = model.generate(prompt, max_new_tokens=16, temperature=0.0, use_cache=True)
    with ours(model_mod):
        mine = model.generate(prompt, max_new_tokens=16, temperature=0.0, use_cache=True)
    assert torch.equal(mine, stock)


@contextlib.contextmanager
def fused_layers(model_mod, model):
    """Every memory layer's forward replaced by ravel_lm_b200.layer.memory_layer_forward."""
    import types

    from ravel_lm_b200.layer import memory_layer_forward
    layers = [b.memory for b in model.blocks if b.memory is not None]
    with ours(model_mod):
        for layer in layers:
            layer.forward = types.MethodType(memory_layer_forward, layer)
        try:
            yield
        finally:
            for layer in layers:
                del layer.forward


@pytest.mark.parametrize("n_layers,literal,learned", [(1, 4, 4), (3, 8, 0)])
def test_fused_memory_layer_forward(ref, n_layers, literal, learned):
    """The layer's read-out on the tensor cores (TF32, as the reference's own CUDA fast_linear):
    logits and gradients within TF32 tolerance of the stock layer.  One layer with learned
    heads (their addresses come from the embeddings, identical in both runs), or literal heads
    only (addresses from the tokens), so that no learned argmax sees the TF32 differences."""
    model_mod, RavelConfig, deferred = ref
    torch.manual_seed(4)
    cfg = cfg5(RavelConfig, n_layers=n_layers, n_literal_heads=literal, n_learned_heads=learned)
    model = model_mod.RavelLM(cfg).cuda()
    x, y = _tokens(4, 1024, 1024, seed=12)
    ref_logits, ref_loss, ref_grads = _step(model, deferred, x, y)
    with fused_layers(model_mod, model):
        logits, loss, grads = _step(model, deferred, x, y)
    _close(logits, ref_logits, 1e-2, "logits")
    _close(loss, ref_loss, 1e-3, "loss")
    for n, g in ref_grads.items():
        _close(grads[n], g, 3e-2, f"grad of {n}")
