"""Gate residual and RMSNorm kernels against the torch expressions they replace.

``gate_residual`` must equal ``x + torch.sigmoid(gate) * fused`` and its
autograd bit for bit (float32 and bfloat16, vector and scalar paths);
``rms_norm`` must match ``torch.nn.functional.rms_norm`` within float32
rounding (1e-5 relative; bf16 1e-2), and its weight gradient must be
bit-identical from run to run.
"""
from __future__ import annotations

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


def _bits_equal(a, b):
    v = {2: torch.int16, 4: torch.int32}[a.element_size()]
    return torch.equal(a.contiguous().view(v), b.contiguous().view(v))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("shape", [(4, 1024, 256), (3, 7, 5), (1, 1, 1)])
def test_gate_residual_equals_torch_bit_for_bit(dtype, shape):
    from ravel_lm_b200.glue import gate_residual
    g = torch.Generator(device="cuda").manual_seed(sum(shape))
    x, gl, f = (torch.randn(*shape, generator=g, device="cuda").mul(3).to(dtype).requires_grad_(True)
                for _ in range(3))
    gy = torch.randn(*shape, generator=g, device="cuda").to(dtype)
    out = gate_residual(x, gl, f)
    ref = x + torch.sigmoid(gl) * f
    assert _bits_equal(out, ref), "forward"
    got = torch.autograd.grad(out, [x, gl, f], gy)
    want = torch.autograd.grad(ref, [x, gl, f], gy)
    for a, b, what in zip(got, want, ("d x", "d gate", "d fused")):
        assert _bits_equal(a, b), what


@pytest.mark.parametrize("dtype,tol", [(torch.float32, 1e-5), (torch.bfloat16, 1e-2)])
@pytest.mark.parametrize("shape", [(4, 1024, 256), (5, 33, 68), (2, 3, 4096)])
def test_rms_norm_matches_torch(dtype, tol, shape):
    from ravel_lm_b200.glue import rms_norm
    g = torch.Generator(device="cuda").manual_seed(shape[-1])
    x = torch.randn(*shape, generator=g, device="cuda").to(dtype).requires_grad_(True)
    w = (1 + 0.1 * torch.randn(shape[-1], generator=g, device="cuda")).to(dtype).requires_grad_(True)
    gy = torch.randn(*shape, generator=g, device="cuda").to(dtype)
    y = rms_norm(x, w, 1e-6)
    dx, dw = torch.autograd.grad(y, [x, w], gy)
    x64, w64 = x.detach().double().requires_grad_(True), w.detach().double().requires_grad_(True)
    y64 = torch.nn.functional.rms_norm(x64, (shape[-1],), w64, 1e-6)
    dx64, dw64 = torch.autograd.grad(y64, [x64, w64], gy.double())
    for a, b, what in ((y, y64, "y"), (dx, dx64, "dx"), (dw, dw64, "dw")):
        err = (a.double() - b).abs().max().item()
        assert err <= tol * max(b.abs().max().item(), 1e-30), f"{what}: {err}"
    # deterministic weight gradient
    dw2 = torch.autograd.grad(rms_norm(x, w, 1e-6), [w], gy)[0]
    assert _bits_equal(dw, dw2)


def test_glue_rejects_what_it_does_not_cover():
    from ravel_lm_b200.glue import gate_residual, rms_norm
    x = torch.randn(2, 3, device="cuda", dtype=torch.float64)
    with pytest.raises(TypeError):
        gate_residual(x, x, x)
    with pytest.raises(ValueError):
        gate_residual(x.float(), x.float()[:, :2], x.float())
    with pytest.raises(ValueError):
        rms_norm(torch.randn(2, 8192, device="cuda"), torch.ones(8192, device="cuda"), 1e-6)
