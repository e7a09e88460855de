"""The memory layer's glue around the operator, on the same CUDA library.

Drop-ins for two functions ``ravel_lm/model.py`` imports from
``ravel_lm/triton_block.py`` (``model.py:12``):

* ``gate_residual(x, gate_lin, fused) = x + sigmoid(gate_lin) * fused``
  (``triton_block.py:383-387``, called at ``model.py:388``): one kernel each way
  instead of three torch kernels forward and several backward; equal bit for
  bit to the torch expression in float32 and bfloat16;
* ``rms_norm(x, g, eps)`` (``triton_block.py:320-323``, used by every
  ``RMSNorm`` module, ``model.py:31-39``): one warp per row forward, a
  deterministic backward (no atomics).

Both take CUDA tensors of float32 or bfloat16 (``rms_norm``: last dimension
up to 4096) and raise on anything else; there is no CPU path.
"""
from __future__ import annotations

import torch

from . import _lib
from .ravel_memory import _require_cuda, _stream

Tensor = torch.Tensor
_CODES = {torch.float32: _lib.RAVEL_F32, torch.bfloat16: _lib.RAVEL_BF16}


def _code(t: Tensor) -> int:
    try:
        return _CODES[t.dtype]
    except KeyError:
        raise TypeError(f"glue kernels take float32 or bfloat16 tensors, got {t.dtype}") from None


class _GateResidualFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, gate_lin, fused):
        dev = _require_cuda(x, gate_lin, fused)
        xc, gc, fc = x.contiguous(), gate_lin.contiguous(), fused.contiguous()
        out = torch.empty_like(xc)
        _lib.call("ravel_gate_residual_fwd", xc.data_ptr(), gc.data_ptr(), fc.data_ptr(), out.data_ptr(),
                  out.numel(), _code(xc), _stream(dev))
        ctx.save_for_backward(gc, fc)
        return out

    @staticmethod
    def backward(ctx, gy):
        gc, fc = ctx.saved_tensors
        gyc = gy.contiguous()
        dgate, dfused = torch.empty_like(gc), torch.empty_like(fc)
        _lib.call("ravel_gate_residual_bwd", gc.data_ptr(), fc.data_ptr(), gyc.data_ptr(), dgate.data_ptr(),
                  dfused.data_ptr(), gc.numel(), _code(gc), _stream(gc.device))
        return gy, dgate, dfused


def gate_residual(x: Tensor, gate_lin: Tensor, fused: Tensor) -> Tensor:
    """x + sigmoid(gate_lin) * fused (ravel_lm/triton_block.py:383-387), one kernel each way."""
    if not (x.shape == gate_lin.shape == fused.shape and x.dtype == gate_lin.dtype == fused.dtype):
        raise ValueError("gate_residual expects x, gate_lin and fused of one shape and dtype")
    _code(x)
    return _GateResidualFn.apply(x, gate_lin, fused)


class _RMSNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, g, eps):
        dev = _require_cuda(x, g)
        K = x.shape[-1]
        x2 = x.reshape(-1, K).contiguous()
        gc = g.contiguous()
        y = torch.empty_like(x2)
        rstd = torch.empty(x2.shape[0], dtype=torch.float32, device=dev)
        _lib.call("ravel_rms_norm_fwd", x2.data_ptr(), gc.data_ptr(), float(eps), y.data_ptr(), rstd.data_ptr(),
                  x2.shape[0], K, _code(x2), _stream(dev))
        ctx.save_for_backward(x2, gc, rstd)
        ctx.shape = x.shape
        return y.view(x.shape)

    @staticmethod
    def backward(ctx, gy):
        x2, gc, rstd = ctx.saved_tensors
        M, K = x2.shape
        gy2 = gy.reshape(M, K).contiguous()
        dx = torch.empty_like(x2)
        dg = torch.empty_like(gc)
        scratch = torch.empty(int(_lib.load().ravel_rms_norm_scratch_bytes(M, K)), dtype=torch.uint8,
                              device=x2.device)
        _lib.call("ravel_rms_norm_bwd", x2.data_ptr(), gc.data_ptr(), gy2.data_ptr(), rstd.data_ptr(), dx.data_ptr(),
                  dg.data_ptr(), M, K, _code(x2), scratch.data_ptr(), scratch.numel(), _stream(x2.device))
        return dx.view(ctx.shape), dg, None


def rms_norm(x: Tensor, g: Tensor, eps: float) -> Tensor:
    """RMSNorm over the last dimension (ravel_lm/triton_block.py:320-323)."""
    if g.dim() != 1 or g.shape[0] != x.shape[-1] or g.dtype != x.dtype:
        raise ValueError("rms_norm expects a weight of shape [x.shape[-1]] and x's dtype")
    _code(x)
    return _RMSNormFn.apply(x, g, float(eps))


__all__ = ["gate_residual", "rms_norm"]
