"""A memory layer's read-out in one tensor-core kernel.

``RavelMemoryLayer.forward`` (``ravel_lm/model.py:367-388``) reads its memory and
projects the result::

    values, _ = causal_last_k_lookup(write, payload, read, address_space=A, k=k)
    sums, _ = causal_sum_lookup(write, payload, read, address_space=A)      # use_sum_read
    fused = fast_linear(torch.cat([values.reshape(B, T, -1), sums.reshape(B, T, -1)], -1), fuse.weight)
    out = gate_residual(x, gate_lin, fused)

``memory_read_linear`` computes ``fused`` (or ``out``) with the latest-k gather
inside the GEMM: a tcgen05 kernel (TF32 inputs, float32 accumulation -- the
precision of the reference's Triton ``fast_linear`` on CUDA) gathers each tile
of the read rows from the payload rows the latest-k tape names, so the
[B, T, C, k, D] values and the concatenated rows are never written.  The
backward gathers the rows once more and uses cuBLAS for the two weight/input
GEMMs, then this package's latest-k and sum backward kernels (one payload
gradient buffer).  float32 payloads and weights, D a multiple of 4.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _lib
from .ravel_memory import (_build_tape, _latestk_bwd_impl, _payload_code, _require_cuda, _segsum_bwd_impl,
                           _segsum_fwd_impl, _stream, _TokenTape, _aliases)

Tensor = torch.Tensor


def _sources(tape, raddr, flags, B, T, C, A, k, device) -> Tensor:
    src = torch.empty(B * T * C, k, dtype=torch.int32, device=device)
    r = raddr if raddr is not None else torch.empty(0, dtype=torch.int32, device=device)
    code = _lib.RAVEL_I64 if r.dtype == torch.int64 else _lib.RAVEL_I32
    _lib.call("ravel_latestk_sources", tape.data_ptr(), flags, r.data_ptr() if flags else None, code, B, T, C, A, k,
              src.data_ptr(), _stream(device))
    return src


class _ReadLinearFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, write, payload, read, write_mask, weight, x, gate, address_space, k, use_sum, prebuilt):
        device = _require_cuda(write, payload, read, write_mask, weight, x, gate)
        B, T, C = write.shape if prebuilt is None else prebuilt.shape
        D = payload.shape[-1]
        N = weight.shape[0]
        p = payload.contiguous()
        w = weight.contiguous()
        if prebuilt is None:
            tape, _scratch, r, _code, flags = _build_tape(write, read, write_mask, address_space, D, k,
                                                         _payload_code(p), device)
        else:
            tape, r, flags = prebuilt.tape, prebuilt.raddr, prebuilt.flags
        src = _sources(tape, r, flags, B, T, C, address_space, k, device)
        sums = None
        if use_sum:
            sums, _smask, _t = _segsum_fwd_impl(write, p, read, write_mask, address_space, prebuilt)
        out = torch.empty(B, T, N, dtype=torch.float32, device=device)
        # A W^T before the gate is kept only for the gate's gradient
        pre = torch.empty_like(out) if (x is not None and ctx.needs_input_grad[6]) else None
        xc = x.contiguous() if x is not None else None
        gc = gate.contiguous() if gate is not None else None
        _lib.call("ravel_gather_gemm", p.data_ptr(), src.data_ptr(), None if sums is None else sums.data_ptr(),
                  B, T, C, D, k, w.data_ptr(), N, None if xc is None else xc.data_ptr(),
                  None if gc is None else gc.data_ptr(), out.data_ptr(), None if pre is None else pre.data_ptr(),
                  _stream(device))
        ctx.save_for_backward(tape, r, p, src, sums, w, pre, gc)
        ctx.meta = (flags, B, T, C, D, N, int(address_space), int(k), bool(use_sum), x is not None)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        tape, r, p, src, sums, w, pre, gate = ctx.saved_tensors
        flags, B, T, C, D, N, A, k, use_sum, gated = ctx.meta
        device = grad_out.device
        st = _stream(device)
        gy = grad_out.contiguous()
        g_x = g_gate = None
        if gated:
            g_pre = torch.empty_like(pre)
            g_gate = torch.empty_like(gate)
            _lib.call("ravel_gate_residual_bwd", gate.data_ptr(), pre.data_ptr(), gy.data_ptr(), g_gate.data_ptr(),
                      g_pre.data_ptr(), pre.numel(), _lib.RAVEL_F32, st)
            g_x = grad_out
        else:
            g_pre = gy
        K = C * k * D + (C * D if use_sum else 0)
        rows = torch.empty(B * T, K, dtype=torch.float32, device=device)
        _lib.call("ravel_gather_rows", p.data_ptr(), src.data_ptr(), None if sums is None else sums.data_ptr(),
                  B, T, C, D, k, rows.data_ptr(), st)
        g2 = g_pre.reshape(B * T, N)
        g_w = torch.mm(g2.t(), rows) if ctx.needs_input_grad[4] else None
        g_p = None
        if ctx.needs_input_grad[1]:
            g_rows = torch.mm(g2, w)
            g_vals = g_rows[:, :C * k * D].reshape(B, T, C, k, D).contiguous()
            raddr = r if r.numel() else torch.empty(0, dtype=torch.int32, device=device)
            if use_sum:
                g_sums = g_rows[:, C * k * D:].reshape(B, T, C, D).contiguous()
                g_p = _segsum_bwd_impl(tape, g_sums, raddr, flags, B, T, C, A)
                _latestk_bwd_impl(tape, g_vals, raddr, flags, B, T, C, A, k, accumulate_into=g_p)
            else:
                g_p = _latestk_bwd_impl(tape, g_vals, raddr, flags, B, T, C, A, k)
        return None, g_p, None, None, g_w, g_x, g_gate, None, None, None, None


def memory_read_linear(write_addresses: Tensor, payloads: Tensor, read_addresses: Optional[Tensor], weight: Tensor,
                       *, address_space: int, k: int = 1, use_sum_read: bool = False,
                       write_mask: Optional[Tensor] = None, x: Optional[Tensor] = None,
                       gate_lin: Optional[Tensor] = None) -> Tensor:
    """``fuse(cat(latest-k values, sums))`` of a memory layer (ravel_lm/model.py:367-386), or with
    ``x`` and ``gate_lin`` the layer's output ``x + sigmoid(gate_lin) * fuse(...)`` (:388).

    Args:
        write_addresses, read_addresses, write_mask, address_space, k: as for
            ``causal_last_k_lookup``.
        payloads: [B, T, C, D] float32, D a multiple of 4.
        weight:   [N, C*k*D (+ C*D with use_sum_read)] float32 (``fuse.weight``).
        x, gate_lin: optional [B, T, N] float32 for the gate residual.
    Returns:
        [B, T, N] float32; differentiable w.r.t. payloads, weight, x and gate_lin.
    """
    if read_addresses is None:
        read_addresses = write_addresses
    B, T, C = write_addresses.shape
    D = payloads.shape[-1]
    if payloads.shape[:3] != (B, T, C) or read_addresses.shape != (B, T, C):
        raise ValueError("payloads leading dimensions must match addresses")
    if payloads.dtype != torch.float32 or weight.dtype != torch.float32:
        raise TypeError("memory_read_linear takes float32 payloads and weight")
    K = C * k * D + (C * D if use_sum_read else 0)
    if weight.ndim != 2 or weight.shape[1] != K:
        raise ValueError(f"weight must be [N, {K}]")
    if (x is None) != (gate_lin is None):
        raise ValueError("x and gate_lin go together")
    if x is not None and (x.shape != (B, T, weight.shape[0]) or gate_lin.shape != x.shape):
        raise ValueError("x and gate_lin must be [B, T, N]")
    if k <= 0:
        raise ValueError("k must be positive")
    if write_mask is not None and write_mask.shape != (B, T):
        raise ValueError("write_mask must have shape [B, T]")
    read = None if _aliases(read_addresses, write_addresses) else read_addresses
    return _ReadLinearFn.apply(write_addresses, payloads, read, write_mask, weight, x, gate_lin, int(address_space),
                               int(k), bool(use_sum_read), None)


def memory_read_linear_tokens(token_ids: Tensor, payloads: Tensor, learned_write: Optional[Tensor],
                              learned_read: Optional[Tensor], weight: Tensor, *, address_space: int,
                              n_literal_heads: int, bos_token_id: int, k: int = 1, use_sum_read: bool = False,
                              write_mask: Optional[Tensor] = None, x: Optional[Tensor] = None,
                              gate_lin: Optional[Tensor] = None) -> Tensor:
    """``memory_read_linear`` addressed from token ids, as ``memory_lookups`` is: the literal
    heads are hashed in the sort's key build (ravel_lm/model.py:195-231, :347-349)."""
    from .ravel_memory import scratch_bytes, tape_bytes
    B, T = token_ids.shape
    C, D = payloads.shape[2], payloads.shape[3]
    L = int(n_literal_heads)
    A = int(address_space)
    device = _require_cuda(token_ids, payloads, learned_write, learned_read, weight, write_mask)
    toks = token_ids.to(torch.int64).contiguous()
    lw = lr = None
    code = _lib.RAVEL_I64
    if learned_write is not None:
        lw = learned_write.to(torch.int64).contiguous()
        lr = lw if (learned_read is None or _aliases(learned_read, learned_write)) else \
            learned_read.to(torch.int64).contiguous()
    general = lr is not None and lr is not lw
    flags = (_lib.RAVEL_TAPE_GENERAL_READS if general else 0) | (_lib.RAVEL_TAPE_WRITE_MASK if write_mask is not None
                                                                else 0)
    m = None if write_mask is None else write_mask.to(torch.bool).contiguous()
    tape = torch.empty(tape_bytes(B, T, C, A, flags), dtype=torch.uint8, device=device)
    scratch = torch.empty(scratch_bytes(B, T, C, D, A, k, _payload_code(payloads), flags), dtype=torch.uint8,
                          device=device)
    raddr = torch.empty((B, T, C) if flags else (0,), dtype=torch.int32, device=device)
    _lib.call("ravel_tape_build_tokens", toks.data_ptr(), L, int(bos_token_id), None if lw is None else lw.data_ptr(),
              None if lr is None else lr.data_ptr(), code, None if m is None else m.data_ptr(), B, T, C, A, flags,
              raddr.data_ptr() if flags else None, tape.data_ptr(), tape.numel(), scratch.data_ptr(), scratch.numel(),
              _stream(device))
    pre = _TokenTape(tape, raddr, flags, (B, T, C))
    return _ReadLinearFn.apply(None, payloads, None, m, weight, x, gate_lin, A, int(k), bool(use_sum_read), pre)


__all__ = ["memory_read_linear", "memory_read_linear_tokens"]
