"""Drop-in replacement of the reference's ``ravel_lm/ravel_memory.py`` on B200.

Same names, signatures, tensor layouts, return values and error behaviour as
the reference module (``ravel_lm/ravel_memory.py:16-292``):

* ``causal_last_k_lookup(write_addresses, payloads, read_addresses=None, *,
  address_space, k=1, write_mask=None) -> (values [B,T,C,k,D], mask [B,T,C,k])``
* ``causal_sum_lookup(write_addresses, payloads, read_addresses=None, *,
  address_space, write_mask=None) -> (sums [B,T,C,D], mask [B,T,C])``
* ``RavelLayerCache(values, filled)`` with ``empty``, ``read``, ``write``.

The computation runs in the CUDA library ``libravel_b200.so`` (C ABI in
``include/ravel_b200.h``), reached through ctypes.  In eager mode the two
lookups are ``torch.autograd.Function``s (the least host time per call); under
``torch.compile`` they are ``torch.library`` custom ops with fake (meta)
implementations and the same autograd formulas.  Both work under CUDA-graph
capture.  Tensors must live on a CUDA device: there is no CPU path and no
fallback.

Differences from the reference that a caller can observe:
* sums (and all gradients) accumulate in float32 (float64 for float64
  payloads) instead of the payload dtype, so bf16/fp16 sums are more accurate
  than the reference's own (which differ from the exact sum by ~10% at long T);
* an invalid slot of ``causal_sum_lookup`` is +0.0 (the reference's is
  ``segcum * 0`` and may be -0.0); latest-k invalid slots do match the
  reference's ``candidate * 0`` bit for bit;
* ``causal_sum_lookup`` also validates ``write_mask`` and ``read_addresses``
  shapes (ValueError) where the reference fails later or not at all.
"""
from __future__ import annotations

import functools
import weakref
from dataclasses import dataclass
from typing import Optional, Tuple

import torch

from . import _lib

Tensor = torch.Tensor

_PAYLOAD_CODES = {torch.float32: _lib.RAVEL_F32, torch.bfloat16: _lib.RAVEL_BF16,
                  torch.float16: _lib.RAVEL_F16, torch.float64: _lib.RAVEL_F64}
_SMALL_INTS = (torch.int8, torch.int16, torch.uint8)


# ------------------------------------------------------------------ helpers
def _composite_key_dtype(B: int, T: int, C: int, address_space: int) -> torch.dtype:
    """ravel_lm/ravel_memory.py:45-49: int32 keys iff B*C*A*(T+1) <= 2^31-1.

    The CUDA path sorts 32-bit per-stream keys regardless; this decides only
    the reference's int64 -> int32 address truncation, which is reproduced.
    """
    key_bound = int(B) * int(C) * int(address_space) * (int(T) + 1)
    return torch.int32 if key_bound <= torch.iinfo(torch.int32).max else torch.int64


def _addr(t: Tensor) -> Tuple[Tensor, int]:
    if t.dtype == torch.int64:
        return t.contiguous(), _lib.RAVEL_I64
    if t.dtype == torch.int32:
        return t.contiguous(), _lib.RAVEL_I32
    if t.dtype in _SMALL_INTS:
        return t.to(torch.int32).contiguous(), _lib.RAVEL_I32
    raise TypeError(f"addresses must be an integer tensor, got {t.dtype}")


def _payload_code(t: Tensor) -> int:
    try:
        return _PAYLOAD_CODES[t.dtype]
    except KeyError:
        raise TypeError(f"payloads must be float32, bfloat16, float16 or float64, got {t.dtype}") from None


def _stream(device: torch.device) -> int:
    """The raw handle of the current CUDA stream of ``device`` (no Stream object is built)."""
    return torch._C._cuda_getCurrentRawStream(device.index if device.index is not None else
                                              torch.cuda.current_device())


def _capturing() -> bool:
    """Whether the current CUDA stream is being captured into a graph (torch's own query)."""
    return torch._C._cuda_isCurrentStreamCapturing()


def _require_cuda(*tensors: Optional[Tensor]) -> torch.device:
    first = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError(
                f"ravel_lm_b200 runs on CUDA tensors only (got a {t.device.type} tensor); "
                "there is no CPU fallback")
        if first is None:
            first = t
        elif t.get_device() != first.get_device():
            raise RuntimeError(f"tensors are on different devices: {first.device} and {t.device}")
    return None if first is None else first.device


def _aliases(read: Optional[Tensor], write: Tensor) -> bool:
    """Reads that are the write tensor (or a view of the same elements) take the aliased path.

    Under torch.compile only identity is checked (data pointers are not
    traceable); a distinct tensor over the same memory then takes the general
    path, which gives the same results.
    """
    if read is None or read is write:
        return True
    if torch.compiler.is_compiling():
        return False
    if read.data_ptr() != write.data_ptr():  # the common case of distinct reads: one comparison
        return False
    return (read.dtype == write.dtype and read.shape == write.shape and read.stride() == write.stride()
            and read.device == write.device)


def _flags(read: Optional[Tensor], write_mask: Optional[Tensor]) -> int:
    f = 0
    if read is not None:
        f |= _lib.RAVEL_TAPE_GENERAL_READS
    if write_mask is not None:
        f |= _lib.RAVEL_TAPE_WRITE_MASK
    return f


def _ptr(t: Optional[Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _host():
    """The C++ host extension (per-step calls without ctypes); raises if it is not built."""
    return _lib._host or _lib.host()


@functools.lru_cache(maxsize=256)
def tape_bytes(B: int, T: int, C: int, A: int, flags: int) -> int:
    return int(_lib.load().ravel_tape_bytes(B, T, C, A, flags))


@functools.lru_cache(maxsize=256)
def scratch_bytes(B: int, T: int, C: int, D: int, A: int, k: int, dtype_code: int, flags: int) -> int:
    return int(_lib.load().ravel_scratch_bytes(B, T, C, D, A, k, dtype_code, flags))


class _TapeCache:
    """The last sorted tape, reused when the next lookup sees the same addresses.

    ``RavelMemoryLayer.forward`` calls ``causal_last_k_lookup`` and then
    ``causal_sum_lookup`` on the same address tensors; both sort the same
    write events.  The cache keeps the last tape and returns it when the write
    / read / mask tensors are the very same objects (checked through weak
    references, so a freed tensor whose memory is reused never matches), none
    of them was modified in place since (torch version counters), and the
    address space, flags and stream agree.  Whether a CUDA graph is being
    captured is part of the key: a tape made during a capture (in the graph's
    memory pool) is reused only inside that capture, and a tape made outside
    one is never referenced by a captured graph.  Writing into an address
    tensor behind torch's back (raw pointers) is not detected: call
    ``clear_tape_cache()`` after that.
    """

    def __init__(self):
        self.key = None
        self.refs = None
        self.value = None
        self.partner = None  # (payload ref, payload version, latest-k node ref) of the tape's latest-k call
        self.touched = None  # the key of the entry the last get hit or put made

    @staticmethod
    def _key(write, read, mask, A, stream):
        return (A, _flags(read, mask), tuple(write.shape), write.dtype, write.device, stream, write._version,
                None if read is None else (read.dtype, read._version),
                None if mask is None else (mask.dtype, mask._version), _capturing())

    def get(self, write, read, mask, A, stream):
        if self.key is None:
            return None
        if self._key(write, read, mask, A, stream) != self.key:
            return None
        w, r, m = (ref() if ref is not None else None for ref in self.refs)
        if w is not write or r is not read or m is not mask:
            return None
        self.touched = self.key
        return self.value

    def put(self, write, read, mask, A, stream, value):
        self.key = self._key(write, read, mask, A, stream)
        self.refs = tuple(None if t is None else weakref.ref(t) for t in (write, read, mask))
        self.value = value
        self.partner = None
        self.touched = self.key

    def note_latest_k(self, payload, node):
        """Remember the latest-k call that just used the cached tape (see ``_SegSumFn.backward``)."""
        if node is not None and self.key is not None and self.touched is self.key:
            self.partner = (weakref.ref(payload), payload._version, weakref.ref(node))

    def latest_k_partner(self, write, read, mask, A, stream, payload):
        """The latest-k node that read this same payload through this same tape, if any."""
        if self.partner is None or self.get(write, read, mask, A, stream) is None:
            return None
        pref, version, node = self.partner
        if pref() is not payload or payload._version != version:
            return None
        return node

    def clear(self):
        self.key = self.refs = self.value = self.partner = self.touched = None


_tape_cache = _TapeCache()


def clear_tape_cache() -> None:
    """Forget the cached tape (see ``_TapeCache``)."""
    _tape_cache.clear()


def _build_tape(write: Tensor, read: Optional[Tensor], write_mask: Optional[Tensor], A: int, D: int, k: int,
                dcode: int, device: torch.device) -> Tuple[Tensor, Tensor, Tensor, int, int]:
    """Sort the write events; returns (tape, scratch, read-or-write addresses, addr code, flags)."""
    B, T, C = write.shape
    flags = _flags(read, write_mask)
    st = _stream(device)
    hit = _tape_cache.get(write, read, write_mask, A, st)
    if hit is not None:
        tape, r, code = hit
        scratch = torch.empty(scratch_bytes(B, T, C, D, A, k, dcode, flags), dtype=torch.uint8, device=device)
        return tape, scratch, r, code, flags
    w, code = _addr(write)
    if read is not None:
        r, rcode = _addr(read)
        if rcode != code:
            w, r = w.to(torch.int64), r.to(torch.int64)
            code = _lib.RAVEL_I64
    else:
        r = w
    m = None
    if write_mask is not None:
        m = write_mask.to(torch.bool).contiguous()
    _, tape, scratch = _lib.run("ravel_tape_build", _host().tape_build, w, r if read is not None else None, code, m,
                                A, flags, D, k, dcode)
    _tape_cache.put(write, read, write_mask, A, st, (tape, r, code))
    return tape, scratch, r, code, flags


# ------------------------------------------------------------------ latest-k custom ops
class _TokenTape:
    """A tape built from token ids (``ravel_tape_build_tokens``) and its reads' folded addresses."""

    def __init__(self, tape: Tensor, raddr: Tensor, flags: int, shape: Tuple[int, int, int]):
        self.tape, self.raddr, self.flags, self.shape = tape, raddr, flags, shape


def _tape_of(write, read, write_mask, address_space, D, k, dcode, device, prebuilt):
    if prebuilt is None:
        return _build_tape(write, read, write_mask, address_space, D, k, dcode, device)
    B, T, C = prebuilt.shape
    scratch = torch.empty(scratch_bytes(B, T, C, D, address_space, k, dcode, prebuilt.flags), dtype=torch.uint8,
                          device=device)
    return prebuilt.tape, scratch, prebuilt.raddr, _lib.RAVEL_I32, prebuilt.flags


def _latestk_fwd_impl(write: Tensor, payload: Tensor, read: Optional[Tensor], write_mask: Optional[Tensor],
                      address_space: int, k: int, prebuilt: Optional[_TokenTape] = None
                      ) -> Tuple[Tensor, Tensor, Tensor]:
    B, T, C = write.shape if prebuilt is None else prebuilt.shape
    D = payload.shape[-1]
    device = _require_cuda(write, payload, read, write_mask)
    tape, _scratch, r, code, flags = _tape_of(write, read, write_mask, address_space, D, k, _payload_code(payload),
                                              device, prebuilt)
    p = payload.contiguous()
    _, vals, mask = _lib.run("ravel_latestk_fwd_tape", _host().latestk_fwd, tape, flags, r if flags else None, code,
                             p, B, T, C, address_space, k)
    return vals, mask, tape


@torch.library.custom_op("ravel_b200::latestk_fwd", mutates_args=())
def _latestk_fwd(write: Tensor, payload: Tensor, read: Optional[Tensor], write_mask: Optional[Tensor],
                 address_space: int, k: int) -> Tuple[Tensor, Tensor, Tensor]:
    return _latestk_fwd_impl(write, payload, read, write_mask, address_space, k)


@_latestk_fwd.register_fake
def _latestk_fwd_fake(write, payload, read, write_mask, address_space, k):
    B, T, C = write.shape
    D = payload.shape[-1]
    flags = _flags(read, write_mask)
    return (payload.new_empty(B, T, C, k, D),
            torch.empty(B, T, C, k, dtype=torch.bool, device=payload.device),
            torch.empty(tape_bytes(B, T, C, address_space, flags), dtype=torch.uint8, device=payload.device))


def _latestk_bwd_impl(tape: Tensor, grad_vals: Tensor, raddr: Tensor, flags: int, B: int, T: int, C: int,
                      address_space: int, k: int, accumulate_into: Optional[Tensor] = None) -> Tensor:
    """Payload gradient of the latest-k values; added to ``accumulate_into`` when given."""
    D = grad_vals.shape[-1]
    device = _require_cuda(tape, grad_vals)
    g = grad_vals.contiguous()
    _payload_code(g)
    entry = "ravel_latestk_bwd"
    if accumulate_into is not None:
        entry = "ravel_latestk_bwd_accumulate"
        a = accumulate_into
        if a.dtype != g.dtype or a.shape != (B, T, C, D) or not a.is_contiguous() or a.device != device:
            raise RuntimeError("accumulation target must be a contiguous [B, T, C, D] tensor of the gradient dtype")
    r, code = _addr(raddr)
    return _lib.run(entry, _host().latestk_bwd, tape, flags, r if flags else None, code, g, B, T, C, address_space, k,
                    accumulate_into)[1]


@torch.library.custom_op("ravel_b200::latestk_bwd", mutates_args=())
def _latestk_bwd(tape: Tensor, grad_vals: Tensor, raddr: Tensor, flags: int, B: int, T: int, C: int,
                 address_space: int, k: int) -> Tensor:
    return _latestk_bwd_impl(tape, grad_vals, raddr, flags, B, T, C, address_space, k)


@_latestk_bwd.register_fake
def _latestk_bwd_fake(tape, grad_vals, raddr, flags, B, T, C, address_space, k):
    return grad_vals.new_empty(B, T, C, grad_vals.shape[-1])


def _latestk_setup(ctx, inputs, output):
    write, payload, read, write_mask, address_space, k = inputs
    _, mask, tape = output
    ctx.save_for_backward(tape, write if read is None else read)
    ctx.meta = (_flags(read, write_mask), *write.shape, int(address_space), int(k))
    ctx.mark_non_differentiable(mask, tape)
    ctx.set_materialize_grads(False)


def _latestk_backward(ctx, grad_vals, _gm, _gt):
    if grad_vals is None:
        return None, None, None, None, None, None
    tape, raddr = ctx.saved_tensors
    flags, B, T, C, A, k = ctx.meta
    grad = _latestk_bwd(tape, grad_vals, raddr, flags, B, T, C, A, k)
    return None, grad, None, None, None, None


_latestk_fwd.register_autograd(_latestk_backward, setup_context=_latestk_setup)


# ------------------------------------------------------------------ sum custom ops
def _segsum_fwd_impl(write: Tensor, payload: Tensor, read: Optional[Tensor], write_mask: Optional[Tensor],
                     address_space: int, prebuilt: Optional[_TokenTape] = None) -> Tuple[Tensor, Tensor, Tensor]:
    B, T, C = write.shape if prebuilt is None else prebuilt.shape
    D = payload.shape[-1]
    device = _require_cuda(write, payload, read, write_mask)
    tape, scratch, r, code, flags = _tape_of(write, read, write_mask, address_space, D, 1, _payload_code(payload),
                                             device, prebuilt)
    p = payload.contiguous()
    _, sums, mask = _lib.run("ravel_segsum_fwd_tape", _host().segsum_fwd, tape, flags, r if flags else None, code, p,
                             scratch, B, T, C, address_space)
    return sums, mask, tape


@torch.library.custom_op("ravel_b200::segsum_fwd", mutates_args=())
def _segsum_fwd(write: Tensor, payload: Tensor, read: Optional[Tensor], write_mask: Optional[Tensor],
                address_space: int) -> Tuple[Tensor, Tensor, Tensor]:
    return _segsum_fwd_impl(write, payload, read, write_mask, address_space)


@_segsum_fwd.register_fake
def _segsum_fwd_fake(write, payload, read, write_mask, address_space):
    B, T, C = write.shape
    D = payload.shape[-1]
    flags = _flags(read, write_mask)
    return (payload.new_empty(B, T, C, D),
            torch.empty(B, T, C, dtype=torch.bool, device=payload.device),
            torch.empty(tape_bytes(B, T, C, address_space, flags), dtype=torch.uint8, device=payload.device))


def _segsum_bwd_impl(tape: Tensor, grad_sums: Tensor, raddr: Tensor, flags: int, B: int, T: int, C: int,
                     address_space: int) -> Tensor:
    D = grad_sums.shape[-1]
    _require_cuda(tape, grad_sums)
    g = grad_sums.contiguous()
    _payload_code(g)
    r, code = _addr(raddr)
    return _lib.run("ravel_segsum_bwd", _host().segsum_bwd, tape, flags, r if flags else None, code, g, B, T, C,
                    address_space)[1]


@torch.library.custom_op("ravel_b200::segsum_bwd", mutates_args=())
def _segsum_bwd(tape: Tensor, grad_sums: Tensor, raddr: Tensor, flags: int, B: int, T: int, C: int,
                address_space: int) -> Tensor:
    return _segsum_bwd_impl(tape, grad_sums, raddr, flags, B, T, C, address_space)


@_segsum_bwd.register_fake
def _segsum_bwd_fake(tape, grad_sums, raddr, flags, B, T, C, address_space):
    return grad_sums.new_empty(B, T, C, grad_sums.shape[-1])


def _segsum_setup(ctx, inputs, output):
    write, payload, read, write_mask, address_space = inputs
    _, mask, tape = output
    ctx.save_for_backward(tape, write if read is None else read)
    ctx.meta = (_flags(read, write_mask), *write.shape, int(address_space))
    ctx.mark_non_differentiable(mask, tape)
    ctx.set_materialize_grads(False)


def _segsum_backward(ctx, grad_sums, _gm, _gt):
    if grad_sums is None:
        return None, None, None, None, None
    tape, raddr = ctx.saved_tensors
    flags, B, T, C, A = ctx.meta
    return None, _segsum_bwd(tape, grad_sums, raddr, flags, B, T, C, A), None, None, None


_segsum_fwd.register_autograd(_segsum_backward, setup_context=_segsum_setup)


# ------------------------------------------------------------------ eager autograd functions
# Outside torch.compile the public functions call these instead of the custom
# ops: same implementation functions, same saved tensors and gradients, without
# the custom-op dispatch (tens of microseconds of host time per call, which
# decides the step time whenever the kernels are short).
#
# One payload, two lookups.  A memory layer reads the same payload tensor with
# both lookups (ravel_lm/model.py:367-384), so autograd would add their two
# payload gradients with an extra elementwise kernel (read both, write the
# sum).  Instead, when the sum lookup reused the tape of a latest-k call on the
# same payload (same tensor, unmodified), its backward -- which the engine runs
# first, being the later node -- checks that the latest-k node runs in the same
# backward pass (``torch._C._will_engine_execute_node``).  If so it hands its
# gradient to that node instead of returning it, and the latest-k backward adds
# its own gradient into that buffer in its kernel
# (``ravel_latestk_bwd_accumulate``) and returns the total.  Whatever else
# happens (only one output used, separate backward calls, create_graph, the
# nodes in the other order) each backward returns its own gradient as usual.
class _LatestKFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, write, payload, read, write_mask, address_space, k, prebuilt=None):
        vals, mask, tape = _latestk_fwd_impl(write, payload, read, write_mask, address_space, k, prebuilt)
        if prebuilt is None:
            ctx.save_for_backward(tape, write if read is None else read)
            ctx.meta = (_flags(read, write_mask), *write.shape, int(address_space), int(k))
        else:
            ctx.save_for_backward(tape, prebuilt.raddr)
            ctx.meta = (prebuilt.flags, *prebuilt.shape, int(address_space), int(k))
        ctx.ravel_stash = None
        ctx.mark_non_differentiable(mask)
        ctx.set_materialize_grads(False)
        return vals, mask

    @staticmethod
    def backward(ctx, grad_vals, _gm):
        stash, ctx.ravel_stash = ctx.ravel_stash, None
        acc = None
        if stash is not None and stash[0] == torch._C._current_graph_task_id():
            acc = stash[1]  # the sum lookup's payload gradient, handed over in this same pass
        if grad_vals is None:
            return None, acc, None, None, None, None, None
        tape, raddr = ctx.saved_tensors
        flags, B, T, C, A, k = ctx.meta
        grad = _latestk_bwd_impl(tape, grad_vals, raddr, flags, B, T, C, A, k, accumulate_into=acc)
        return None, grad, None, None, None, None, None


class _SegSumFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, write, payload, read, write_mask, address_space, partner, prebuilt=None):
        sums, mask, tape = _segsum_fwd_impl(write, payload, read, write_mask, address_space, prebuilt)
        if prebuilt is None:
            ctx.save_for_backward(tape, write if read is None else read)
            ctx.meta = (_flags(read, write_mask), *write.shape, int(address_space))
        else:
            ctx.save_for_backward(tape, prebuilt.raddr)
            ctx.meta = (prebuilt.flags, *prebuilt.shape, int(address_space))
        ctx.partner = partner
        ctx.mark_non_differentiable(mask)
        ctx.set_materialize_grads(False)
        return sums, mask

    @staticmethod
    def backward(ctx, grad_sums, _gm):
        if grad_sums is None:
            return None, None, None, None, None, None, None
        tape, raddr = ctx.saved_tensors
        flags, B, T, C, A = ctx.meta
        grad = _segsum_bwd_impl(tape, grad_sums, raddr, flags, B, T, C, A)
        node = ctx.partner() if ctx.partner is not None else None
        if (node is not None and not torch.is_grad_enabled() and getattr(node, "ravel_stash", 1) is None
                and torch._C._will_engine_execute_node(node)):
            node.ravel_stash = (torch._C._current_graph_task_id(), grad)
            return None, None, None, None, None, None, None
        return None, grad, None, None, None, None, None


# ------------------------------------------------------------------ public API
def causal_last_k_lookup(
    write_addresses: Tensor,
    payloads: Tensor,
    read_addresses: Optional[Tensor] = None,
    *,
    address_space: int,
    k: int = 1,
    write_mask: Optional[Tensor] = None,
) -> Tuple[Tensor, Tensor]:
    """Exact causal last-k lookup over an event tape (ravel_lm/ravel_memory.py:52-176).

    For every read at time ``t`` returns the latest ``k`` payloads written with
    the same ``(batch, head, address)`` at a time ``< t``.

    Args:
        write_addresses: [B, T, C] integer addresses for writes.
        payloads:        [B, T, C, D] float32 / bfloat16 / float16 / float64.
        read_addresses:  [B, T, C] integer read addresses. Defaults to writes.
        address_space:   number of legal addresses per memory head; addresses
                         are reduced modulo it (negative values wrap).
        k:               number of latest records to return.
        write_mask:      optional [B, T] boolean mask; false entries do not write.

    Returns:
        values: [B, T, C, k, D] (payload dtype), mask: [B, T, C, k] bool.
    """
    if read_addresses is None:
        read_addresses = write_addresses
    if write_addresses.shape != read_addresses.shape:
        raise ValueError("write_addresses and read_addresses must have the same shape")
    if write_addresses.ndim != 3:
        raise ValueError("addresses must have shape [B, T, C]")
    if payloads.ndim != 4:
        raise ValueError("payloads must have shape [B, T, C, D]")
    B, T, C = write_addresses.shape
    if payloads.shape[:3] != (B, T, C):
        raise ValueError("payloads leading dimensions must match addresses")
    if k <= 0:
        raise ValueError("k must be positive")
    if write_mask is not None and write_mask.shape != (B, T):
        raise ValueError("write_mask must have shape [B, T]")
    _require_cuda(write_addresses, payloads, read_addresses, write_mask)
    read = None if _aliases(read_addresses, write_addresses) else read_addresses
    if B * T * C == 0:
        return payloads.new_zeros(B, T, C, k, payloads.shape[-1]), torch.zeros(
            B, T, C, k, dtype=torch.bool, device=payloads.device)
    if torch.compiler.is_compiling():
        vals, mask, _tape = _latestk_fwd(write_addresses, payloads, read, write_mask, int(address_space), int(k))
        return vals, mask
    _tape_cache.touched = None
    vals, mask = _LatestKFn.apply(write_addresses, payloads, read, write_mask, int(address_space), int(k))
    if vals.grad_fn is not None:
        _tape_cache.note_latest_k(payloads, vals.grad_fn)
    return vals, mask


def causal_sum_lookup(
    write_addresses: Tensor,
    payloads: Tensor,
    read_addresses: Optional[Tensor] = None,
    *,
    address_space: int,
    write_mask: Optional[Tensor] = None,
) -> Tuple[Tensor, Tensor]:
    """Exact causal segmented prefix-sum lookup (ravel_lm/ravel_memory.py:179-241).

    For every read at time ``t`` returns the sum of all payloads with matching
    ``(batch, head, address)`` and time ``< t``; differentiable w.r.t. payloads.
    """
    if read_addresses is None:
        read_addresses = write_addresses
    if write_addresses.ndim != 3 or payloads.ndim != 4:
        raise ValueError("expected write_addresses [B,T,C] and payloads [B,T,C,D]")
    B, T, C = write_addresses.shape
    if read_addresses.shape != write_addresses.shape:
        raise ValueError("write_addresses and read_addresses must have the same shape")
    if payloads.shape[:3] != (B, T, C):
        raise ValueError("payloads leading dimensions must match addresses")
    if write_mask is not None and write_mask.shape != (B, T):
        raise ValueError("write_mask must have shape [B, T]")
    _require_cuda(write_addresses, payloads, read_addresses, write_mask)
    read = None if _aliases(read_addresses, write_addresses) else read_addresses
    if B * T * C == 0:
        return payloads.new_zeros(B, T, C, payloads.shape[-1]), torch.zeros(
            B, T, C, dtype=torch.bool, device=payloads.device)
    if torch.compiler.is_compiling():
        sums, mask, _tape = _segsum_fwd(write_addresses, payloads, read, write_mask, int(address_space))
        return sums, mask
    partner = None
    if payloads.requires_grad and torch.is_grad_enabled():
        partner = _tape_cache.latest_k_partner(write_addresses, read, write_mask, int(address_space),
                                               _stream(payloads.device), payloads)
    return _SegSumFn.apply(write_addresses, payloads, read, write_mask, int(address_space), partner)


# ------------------------------------------------------------------ decode cache
@dataclass
class RavelLayerCache:
    """Latest-value cache for decoding (ravel_lm/ravel_memory.py:244-292).

    ``values [B, C, A, D]`` and ``filled [B, C, A]`` stay plain tensors, so the
    cache pickles and state-dicts exactly like the reference's.  ``read`` and
    ``write`` are one kernel launch each on the current stream; ``step`` does a
    read followed by a write in a single launch.  Addresses are clamped to
    [0, A-1] as in the reference.
    """

    values: Tensor
    filled: Tensor

    @classmethod
    def empty(cls, batch_size: int, n_heads: int, address_space: int, payload_dim: int, *,
              device: torch.device | str, dtype: torch.dtype) -> "RavelLayerCache":
        values = torch.zeros(batch_size, n_heads, address_space, payload_dim, device=device, dtype=dtype)
        filled = torch.zeros(batch_size, n_heads, address_space, device=device, dtype=torch.bool)
        return cls(values=values, filled=filled)

    def _check_storage(self) -> None:
        if not (self.values.is_contiguous() and self.filled.is_contiguous()):
            raise ValueError("cache tensors must be contiguous")
        if self.filled.dtype != torch.bool:
            raise ValueError("cache.filled must be a bool tensor")
        _payload_code(self.values)

    def read(self, addresses: Tensor) -> Tuple[Tensor, Tensor]:
        """Read latest values for addresses [B, C]. Returns ([B,C,D], [B,C])."""
        B, C = addresses.shape
        if self.values.shape[:2] != (B, C):
            raise ValueError(f"cache shape {self.values.shape[:2]} does not match addresses {(B, C)}")
        device = _require_cuda(self.values, self.filled, addresses)
        self._check_storage()
        A, D = self.values.shape[2], self.values.shape[3]
        a, code = _addr(addresses)
        vals = self.values.new_empty(B, C, D)
        mask = torch.empty(B, C, dtype=torch.bool, device=device)
        _lib.call("ravel_cache_read", self.values.data_ptr(), self.filled.data_ptr(), a.data_ptr(), code,
                  _payload_code(self.values), B, C, A, D, vals.data_ptr(), mask.data_ptr(), _stream(device))
        return vals, mask

    def write(self, addresses: Tensor, payloads: Tensor) -> None:
        """Write latest payloads. addresses [B,C], payloads [B,C,D]."""
        B, C = addresses.shape
        D = payloads.shape[-1]
        if self.values.shape[:2] != (B, C) or self.values.shape[-1] != D:
            raise ValueError("cache and payload shapes do not match")
        if payloads.shape[:2] != (B, C):
            raise ValueError("cache and payload shapes do not match")
        device = _require_cuda(self.values, self.filled, addresses, payloads)
        self._check_storage()
        a, code = _addr(addresses)
        p = payloads.to(self.values.dtype).contiguous()
        _lib.call("ravel_cache_write", self.values.data_ptr(), self.filled.data_ptr(), a.data_ptr(), code,
                  p.data_ptr(), _payload_code(self.values), B, C, self.values.shape[2], D, _stream(device))

    def prefill(self, write_addresses: Tensor, payloads: Tensor) -> None:
        """All writes of a prefill at once: the cache state left by ``write(write_addresses[:, t],
        payloads[:, t])`` for t = 0 .. T-1 in order.  addresses [B, T, C], payloads [B, T, C, D].

        The reference prefills token by token (ravel_lm/model.py:600-602), one ``write`` per position
        and layer; this sorts each stream's writes once and copies the last write of every address.
        """
        if write_addresses.dim() != 3:
            raise ValueError("write_addresses must have shape [B, T, C]")
        B, T, C = write_addresses.shape
        D = payloads.shape[-1]
        if self.values.shape[:2] != (B, C) or self.values.shape[-1] != D:
            raise ValueError("cache and payload shapes do not match")
        if payloads.shape[:3] != (B, T, C):
            raise ValueError("cache and payload shapes do not match")
        device = _require_cuda(self.values, self.filled, write_addresses, payloads)
        self._check_storage()
        if B * T * C == 0:
            return
        A = self.values.shape[2]
        a, code = _addr(write_addresses)
        p = payloads.to(self.values.dtype).contiguous()
        lib = _lib.load()
        scratch = torch.empty(int(lib.ravel_cache_prefill_scratch_bytes(B, T, C, A)), dtype=torch.uint8,
                              device=device)
        _lib.call("ravel_cache_prefill", self.values.data_ptr(), self.filled.data_ptr(), a.data_ptr(), code,
                  p.data_ptr(), _payload_code(self.values), B, T, C, A, D, scratch.data_ptr(), scratch.numel(),
                  _stream(device))

    def step(self, read_addresses: Tensor, write_addresses: Tensor, payloads: Tensor,
             out: Optional[Tuple[Tensor, Tensor]] = None) -> Tuple[Tensor, Tensor]:
        """``read(read_addresses)`` then ``write(write_addresses, payloads)`` in one launch.

        Decode calls this once per memory layer and token, so the common case --
        contiguous CUDA tensors on one device, int64 (or int32) addresses of one
        type, payloads in the cache's dtype -- is checked and launched by one
        call into the C++ host extension; anything else goes through the same
        checks as ``read`` and ``write``.  ``out``: a (values [B, C, D], mask
        [B, C] bool) pair of contiguous tensors to write the read into instead of
        new ones (a decode loop that reuses its buffers).
        """
        values, filled = self.values, self.filled
        if _lib._call_hook is None and isinstance(read_addresses, Tensor) and isinstance(write_addresses, Tensor) \
                and isinstance(payloads, Tensor):
            # the common case, checked, allocated and launched in C++ (None: anything else)
            res = (_lib._host or _lib.host()).cache_step(values, filled, read_addresses, write_addresses, payloads, out)
            if res.__class__ is tuple:
                return res
            if res is not None:
                _lib.check("ravel_cache_step", res)
        B, C = read_addresses.shape
        D = payloads.shape[-1]
        if write_addresses.shape != (B, C) or values.shape[:2] != (B, C) or values.shape[-1] != D:
            raise ValueError("cache and payload shapes do not match")
        if payloads.shape[:2] != (B, C):
            raise ValueError("cache and payload shapes do not match")
        device = _require_cuda(values, filled, read_addresses, write_addresses, payloads)
        self._check_storage()
        ra, rcode = _addr(read_addresses)
        wa, wcode = _addr(write_addresses)
        if rcode != wcode:
            ra, wa, rcode = ra.to(torch.int64), wa.to(torch.int64), _lib.RAVEL_I64
        p = payloads.to(values.dtype).contiguous()
        code = _payload_code(values)
        if out is None:
            vals = values.new_empty(B, C, D)
            mask = torch.empty(B, C, dtype=torch.bool, device=device)
        else:
            vals, mask = out
            if (vals.shape != (B, C, D) or vals.dtype != values.dtype or mask.shape != (B, C)
                    or mask.dtype != torch.bool or vals.device != device or mask.device != device
                    or not (vals.is_contiguous() and mask.is_contiguous())):
                raise ValueError("out must be contiguous (values [B, C, D] of the cache dtype, mask [B, C] bool)")
        _lib.call("ravel_cache_step", values.data_ptr(), filled.data_ptr(), ra.data_ptr(), wa.data_ptr(), rcode,
                  p.data_ptr(), code, B, C, values.shape[2], D, vals.data_ptr(), mask.data_ptr(), _stream(device))
        return vals, mask


# ------------------------------------------------------------------ memory-layer addresses from token ids
@torch.library.custom_op("ravel_b200::literal_addresses", mutates_args=())
def _literal_addresses(token_ids: Tensor, address_space: int, n_heads: int, bos_token_id: int) -> Tensor:
    B, T = token_ids.shape
    device = _require_cuda(token_ids)
    toks = token_ids.to(torch.int64).contiguous()
    out = torch.empty(B, T, n_heads, dtype=torch.int64, device=device)
    _lib.call("ravel_literal_addresses", toks.data_ptr(), B, T, n_heads, bos_token_id, address_space, out.data_ptr(),
              _stream(device))
    return out


@_literal_addresses.register_fake
def _literal_addresses_fake(token_ids, address_space, n_heads, bos_token_id):
    return torch.empty(*token_ids.shape, n_heads, dtype=torch.int64, device=token_ids.device)


def literal_addresses_from_tokens(token_ids: Tensor, *, address_space: int, n_heads: int,
                                  bos_token_id: int) -> Tensor:
    """Literal address families from token ids (ravel_lm/model.py:195-231), one kernel.

    Heads, in order: the token id; a rolling bigram hash; a rolling trigram hash;
    token/position mixed hashes; each modulo ``address_space``.  Returns
    [B, T, n_heads] int64, equal to the reference's values.
    """
    if token_ids.ndim != 2:
        raise ValueError("token_ids must have shape [B,T]")
    if int(address_space) <= 0:
        raise ValueError("address_space must be positive")
    B, T = token_ids.shape
    if B * T * int(n_heads) == 0:
        return torch.empty(B, T, int(n_heads), dtype=torch.long, device=token_ids.device)
    return _literal_addresses(token_ids, int(address_space), int(n_heads), int(bos_token_id))


def memory_lookups(token_ids: Tensor, payloads: Tensor, learned_write: Optional[Tensor] = None,
                   learned_read: Optional[Tensor] = None, *, address_space: int, n_literal_heads: int,
                   bos_token_id: int, k: int = 1, use_sum_read: bool = False, write_mask: Optional[Tensor] = None
                   ) -> Tuple[Tensor, Tensor, Optional[Tensor], Optional[Tensor]]:
    """The lookups of one memory layer, addressed from its token ids.

    Equal to what ``RavelMemoryLayer.forward`` (ravel_lm/model.py:333-384) computes
    with this package's three functions::

        literal = literal_addresses_from_tokens(token_ids, address_space=A, n_heads=L, bos_token_id=bos)
        write = torch.cat([literal, learned_write], -1); read = torch.cat([literal, learned_read], -1)
        values, mask = causal_last_k_lookup(write, payloads, read, address_space=A, k=k, write_mask=m)
        sums, smask = causal_sum_lookup(write, payloads, read, address_space=A, write_mask=m)

    but the literal heads are hashed inside the sort's key build
    (``ravel_tape_build_tokens``): no [B, T, C] address tensor is made, one sort
    serves both lookups, and one backward pass writes the payload gradient once.

    Args:
        token_ids:     [B, T] integer token ids.
        payloads:      [B, T, C, D] with C = n_literal_heads + learned heads.
        learned_write: [B, T, C - n_literal_heads] integer addresses of the learned
                       heads' writes (None when every head is literal).
        learned_read:  the same for reads; None (or the write tensor) reads where it writes.
        use_sum_read:  also return the segmented sums.
    Returns:
        values [B, T, C, k, D], mask [B, T, C, k], and sums [B, T, C, D] and their
        mask [B, T, C] (None, None without ``use_sum_read``).
    """
    if token_ids.ndim != 2 or payloads.ndim != 4:
        raise ValueError("expected token_ids [B,T] and payloads [B,T,C,D]")
    B, T = token_ids.shape
    L = int(n_literal_heads)
    C = payloads.shape[2]
    if payloads.shape[:2] != (B, T) or not 0 <= L <= C:
        raise ValueError("payloads must be [B, T, C, D] with C >= n_literal_heads")
    if (learned_write is None) != (C == L):
        raise ValueError("learned_write must be given exactly when there are learned heads")
    for t in (learned_write, learned_read):
        if t is not None and tuple(t.shape) != (B, T, C - L):
            raise ValueError("learned addresses must have shape [B, T, C - n_literal_heads]")
    if k <= 0:
        raise ValueError("k must be positive")
    if write_mask is not None and write_mask.shape != (B, T):
        raise ValueError("write_mask must have shape [B, T]")
    A = int(address_space)
    if A <= 0 or A > 2**31 - 1:
        raise ValueError("address_space must be in [1, 2^31 - 1]")
    if torch.compiler.is_compiling() or B * T * C == 0:
        lit = literal_addresses_from_tokens(token_ids, address_space=A, n_heads=L, bos_token_id=bos_token_id)
        write = lit if learned_write is None else torch.cat([lit, learned_write.to(torch.int64)], -1)
        read = None
        if learned_read is not None and learned_read is not learned_write:
            read = torch.cat([lit, learned_read.to(torch.int64)], -1)
        vals, mask = causal_last_k_lookup(write, payloads, read, address_space=A, k=k, write_mask=write_mask)
        if not use_sum_read:
            return vals, mask, None, None
        sums, smask = causal_sum_lookup(write, payloads, read, address_space=A, write_mask=write_mask)
        return vals, mask, sums, smask
    device = _require_cuda(token_ids, payloads, learned_write, learned_read, write_mask)
    toks = token_ids.to(torch.int64).contiguous()
    lw = lr = None
    code = _lib.RAVEL_I64
    if learned_write is not None:
        lw, code = _addr(learned_write)
        lr = lw
        if learned_read is not None and not _aliases(learned_read, learned_write):
            lr, rcode = _addr(learned_read)
            if rcode != code:
                lw, lr, code = lw.to(torch.int64), lr.to(torch.int64), _lib.RAVEL_I64
    general = lr is not None and lr is not lw
    flags = (_lib.RAVEL_TAPE_GENERAL_READS if general else 0) | (_lib.RAVEL_TAPE_WRITE_MASK if write_mask is not None
                                                                else 0)
    m = None if write_mask is None else write_mask.to(torch.bool).contiguous()
    D = payloads.shape[-1]
    tape = torch.empty(tape_bytes(B, T, C, A, flags), dtype=torch.uint8, device=device)
    scratch = torch.empty(scratch_bytes(B, T, C, D, A, k, _payload_code(payloads), flags), dtype=torch.uint8,
                          device=device)
    raddr = torch.empty((B, T, C) if flags else (0,), dtype=torch.int32, device=device)
    _lib.call("ravel_tape_build_tokens", toks.data_ptr(), L, int(bos_token_id), _ptr(lw), _ptr(lr), code, _ptr(m),
              B, T, C, A, flags, raddr.data_ptr() if flags else None, tape.data_ptr(), tape.numel(),
              scratch.data_ptr(), scratch.numel(), _stream(device))
    pre = _TokenTape(tape, raddr, flags, (B, T, C))
    vals, mask = _LatestKFn.apply(None, payloads, None, m, A, int(k), pre)
    if not use_sum_read:
        return vals, mask, None, None
    partner = None
    if vals.grad_fn is not None and torch.is_grad_enabled():
        partner = weakref.ref(vals.grad_fn)
    sums, smask = _SegSumFn.apply(None, payloads, None, m, A, partner, pre)
    return vals, mask, sums, smask


__all__ = ["RavelLayerCache", "causal_last_k_lookup", "causal_sum_lookup", "clear_tape_cache",
           "literal_addresses_from_tokens", "memory_lookups", "_composite_key_dtype"]
