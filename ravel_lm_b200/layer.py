"""``RavelMemoryLayer.forward`` on this package's fused kernels.

The reference's memory layer (``ravel_lm/model.py:309-390``) computes, after its
packed input GEMM: literal addresses from the token ids, learned addresses from
the frozen product-code projections, both lookups, the concatenation of their
results, the ``fuse`` Linear and the gate residual.  ``memory_layer_forward``
computes the same output with

* the literal heads hashed inside the sort's key build
  (``ravel_tape_build_tokens``; no address tensor is built);
* the latest-k gather, the sum read, ``fuse`` and the gate residual in one
  tcgen05 kernel (``ravel_gather_gemm``, TF32 like the reference's
  ``fast_linear`` on CUDA);

and leaves the layer's norm, packed GEMM and learned-address decoding to the
layer's own modules.  Bind it to a layer (``layer.forward =
types.MethodType(memory_layer_forward, layer)``) or to the class; layers with
dropout, or whose payloads are not float32, run their own ``forward``.
"""
from __future__ import annotations

import sys
from typing import Optional

import torch

from .fused import memory_read_linear_tokens

Tensor = torch.Tensor


def memory_layer_forward(layer, x: Tensor, token_ids: Tensor, write_mask: Optional[Tensor] = None,
                         literal_addr: Optional[Tensor] = None) -> Tensor:
    """Drop-in for ``RavelMemoryLayer.forward(x, token_ids, write_mask, literal_addr)``
    (ravel_lm/model.py:309-390).  ``literal_addr`` is not needed: the literal heads are
    hashed from ``token_ids`` during the sort."""
    cfg = layer.cfg
    if layer.dropout.p != 0.0 or x.dtype != torch.float32 or cfg.payload_dim % 4 != 0:
        return type(layer).forward(layer, x, token_ids, write_mask=write_mask, literal_addr=literal_addr)
    model_mod = sys.modules[type(layer).__module__]
    B, T, _ = x.shape
    C = cfg.n_memory_heads
    xn = layer.norm(x)
    n_pay = layer.payload.weight.shape[0]
    n_gate = layer.gate.weight.shape[0]
    weights = [layer.payload.weight, layer.gate.weight]
    if layer.write_addr.proj is not None:
        weights.append(layer.write_addr.proj.weight)
        weights.append(layer.read_addr.proj.weight)
    packed = model_mod.fast_linear_packed(xn, weights)
    payload = packed[..., :n_pay].reshape(B, T, C, cfg.payload_dim)
    gate_lin = packed[..., n_pay:n_pay + n_gate] + layer.gate.bias
    learned_write = learned_read = None
    if layer.write_addr.proj is not None:
        n_addr = layer.write_addr.proj.weight.shape[0]
        addr_logits = packed[..., n_pay + n_gate:].detach()
        learned_write = layer._decode_codes(layer.write_addr, addr_logits[..., :n_addr])
        learned_read = layer._decode_codes(layer.read_addr, addr_logits[..., n_addr:])
    return memory_read_linear_tokens(token_ids, payload, learned_write, learned_read, layer.fuse.weight,
                                     address_space=cfg.address_space, n_literal_heads=cfg.n_literal_heads,
                                     bos_token_id=cfg.bos_token_id, k=cfg.last_k, use_sum_read=cfg.use_sum_read,
                                     write_mask=write_mask, x=x, gate_lin=gate_lin)


__all__ = ["memory_layer_forward"]
