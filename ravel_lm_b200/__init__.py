"""ravel_lm_b200 -- RAVEL's exact event-memory operator on B200 (sm_100a).

A drop-in for ``ravel_lm.ravel_memory`` of the ravel-lm project: the same
``causal_last_k_lookup``, ``causal_sum_lookup`` and ``RavelLayerCache``,
computed by hand-written CUDA kernels in ``libravel_b200.so`` (C ABI:
``include/ravel_b200.h``).  Multi-GPU helpers (stream sharding, optional
replicated outputs over NCCL) are in ``ravel_lm_b200.sharding``.
"""
from .ravel_memory import (  # noqa: F401
    RavelLayerCache,
    _composite_key_dtype,
    causal_last_k_lookup,
    causal_sum_lookup,
    literal_addresses_from_tokens,
    memory_lookups,
)

__all__ = ["RavelLayerCache", "causal_last_k_lookup", "causal_sum_lookup", "literal_addresses_from_tokens",
           "memory_lookups"]
__version__ = "0.1.0"
