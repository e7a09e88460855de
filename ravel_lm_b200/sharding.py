"""Stream sharding of the event-memory operator across the GPUs of one node.

A stream is one (batch row b, memory head c) pair.  Streams never interact:
the reference's composite key puts (b*C + c) in its high bits
(ravel_lm/ravel_memory.py:26-38), so every lookup of stream (b, c) reads only
writes of (b, c).  The operator therefore shards over streams with no
exchange on the forward or backward path: each rank runs the ordinary
single-GPU entry points on its own slice.

Partition (``shard_streams``):
  * B >= world and B % world == 0: rank g owns batch rows [g*B/W, (g+1)*B/W),
    all heads -- contiguous in every [B, T, C, ...] tensor;
  * B < world and world % B == 0 and C % (world/B) == 0: rank g owns batch row
    g // (W/B) and heads [h0, h0 + C*B/W) with h0 = (g % (W/B)) * C*B/W.
Other shapes are rejected (ValueError): shards must be equal for the
collective below.

Replicated outputs are optional (``gather_outputs``): one
``all_gather_into_tensor`` of the equally shaped shards over the process
group (NCCL over NVLink on GPUs, gloo on CPU) and a local reorder back to the
full layout.

The reference's int64 -> int32 address truncation depends on the size of the
whole call (ravel_lm/ravel_memory.py:45-49); ``sharded_lookup`` applies the
whole problem's rule to every shard.

Sharded results equal the unsharded ones as values.  The one bit that can
differ is the sign of an invalid latest-k slot at the very start of a stream:
the reference fills such a slot with candidate*0, where the candidate is the
previous stream's last write in its global sort order, and a shard's previous
stream is not the full problem's.  Masks, valid values and sums are identical.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional, Sequence

import torch


@dataclass(frozen=True)
class StreamShard:
    """Streams owned by one rank: batch rows [b0, b1) x heads [c0, c1)."""

    rank: int
    world: int
    B: int
    C: int
    b0: int
    b1: int
    c0: int
    c1: int

    @property
    def streams(self) -> int:
        return (self.b1 - self.b0) * (self.c1 - self.c0)

    @property
    def splits_heads(self) -> bool:
        return (self.c1 - self.c0) != self.C

    def take(self, t: Optional[torch.Tensor], head_dim: bool = True) -> Optional[torch.Tensor]:
        """This rank's slice of a [B, T, C, ...] tensor ([B, T] when head_dim=False), contiguous."""
        if t is None:
            return None
        x = t[self.b0:self.b1]
        if head_dim:
            x = x[:, :, self.c0:self.c1]
        return x.contiguous()


def shard_streams(B: int, C: int, world: int, rank: int) -> StreamShard:
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    if B >= world:
        if B % world:
            raise ValueError(f"batch {B} does not divide over {world} ranks")
        per = B // world
        return StreamShard(rank, world, B, C, rank * per, (rank + 1) * per, 0, C)
    if world % B:
        raise ValueError(f"{world} ranks do not divide over batch {B}")
    parts = world // B
    if C % parts:
        raise ValueError(f"{C} heads do not divide into {parts} parts")
    hc = C // parts
    b = rank // parts
    h0 = (rank % parts) * hc
    return StreamShard(rank, world, B, C, b, b + 1, h0, h0 + hc)


def all_shards(B: int, C: int, world: int) -> list[StreamShard]:
    return [shard_streams(B, C, world, g) for g in range(world)]


def assemble(pieces: Sequence[torch.Tensor], shards: Sequence[StreamShard]) -> torch.Tensor:
    """Put per-rank outputs [b1-b0, T, c1-c0, ...] back into the full [B, T, C, ...] layout."""
    sh0 = shards[0]
    ref = pieces[0]
    full = ref.new_empty((sh0.B, ref.shape[1], sh0.C) + tuple(ref.shape[3:]))
    for piece, sh in zip(pieces, shards):
        full[sh.b0:sh.b1, :, sh.c0:sh.c1] = piece
    return full


def gather_outputs(local: torch.Tensor, shard: StreamShard, group=None) -> torch.Tensor:
    """Replicate a sharded output on every rank: all_gather_into_tensor + reorder.

    ``local`` is this rank's [b1-b0, T, c1-c0, ...] output.  Every rank gets
    the full [B, T, C, ...] tensor.  One collective; its cost is the full
    output crossing NVLink once per rank, so only call it when the caller
    needs replicated results.
    """
    import torch.distributed as dist
    world = shard.world
    is_bool = local.dtype == torch.bool
    flat = (local.view(torch.uint8) if is_bool else local).contiguous()
    buf = flat.new_empty((world * flat.shape[0],) + tuple(flat.shape[1:]))  # concatenated along dim 0
    dist.all_gather_into_tensor(buf, flat, group=group)
    shards = all_shards(shard.B, shard.C, world)
    full = assemble(list(buf.view((world,) + tuple(flat.shape)).unbind(0)), shards)
    return full.view(torch.bool) if is_bool else full


def _global_fold(addr: Optional[torch.Tensor], shard: StreamShard, T: int, A: int) -> Optional[torch.Tensor]:
    """Addresses of one shard, reduced with the FULL problem's key-width rule.

    The reference converts int64 addresses to its composite key dtype before
    the floor modulo (ravel_lm/ravel_memory.py:126-128), and that dtype depends
    on B*C*A*(T+1) of the whole call (:45-49).  A shard has a smaller B*C and can
    fall under the int32 bound where the full problem does not; the library
    would then truncate int64 addresses to 32 bits that the reference keeps.
    When the two rules differ, the shard's int64 addresses are reduced here
    with the full problem's rule (no truncation, floor modulo of A), which both
    rules then leave unchanged.
    """
    from .ravel_memory import _composite_key_dtype
    if addr is None or addr.dtype != torch.int64:
        return addr
    full = _composite_key_dtype(shard.B, T, shard.C, A)
    local = _composite_key_dtype(shard.b1 - shard.b0, T, shard.c1 - shard.c0, A)
    if full == local:
        return addr
    return addr.remainder(int(A))


def sharded_lookup(write_addresses: torch.Tensor, payloads: torch.Tensor, read_addresses=None, *,
                   address_space: int, k: int = 1, write_mask=None, world: int, rank: int,
                   replicate: bool = False, group=None, use_sum: bool = False,
                   full_shape: Optional[tuple[int, int]] = None):
    """Run this rank's shard of ``causal_last_k_lookup`` (or ``causal_sum_lookup``).

    By default the inputs are the full [B, T, C, ...] tensors and this rank
    slices its streams out of them.  When the caller already holds only this
    rank's slice ([b1-b0, T, c1-c0, ...], and [b1-b0, T] for the mask), it
    passes ``full_shape=(B, C)`` of the whole problem; the inputs are then used
    as they are (their shape must be the shard's).  Either way the key-width
    rule of the whole problem is applied (see ``_global_fold``), so the values
    equal those of the unsharded call.  Returns this rank's outputs, or the
    replicated full outputs when ``replicate`` is set (one NCCL all-gather per
    output).
    """
    from .ravel_memory import causal_last_k_lookup, causal_sum_lookup
    Bi, T, Ci = write_addresses.shape
    if full_shape is None:
        sh = shard_streams(Bi, Ci, world, rank)
        w, p, r = sh.take(write_addresses), sh.take(payloads), sh.take(read_addresses)
        m = None if write_mask is None else sh.take(write_mask, head_dim=False)
    else:
        B, C = (int(x) for x in full_shape)
        sh = shard_streams(B, C, world, rank)
        if (Bi, Ci) != (sh.b1 - sh.b0, sh.c1 - sh.c0):
            raise ValueError(f"inputs of shape {(Bi, T, Ci)} are not rank {rank}'s slice of a [{B}, T, {C}] "
                             f"problem over {world} ranks (expected {(sh.b1 - sh.b0, T, sh.c1 - sh.c0)})")
        w, p, r, m = write_addresses, payloads, read_addresses, write_mask
    if r is None or r is w:
        w = _global_fold(w, sh, T, address_space)
        r = None if r is None else w
    else:
        w, r = _global_fold(w, sh, T, address_space), _global_fold(r, sh, T, address_space)
    if use_sum:
        vals, mask = causal_sum_lookup(w, p, r, address_space=address_space, write_mask=m)
    else:
        vals, mask = causal_last_k_lookup(w, p, r, address_space=address_space, k=k, write_mask=m)
    if not replicate:
        return vals, mask
    return gather_outputs(vals, sh, group), gather_outputs(mask, sh, group)


__all__ = ["StreamShard", "all_shards", "assemble", "gather_outputs", "shard_streams", "sharded_lookup"]
