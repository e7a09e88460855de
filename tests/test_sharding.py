"""Stream sharding across ranks: partition logic and a world-size-2 gloo run.

The per-rank compute in the multi-process test is the CPU oracle (this file
checks the host-side partition, collective and reassembly, not the kernels).
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from ravel_lm_b200.sharding import all_shards, assemble, shard_streams


@pytest.mark.parametrize("B,C,world", [(4, 16, 1), (4, 16, 2), (4, 16, 4), (8, 3, 8), (4, 16, 8), (1, 8, 2),
                                       (2, 6, 6)])
def test_partition_covers_every_stream_once(B, C, world):
    shards = all_shards(B, C, world)
    seen = np.zeros((B, C), int)
    for sh in shards:
        seen[sh.b0:sh.b1, sh.c0:sh.c1] += 1
    assert (seen == 1).all()
    assert len({sh.streams for sh in shards}) == 1  # equal shards for the collective


@pytest.mark.parametrize("B,C,world", [(3, 4, 2), (1, 3, 2), (2, 4, 3)])
def test_partition_rejects_unequal_shapes(B, C, world):
    with pytest.raises(ValueError):
        all_shards(B, C, world)


def test_assemble_round_trip():
    g = torch.Generator().manual_seed(0)
    x = torch.randn(2, 5, 8, 3, generator=g)
    shards = all_shards(2, 8, 4)
    pieces = [sh.take(x) for sh in shards]
    assert torch.equal(assemble(pieces, shards), x)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, B, T, C, D, A, k, out_q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        import oracle
        from ravel_lm_b200.sharding import gather_outputs
        g = torch.Generator().manual_seed(77)
        w = torch.randint(0, A, (B, T, C), generator=g)
        r = torch.randint(0, A, (B, T, C), generator=g)
        p = torch.randn(B, T, C, D, generator=g)
        sh = shard_streams(B, C, world, rank)
        vals, mask, _src, tape = oracle.latestk_fwd(sh.take(w).numpy(), sh.take(p).numpy(), sh.take(r).numpy(),
                                                    address_space=A, k=k)
        sums, smask, _ = oracle.segsum_fwd(sh.take(w).numpy(), sh.take(p).double().numpy(), sh.take(r).numpy(),
                                           address_space=A, tape=tape)
        full_vals = gather_outputs(torch.from_numpy(vals), sh)
        full_mask = gather_outputs(torch.from_numpy(mask), sh)
        full_sums = gather_outputs(torch.from_numpy(sums), sh)
        if rank == 0:
            ev, em, _, et = oracle.latestk_fwd(w.numpy(), p.numpy(), r.numpy(), address_space=A, k=k)
            es, esm, _ = oracle.segsum_fwd(w.numpy(), p.double().numpy(), r.numpy(), address_space=A, tape=et)
            ok = (np.array_equal(full_vals.numpy(), ev) and np.array_equal(full_mask.numpy(), em)
                  and np.allclose(full_sums.numpy(), es, rtol=0, atol=1e-12))
            out_q.put(bool(ok))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("B,C", [(4, 3), (1, 4)])
def test_gloo_world2_sharded_equals_unsharded(B, C):
    """Batch-row split (B >= world) and head split (B < world) over 2 gloo ranks."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(g, 2, port, B, 60, C, 4, 9, 2, q)) for g in range(2)]
    for pr in procs:
        pr.start()
    for pr in procs:
        pr.join(timeout=120)
    for pr in procs:
        if pr.is_alive():
            pr.kill()
    assert all(pr.exitcode == 0 for pr in procs)
    assert q.get(timeout=5) is True


def test_shards_apply_the_whole_problems_key_width():
    """A shard small enough for int32 keys must not truncate int64 addresses that the
    whole problem (int64 keys, ravel_lm/ravel_memory.py:45-49) keeps whole."""
    import oracle
    from ravel_lm_b200.ravel_memory import _composite_key_dtype
    from ravel_lm_b200.sharding import _global_fold
    B, T, C, D, A, k, world = 8, 70, 4, 3, 1_000_003, 2, 8
    assert _composite_key_dtype(B, T, C, A) == torch.int64
    assert _composite_key_dtype(B // world, T, C, A) == torch.int32
    g = torch.Generator().manual_seed(5)
    # addresses far outside int32: their low 32 bits and their true value fold differently
    w = torch.randint(-(1 << 40), 1 << 40, (B, T, C), generator=g, dtype=torch.int64)
    w[:, 1::3] = w[:, 0:-1:3]  # exact repeats: hits under either rule
    w[:, 2::3] = w[:, 0:-2:3] + (1 << 32)  # equal low 32 bits: a hit only after truncation
    p = torch.randn(B, T, C, D, generator=g)
    ev, em, _, _ = oracle.latestk_fwd(w.numpy(), p.numpy(), address_space=A, k=k)
    folded_differs = False
    for sh in all_shards(B, C, world):
        ws = sh.take(w)
        fv, fm, _, _ = oracle.latestk_fwd(_global_fold(ws, sh, T, A).numpy(), sh.take(p).numpy(),
                                          address_space=A, k=k)
        assert np.array_equal(fm, em[sh.b0:sh.b1, :, sh.c0:sh.c1])
        assert np.array_equal(fv * fm[..., None], ev[sh.b0:sh.b1, :, sh.c0:sh.c1] * fm[..., None])
        _, raw_m, _, _ = oracle.latestk_fwd(ws.numpy(), sh.take(p).numpy(), address_space=A, k=k)
        folded_differs |= not np.array_equal(raw_m, fm)
    assert folded_differs, "the case does not exercise the truncation"


def test_global_fold_leaves_equal_rules_alone():
    from ravel_lm_b200.sharding import _global_fold
    sh = shard_streams(4, 16, 2, 1)
    a = torch.arange(-5, 5, dtype=torch.int64).view(1, 10, 1).expand(2, 10, 16).contiguous()
    assert _global_fold(a, sh, 10, 7) is a
    a32 = a.to(torch.int32)
    assert _global_fold(a32, sh, 10, 7) is a32


def _failing_worker(rank, world, port, out_q):
    """Rank 1 fails before the collective; rank 0's gather must end with an error, not hang."""
    import datetime

    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    try:
        from ravel_lm_b200.sharding import gather_outputs
        sh = shard_streams(2, 4, world, rank)
        if rank == 1:
            raise RuntimeError("injected failure on rank 1")
        try:
            gather_outputs(torch.zeros(1, 3, 4, 2), sh)
            out_q.put("no error")
        except Exception as exc:  # the process group's timeout or the peer's disconnect
            out_q.put(type(exc).__name__)
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def test_a_rank_that_fails_before_the_all_gather_is_detected():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(g, 2, port, q)) for g in range(2)]
    for pr in procs:
        pr.start()
    for pr in procs:
        pr.join(timeout=90)
    for pr in procs:
        if pr.is_alive():
            pr.kill()
    assert procs[1].exitcode != 0
    got = q.get(timeout=5)
    assert got != "no error", "rank 0 must see the failure as an error"
