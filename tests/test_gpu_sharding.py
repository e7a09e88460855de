"""Stream sharding with the CUDA kernels computing every shard.

* One GPU: ``sharded_lookup`` is called for every rank of worlds 2, 4 and 8
  in turn (batch-row split and head split), the pieces are put back together
  and compared with the unsharded call, for both lookups, for full inputs and
  for inputs the caller has already sliced (``full_shape``), and for int64
  addresses whose truncation rule depends on the whole problem's size.
* Two GPUs (skipped with fewer): two processes over NCCL, each computing its
  own shard, with ``replicate=True`` (one all-gather per output); rank 0
  compares the replicated result with the unsharded call.
"""
from __future__ import annotations

import datetime
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import ravel_lm_b200._lib as L
    L.load()
    yield
    torch.cuda.synchronize()
    assert L.device_error(torch.cuda.current_stream().cuda_stream) == 0


def _case(B, T, C, D, A, seed, *, wide=False):
    g = torch.Generator(device="cuda").manual_seed(seed)
    if wide:
        w = torch.randint(-(1 << 40), 1 << 40, (B, T, C), generator=g, device="cuda")
        w[:, 1::3] = w[:, 0:-1:3]
        w[:, 2::3] = w[:, 0:-2:3] + (1 << 32)
        r = None
        m = None
    else:
        w = torch.randint(0, A, (B, T, C), generator=g, device="cuda")
        r = torch.randint(0, A, (B, T, C), generator=g, device="cuda")
        m = torch.rand(B, T, generator=g, device="cuda") < 0.75
    p = torch.randn(B, T, C, D, generator=g, device="cuda")
    return w, p, r, m


def _check(full, pieces, shards, mask_full, mask_pieces, exact):
    from ravel_lm_b200.sharding import assemble
    got = assemble(pieces, shards)
    got_mask = assemble(mask_pieces, shards)
    assert torch.equal(got_mask, mask_full)
    mk = mask_full.unsqueeze(-1).to(full.dtype)
    if exact:
        # the sign of an invalid slot's zero may differ at a stream's start (see sharding.py)
        assert torch.equal(got * mk, full * mk)
    else:
        torch.testing.assert_close(got, full, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("use_sum", [False, True])
def test_every_rank_of_a_world_on_one_gpu(world, use_sum):
    from ravel_lm_b200 import causal_last_k_lookup, causal_sum_lookup
    from ravel_lm_b200.sharding import all_shards, sharded_lookup
    B, T, C, D, A, k = 4, 2000, 8, 16, 500, 3
    w, p, r, m = _case(B, T, C, D, A, seed=world)
    if use_sum:
        full, fmask = causal_sum_lookup(w, p, r, address_space=A, write_mask=m)
    else:
        full, fmask = causal_last_k_lookup(w, p, r, address_space=A, k=k, write_mask=m)
    shards = all_shards(B, C, world)
    assert shards[0].splits_heads == (world > B)
    for presliced in (False, True):
        vals, masks = [], []
        for sh in shards:
            if presliced:
                args = (sh.take(w), sh.take(p), sh.take(r))
                kw = dict(write_mask=sh.take(m, head_dim=False), full_shape=(B, C))
            else:
                args, kw = (w, p, r), dict(write_mask=m)
            v, mk = sharded_lookup(*args, address_space=A, k=k, world=world, rank=sh.rank, use_sum=use_sum, **kw)
            vals.append(v)
            masks.append(mk)
        _check(full, vals, shards, fmask, masks, exact=not use_sum)


def test_presliced_inputs_of_the_wrong_shape_are_rejected():
    from ravel_lm_b200.sharding import sharded_lookup
    w, p, r, m = _case(4, 64, 8, 4, 50, seed=3)
    with pytest.raises(ValueError):
        sharded_lookup(w[:1], p[:1], address_space=50, world=2, rank=0, full_shape=(4, 8))


def test_wide_int64_addresses_follow_the_whole_problems_key_rule():
    from ravel_lm_b200 import causal_last_k_lookup
    from ravel_lm_b200.sharding import all_shards, sharded_lookup
    B, T, C, D, A, k, world = 8, 70, 4, 3, 1_000_003, 2, 8
    w, p, _, _ = _case(B, T, C, D, A, seed=11, wide=True)
    full, fmask = causal_last_k_lookup(w, p, address_space=A, k=k)
    shards = all_shards(B, C, world)
    out = [sharded_lookup(w, p, address_space=A, k=k, world=world, rank=sh.rank) for sh in shards]
    _check(full, [o[0] for o in out], shards, fmask, [o[1] for o in out], exact=True)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from ravel_lm_b200 import causal_last_k_lookup, causal_sum_lookup
        from ravel_lm_b200.sharding import sharded_lookup
        B, T, C, D, A, k = 1, 3000, 8, 32, 700, 4  # B < world: the head split
        ok = True
        for use_sum in (False, True):
            w, p, r, m = _case(B, T, C, D, A, seed=21)
            vals, mask = sharded_lookup(w, p, r, address_space=A, k=k, write_mask=m, world=world, rank=rank,
                                        replicate=True, use_sum=use_sum)
            if use_sum:
                fv, fm = causal_sum_lookup(w, p, r, address_space=A, write_mask=m)
                ok &= torch.equal(mask, fm) and torch.allclose(vals, fv, rtol=1e-5, atol=1e-5)
            else:
                fv, fm = causal_last_k_lookup(w, p, r, address_space=A, k=k, write_mask=m)
                mk = fm.unsqueeze(-1).float()
                ok &= torch.equal(mask, fm) and torch.equal(vals * mk, fv * mk)
        torch.cuda.synchronize()
        q.put((rank, bool(ok)))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_gpus_over_nccl_replicated_outputs():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_worker, args=(g, 2, port, q)) for g in range(2)]
    for pr in procs:
        pr.start()
    for pr in procs:
        pr.join(timeout=180)
    for pr in procs:
        if pr.is_alive():
            pr.kill()
    assert all(pr.exitcode == 0 for pr in procs), [pr.exitcode for pr in procs]
    res = dict(q.get(timeout=5) for _ in range(2))
    assert res == {0: True, 1: True}
