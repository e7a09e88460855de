"""Generate golden vectors from the reference's own Python implementation.

Run in a container where the ravel-lm reference tree is available:

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py /path/to/ravel-lm

It imports ``ravel_lm.ravel_memory`` from that tree (read-only: bytecode
writing is disabled), runs ``causal_last_k_lookup``, ``causal_sum_lookup``,
their autograd backward passes and ``RavelLayerCache`` on small seeded inputs,
and writes one ``.npz`` per case next to this script.  The reference cannot be
shipped to the GPU machine, so these committed fixtures are how the oracle and
the CUDA path are pinned to it.

Cases re-express the reference's own known-answer tests
(tests/test_memory.py:16-79, tests/test_triton_memory.py:12-50,
tests/test_metal_kernels.py:18-64) plus seeded cases covering every option of
the operator: read != write, write_mask, k > 1, int32 / int64 / negative /
out-of-int32 addresses, float32 / bfloat16 / float16 / float64 payloads, odd D,
T = 1, a single address, all writes masked, and the first rows of each
benchmark configuration at reduced T.

Stored per case (``None`` inputs are omitted):
  waddr, raddr, wmask, payload (bf16 as uint16 bits), A, k, dtype
  lk_vals (bits for bf16), lk_mask, ss_sums64, ss_mask,
  lk_grad64, ss_grad64 (reference run on payloads.double()), g_lk, g_ss.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

sys.dont_write_bytecode = True
HERE = Path(__file__).resolve().parent


def _import_reference(root: str):
    sys.path.insert(0, root)
    from ravel_lm import ravel_memory  # noqa: E402
    return ravel_memory


def _bits(t: torch.Tensor) -> np.ndarray:
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()
    return t.detach().contiguous().numpy().copy()


def _zipf(rng: np.random.Generator, n: int, s: float, size) -> np.ndarray:
    p = np.arange(1, n + 1, dtype=np.float64) ** (-s)
    p /= p.sum()
    return rng.choice(n, size=size, p=p).astype(np.int64)


def run_case(rm, name: str, waddr, payload: torch.Tensor, raddr=None, wmask=None, *, A: int, k: int,
             grad_seed: int = 0):
    out = {"A": np.int64(A), "k": np.int64(k), "dtype": np.array(str(payload.dtype).replace("torch.", ""))}
    w = torch.as_tensor(waddr)
    r = None if raddr is None else torch.as_tensor(raddr)
    m = None if wmask is None else torch.as_tensor(wmask, dtype=torch.bool)
    out["waddr"] = w.numpy().copy()
    if r is not None:
        out["raddr"] = r.numpy().copy()
    if m is not None:
        out["wmask"] = m.numpy().astype(np.uint8)
    out["payload"] = _bits(payload)

    vals, mask = rm.causal_last_k_lookup(w, payload, r, address_space=A, k=k, write_mask=m)
    out["lk_vals"] = _bits(vals)
    out["lk_mask"] = mask.numpy().astype(np.uint8)

    g = torch.Generator().manual_seed(grad_seed)
    p64 = payload.detach().double().requires_grad_(True)
    v64, _ = rm.causal_last_k_lookup(w, p64, r, address_space=A, k=k, write_mask=m)
    g_lk = torch.randn(v64.shape, generator=g, dtype=torch.float32)
    if v64.requires_grad:
        (v64 * g_lk.double()).sum().backward()
    out["lk_grad64"] = p64.grad.numpy().copy() if p64.grad is not None else np.zeros(p64.shape)
    out["g_lk"] = g_lk.numpy()

    q64 = payload.detach().double().requires_grad_(True)
    s64, smask = rm.causal_sum_lookup(w, q64, r, address_space=A, write_mask=m)
    g_ss = torch.randn(s64.shape, generator=g, dtype=torch.float32)
    if s64.requires_grad:
        (s64 * g_ss.double()).sum().backward()
    out["ss_sums64"] = s64.detach().numpy().copy()
    out["ss_mask"] = smask.numpy().astype(np.uint8)
    out["ss_grad64"] = q64.grad.numpy().copy() if q64.grad is not None else np.zeros(q64.shape)
    out["g_ss"] = g_ss.numpy()
    np.savez_compressed(HERE / f"{name}.npz", **out)
    print(f"{name}: B,T,C={tuple(w.shape)} D={payload.shape[-1]} A={A} k={k} {payload.dtype}")


def cache_case(rm):
    """tests/test_memory.py:70-79 plus a seeded write/read sequence with clamping."""
    rng = np.random.default_rng(5)
    B, C, A, D = 2, 3, 16, 4
    cache = rm.RavelLayerCache.empty(B, C, A, D, device="cpu", dtype=torch.float32)
    steps = 12
    raddr = rng.integers(-3, A + 3, size=(steps, B, C))
    waddr = rng.integers(-3, A + 3, size=(steps, B, C))
    pay = rng.normal(size=(steps, B, C, D)).astype(np.float32)
    pay[pay > 1.5] *= -1.0
    vals_out, mask_out = [], []
    for s in range(steps):
        v, m = cache.read(torch.from_numpy(raddr[s]))
        vals_out.append(v.numpy().copy())
        mask_out.append(m.numpy().astype(np.uint8))
        cache.write(torch.from_numpy(waddr[s]), torch.from_numpy(pay[s]))
    np.savez_compressed(HERE / "cache_sequence.npz", raddr=raddr, waddr=waddr, payload=pay,
                        vals=np.stack(vals_out), mask=np.stack(mask_out),
                        final_values=cache.values.numpy(), final_filled=cache.filled.numpy().astype(np.uint8),
                        B=B, C=C, A=A, D=D)
    print("cache_sequence")


def main(root: str) -> None:
    rm = _import_reference(root)

    # tests/test_memory.py:11-13
    np.savez_compressed(HERE / "key_dtype.npz",
                        cases=np.array([[1, 2048, 3, 1024], [1024, 65536, 64, 65536],
                                        [8, 256, 4, 256], [16, 2048, 8, 4096], [4, 32768, 16, 65536],
                                        [1, 1, 1, 2147483647], [1, 1, 1, 1073741823]], dtype=np.int64),
                        is_int32=np.array([rm._composite_key_dtype(*c) == torch.int32 for c in
                                           [(1, 2048, 3, 1024), (1024, 65536, 64, 65536), (8, 256, 4, 256),
                                            (16, 2048, 8, 4096), (4, 32768, 16, 65536),
                                            (1, 1, 1, 2147483647), (1, 1, 1, 1073741823)]]))

    # tests/test_memory.py:16-23
    run_case(rm, "kat_latest", [[[1], [2], [1], [3], [1]]],
             torch.arange(5, dtype=torch.float32).view(1, 5, 1, 1), A=8, k=2)
    # tests/test_memory.py:26-58
    torch.manual_seed(0)
    run_case(rm, "kat_separate_mask", [[[1], [2], [1], [3], [2], [1]]], torch.randn(1, 6, 1, 3),
             [[[1], [1], [2], [1], [2], [3]]], [[True, True, False, True, True, True]], A=8, k=2)
    # tests/test_memory.py:61-67
    run_case(rm, "kat_sum", [[[1], [2], [1], [1]]], torch.tensor([1.0, 10.0, 3.0, 7.0]).view(1, 4, 1, 1),
             A=8, k=1)
    # tests/test_triton_memory.py:12-50 (B2 T17 C3 D5 A11 seed 7, read != write)
    torch.manual_seed(7)
    B, T, C, D, A = 2, 17, 3, 5, 11
    w = torch.randint(0, A, (B, T, C))
    r = torch.randint(0, A, (B, T, C))
    run_case(rm, "triton_parity", w, torch.randn(B, T, C, D), r, A=A, k=1)
    # tests/test_metal_kernels.py:18-46 (with write_mask) and :48-64 (D=5 tail)
    rng = np.random.default_rng(0)
    B, T, C, D, A = 2, 7, 3, 4, 8
    w = rng.integers(0, A, size=(B, T, C)).astype(np.int64)
    r = rng.integers(0, A, size=(B, T, C)).astype(np.int64)
    p = rng.normal(size=(B, T, C, D)).astype(np.float32)
    m = rng.integers(0, 2, size=(B, T)).astype(bool)
    run_case(rm, "metal_mask", w, torch.from_numpy(p), r, m, A=A, k=1)
    rng = np.random.default_rng(4)
    B, T, C, D, A = 1, 13, 2, 5, 16
    w = rng.integers(0, A, size=(B, T, C)).astype(np.int64)
    r = rng.integers(0, A, size=(B, T, C)).astype(np.int64)
    p = rng.normal(size=(B, T, C, D)).astype(np.float32)
    run_case(rm, "metal_tail", w, torch.from_numpy(p), r, A=A, k=1)

    # Seeded cases over the operator's options.
    rng = np.random.default_rng(1234)
    # config-1 shape at reduced B: latest-1 literal byte addresses, Zipf(1.1) over 256
    w = _zipf(rng, 256, 1.1, (1, 256, 4))
    run_case(rm, "cfg1_small", w, torch.from_numpy(rng.normal(size=(1, 256, 4, 16)).astype(np.float32)),
             A=256, k=1)
    # config-2 shape at reduced B,T: product-code addresses, k=4
    c1 = rng.integers(0, 64, size=(1, 128, 4))
    c2 = rng.integers(0, 64, size=(1, 128, 4))
    run_case(rm, "cfg2_small", c1 * 64 + c2,
             torch.from_numpy(rng.normal(size=(1, 128, 4, 32)).astype(np.float32)), A=4096, k=4)
    # config-3 shape at reduced B,T,C: bf16 payloads, Zipf(1.05) over 65536, k=8
    w = _zipf(rng, 65536, 1.05, (1, 128, 2))
    pay = torch.from_numpy(rng.normal(size=(1, 128, 2, 64)).astype(np.float32)).bfloat16()
    run_case(rm, "cfg3_small_bf16", w, pay, A=65536, k=8)
    # read != write, write_mask, k=3, negative addresses, int32 dtype
    w = rng.integers(-40, 40, size=(3, 50, 5)).astype(np.int32)
    r = rng.integers(-40, 40, size=(3, 50, 5)).astype(np.int32)
    m = rng.random((3, 50)) < 0.6
    run_case(rm, "general_mask_neg_i32", w, torch.from_numpy(rng.normal(size=(3, 50, 5, 7)).astype(np.float32)),
             r, m, A=23, k=3)
    # int64 addresses beyond int32 with int32 keys (truncation before remainder)
    pool = rng.integers(-2**40, 2**40, size=12).astype(np.int64)
    w = pool[rng.integers(0, 12, size=(2, 33, 2))]
    r = w.copy()
    r[:, 5:9] = pool[rng.integers(0, 12, size=(2, 4, 2))]
    run_case(rm, "wide_i64_key32", w, torch.from_numpy(rng.normal(size=(2, 33, 2, 8)).astype(np.float32)),
             r, A=1000, k=2)
    # int64 keys (bound beyond int32): A large
    w = rng.integers(0, 3, size=(2, 40, 3)).astype(np.int64) * 2**30 + rng.integers(0, 3, size=(2, 40, 3))
    run_case(rm, "key64", w, torch.from_numpy(rng.normal(size=(2, 40, 3, 4)).astype(np.float32)),
             A=2**31, k=2)
    # f16 payloads, k=5, small A (long segments)
    w = rng.integers(0, 3, size=(2, 80, 2)).astype(np.int64)
    run_case(rm, "f16_k5", w, torch.from_numpy(rng.normal(size=(2, 80, 2, 12)).astype(np.float32)).half(),
             A=3, k=5)
    # f64 payloads, D=1, odd sizes, mask
    w = rng.integers(0, 6, size=(3, 21, 3)).astype(np.int64)
    m = rng.random((3, 21)) < 0.5
    run_case(rm, "f64_d1_mask", w, torch.from_numpy(rng.normal(size=(3, 21, 3, 1))), None, m, A=6, k=2)
    # T = 1
    run_case(rm, "t1", rng.integers(0, 4, size=(3, 1, 2)),
             torch.from_numpy(rng.normal(size=(3, 1, 2, 6)).astype(np.float32)), A=4, k=2)
    # single address everywhere (one segment per stream), negative payloads to expose -0.0
    pay = -np.abs(rng.normal(size=(2, 40, 2, 8))).astype(np.float32)
    run_case(rm, "one_address", np.zeros((2, 40, 2), np.int64), torch.from_numpy(pay), A=1, k=4)
    # all writes masked -> zeros + false
    run_case(rm, "all_masked", rng.integers(0, 5, size=(2, 9, 2)),
             torch.from_numpy(rng.normal(size=(2, 9, 2, 3)).astype(np.float32)),
             rng.integers(0, 5, size=(2, 9, 2)), np.zeros((2, 9), bool), A=5, k=2)
    # one batch row fully masked (empty streams in the middle of the tape)
    m = np.ones((3, 30), bool)
    m[1] = False
    run_case(rm, "empty_stream_mask", rng.integers(0, 7, size=(3, 30, 2)),
             torch.from_numpy(rng.normal(size=(3, 30, 2, 4)).astype(np.float32)),
             rng.integers(0, 7, size=(3, 30, 2)), m, A=7, k=3)
    # config-5 style: literal heads read == write, learned heads read != write
    toks = _zipf(rng, 1024, 1.1, (2, 64))
    lit = np.stack([toks % 1024, (np.roll(toks, 1, 1) * 257 + toks * 131 + 17) % 1024], -1)
    wl = rng.integers(0, 32, size=(2, 64, 2)) * 32 + rng.integers(0, 32, size=(2, 64, 2))
    rl = rng.integers(0, 32, size=(2, 64, 2)) * 32 + rng.integers(0, 32, size=(2, 64, 2))
    run_case(rm, "cfg5_small", np.concatenate([lit, wl], -1),
             torch.from_numpy(rng.normal(size=(2, 64, 4, 32)).astype(np.float32)),
             np.concatenate([lit, rl], -1), A=1024, k=2)
    cache_case(rm)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_golden.py <path to the ravel-lm reference tree>")
    main(sys.argv[1])
