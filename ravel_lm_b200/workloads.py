"""Seeded synthetic inputs for the operator at the five benchmark configurations.

No dataset is involved anywhere: every configuration of the benchmark is
synthetic by definition (address distributions, payloads and gradients drawn
from fixed seeds).  Inputs are generated on the CPU with
``torch.Generator().manual_seed(seed)`` in the order addresses, payloads,
grad_out, so the same seed gives the same tensors on every machine.

Configurations (B, T, C = memory heads, D, A = address space, k):
  1  latest-1 literal byte addresses, Zipf(1.1) over 256     8 x 256 x 4,  D16 fp32, k1
  2  product-code addresses c1*64+c2, uniform, A=4096        16 x 2048 x 8, D32 fp32, k4
  3  long-context prefill, Zipf(1.05) over 65536             4 x 32768 x 16, D64 bf16, k8
  4  decode cache: 256 streams, H=16, A=4096 uniform, D64 bf16
  5  model-shaped: 4 literal heads from token hashes of Zipf(1.1) token ids over
     1024 (the hashes of ravel_lm/model.py:195-231) + 4 learned product-code
     heads 32x32 with independent read/write codes; B=8 per GPU, T=1024, D32
     fp32, k2
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional

import torch


@dataclass(frozen=True)
class Config:
    cfg: int
    B: int
    T: int
    C: int
    D: int
    A: int
    k: int
    dtype: torch.dtype
    addressing: str
    zipf_s: float = 0.0
    backward: bool = True
    extra: dict = field(default_factory=dict)

    @property
    def N(self) -> int:
        return self.B * self.T * self.C

    @property
    def tokens(self) -> int:
        return self.B * self.T

    def with_batch(self, B: int) -> "Config":
        return Config(self.cfg, B, self.T, self.C, self.D, self.A, self.k, self.dtype, self.addressing,
                      self.zipf_s, self.backward, dict(self.extra))


CONFIGS = {
    1: Config(1, 8, 256, 4, 16, 256, 1, torch.float32, "zipf", 1.1, backward=False),
    2: Config(2, 16, 2048, 8, 32, 4096, 4, torch.float32, "product64", backward=True),
    3: Config(3, 4, 32768, 16, 64, 65536, 8, torch.bfloat16, "zipf", 1.05, backward=True),
    5: Config(5, 8, 1024, 8, 32, 1024, 2, torch.float32, "model", 1.1, backward=True,
              extra={"literal_heads": 4, "vocab": 1024, "codebook": 32}),
}

DECODE = {"streams": 256, "H": 16, "A": 4096, "D": 64, "dtype": torch.bfloat16, "prefill": 4096, "steps": 1024}


def zipf_ranks(n: int, s: float, shape, gen: torch.Generator) -> torch.Tensor:
    """rank-1 of a finite Zipf(s) over n values (p proportional to r^-s)."""
    dev = gen.device
    p = torch.arange(1, n + 1, dtype=torch.float64, device=dev).pow(-s)
    p = p / p.sum()
    numel = 1
    for x in shape:
        numel *= x
    # inverse-CDF sampling (multinomial caps the category count)
    cdf = torch.cumsum(p, 0)
    u = torch.rand(numel, generator=gen, dtype=torch.float64, device=dev)
    idx = torch.searchsorted(cdf, u).clamp_max(n - 1)
    return idx.view(*shape).to(torch.int64)


def literal_hash_heads(tokens: torch.Tensor, n_heads: int, A: int, bos: int = 0) -> torch.Tensor:
    """Literal address families from token ids (ravel_lm/model.py:195-231)."""
    B, T = tokens.shape
    toks = tokens.long()
    dev = toks.device
    heads = []
    if n_heads >= 1:
        heads.append(toks.remainder(A))
    prev1 = torch.cat([torch.full((B, 1), bos, dtype=torch.long, device=dev), toks[:, :-1]], dim=1)
    prev2 = torch.cat([torch.full((B, 2), bos, dtype=torch.long, device=dev), toks[:, :-2]], dim=1)
    if n_heads >= 2:
        heads.append((prev1 * 257 + toks * 131 + 17).remainder(A))
    if n_heads >= 3:
        heads.append((prev2 * 65537 + prev1 * 257 + toks * 131 + 31).remainder(A))
    pos = torch.arange(T, dtype=torch.long, device=dev).view(1, T).expand(B, T)
    for j in range(3, n_heads):
        heads.append((toks * (1009 + 2 * j) + pos * (9176 + j) + j * 97).remainder(A))
    return torch.stack(heads, dim=-1)


def make_inputs(cfg: Config, seed: Optional[int] = None, *, grads: bool = True, device: str = "cpu") -> dict:
    """Tensors write, read (None when reads alias writes), payload, g_vals, g_sums.

    Generated on ``device`` with a generator of that device (CPU and CUDA
    streams of random numbers differ, so tests that compare against the CPU
    oracle generate on the CPU).
    """
    dev = torch.device(device)
    gen = torch.Generator(device=dev).manual_seed(1000 + cfg.cfg if seed is None else seed)
    B, T, C, D, A = cfg.B, cfg.T, cfg.C, cfg.D, cfg.A
    read = None
    if cfg.addressing == "zipf":
        write = zipf_ranks(A, cfg.zipf_s, (B, T, C), gen)
    elif cfg.addressing == "product64":
        c1 = torch.randint(0, 64, (B, T, C), generator=gen, device=dev)
        c2 = torch.randint(0, 64, (B, T, C), generator=gen, device=dev)
        write = c1 * 64 + c2
    elif cfg.addressing == "uniform":
        write = torch.randint(0, A, (B, T, C), generator=gen, device=dev)
    elif cfg.addressing == "model":
        lit = cfg.extra["literal_heads"]
        cb = cfg.extra["codebook"]
        toks = zipf_ranks(cfg.extra["vocab"], cfg.zipf_s, (B, T), gen)
        literal = literal_hash_heads(toks, lit, A)
        nl = C - lit

        def code():
            return (torch.randint(0, cb, (B, T, nl), generator=gen, device=dev) * cb
                    + torch.randint(0, cb, (B, T, nl), generator=gen, device=dev))
        wl = code()
        rl = code()
        write = torch.cat([literal, wl.remainder(A)], -1)
        read = torch.cat([literal, rl.remainder(A)], -1)
    else:
        raise ValueError(cfg.addressing)
    payload = torch.randn(B, T, C, D, generator=gen, dtype=torch.float32, device=dev).to(cfg.dtype)
    out = {"write": write.contiguous(), "read": None if read is None else read.contiguous(), "payload": payload}
    if grads and cfg.backward:
        out["g_vals"] = torch.randn(B, T, C, cfg.k, D, generator=gen, dtype=torch.float32, device=dev).to(cfg.dtype)
        out["g_sums"] = torch.randn(B, T, C, D, generator=gen, dtype=torch.float32, device=dev).to(cfg.dtype)
    return out


def algorithmic_bytes(cfg: Config, *, aliased_reads: bool = True) -> dict:
    """Bytes each op must move at minimum (addresses int64, read once if aliased)."""
    N, D, k = cfg.N, cfg.D, cfg.k
    e = torch.finfo(cfg.dtype).bits // 8
    aw = 8
    ar = 0 if aliased_reads else 8
    return {
        "lk_fwd": N * (aw + ar + D * e + k * D * e + k),
        "ss_fwd": N * (aw + ar + 2 * D * e + 1),
        "lk_bwd": N * (aw + ar + k * D * e + D * e),
        "ss_bwd": N * (aw + ar + 2 * D * e),
    }
