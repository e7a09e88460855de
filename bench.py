#!/usr/bin/env python
"""Benchmark of RAVEL's exact event-memory operator on B200.

One step = the operator's full training pass on one batch of synthetic input:
causal_last_k_lookup + causal_sum_lookup forward and backward, through the
public drop-in API (autograd), on benchmark configuration 3 by default
(B=4 T=32768 H=16 D=64 bf16, k=8, Zipf(1.05) addresses over 65536).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Multi-GPU (weak scaling): one process per GPU under torchrun; rank r owns
batch rows [4r, 4r+4) of a global batch of 4N, i.e. its own 64 streams.
Streams never interact, so there is no collective on the data path; NCCL is
used only for the barrier and the max over ranks of the step time.

The JSON line carries the device-timed throughput (``value``), the roofline
of the dominant kernel (CUDA events around its entry point inside the timed
region), an end-to-end number through the API with pinned host buffers
(``e2e``), the CPU oracle port timed on the host (``cpu_baseline``, rank 0 at
N=1), decode microseconds per step for configuration 4, and the SM clocks
sampled during the timed region.

``--impl reference`` times the CPU port of the reference's algorithm
(oracle/, OpenMP over all host cores) on a bounded sample of the same
workload; under torchrun only rank 0 works.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from collections import defaultdict
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

DTYPE_NAMES = {"torch.bfloat16": "bf16", "torch.float32": "f32", "torch.float16": "f16", "torch.float64": "f64"}
METRIC = "RAVEL memory-op tokens/sec/GPU + % HBM roofline at 1/2/4/8 B200; decode µs/step"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", type=int, default=3, choices=[2, 3, 5])
    ap.add_argument("--e2e-steps", type=int, default=8)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-decode", action="store_true")
    ap.add_argument("--no-general", action="store_true",
                    help="skip the extra timing of the general path (reads drawn apart from the writes)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-reference-gpu", action="store_true",
                    help="skip timing the reference's own functions on CUDA tensors (needs baseline/_ref)")
    ap.add_argument("--cpu-streams", type=int, default=8, help="streams in the CPU baseline sample")
    ap.add_argument("--batch", type=int, default=None, help="override B per GPU (small profiling cases)")
    ap.add_argument("--ops", choices=["all", "lk", "ss"], default="all",
                    help="ops in a step (profiling a single op; the benchmark runs all)")
    return ap.parse_args()


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi samples every 200 ms while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.gpu_id = gpu_id
        self.lines: list[str] = []
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", self.gpu_id, f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (OSError, FileNotFoundError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, power, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
                power.append(float(parts[3]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "power_w_max": max(power) if power else None, "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------- distributed
def dist_setup():
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180))
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch
        import torch.distributed as dist
        dist.barrier(device_ids=[torch.cuda.current_device()])


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------- CPU port (reference arm, cpu_baseline)
def cpu_sample(cfg, n_streams: int, seed: int = 4242):
    """A bounded sample of the workload: the first n_streams (b, c) streams."""
    import numpy as np
    import torch
    from ravel_lm_b200.workloads import make_inputs
    sub = cfg.with_batch(1)
    x = make_inputs(sub, seed=seed)
    C = min(n_streams, cfg.C)
    w = x["write"][:, :, :C].contiguous().numpy()
    r = None if x["read"] is None else x["read"][:, :, :C].contiguous().numpy()
    p = x["payload"][:, :, :C].contiguous()
    gv = x["g_vals"][:, :, :C].contiguous()
    gs = x["g_sums"][:, :, :C].contiguous()
    code = {torch.bfloat16: "bf16", torch.float16: "f16"}.get(p.dtype)
    pbits = p.view(torch.int16).numpy().view(np.uint16) if code else p.numpy()
    return dict(w=w, r=r, p=p, pbits=pbits, code=code, gv=gv, gs=gs, streams=C, T=cfg.T,
                tokens_equiv=cfg.T * C / cfg.C)


def cpu_step(oracle, s, cfg):
    """LK fwd + SS fwd + LK bwd + SS bwd of the CPU port on the sample."""
    vals, mask, src, tape = oracle.latestk_fwd(s["w"], s["pbits"], s["r"], address_space=cfg.A, k=cfg.k,
                                               dtype=s["code"])
    sums, smask, _ = oracle.segsum_fwd(s["w"], s["p"].double().numpy(), s["r"], address_space=cfg.A, tape=tape)
    B, T, C, D = s["p"].shape
    g1 = oracle.latestk_bwd(mask, src, s["gv"].double().numpy(), B * T * C)
    g2 = oracle.segsum_bwd(tape, smask, s["gs"].double().numpy())
    return g1.sum() + g2.sum()


def run_cpu_baseline(cfg, steps: int, warmup: int, n_streams: int) -> dict:
    import oracle
    oracle.set_num_threads(os.cpu_count() or 1)
    s = cpu_sample(cfg, n_streams)
    for _ in range(warmup):
        cpu_step(oracle, s, cfg)
    t0 = time.perf_counter()
    for _ in range(steps):
        cpu_step(oracle, s, cfg)
    dt = (time.perf_counter() - t0) / max(steps, 1)
    return {"value": s["tokens_equiv"] / dt, "unit": "tokens/s", "cores": oracle.num_threads(), "kind": "port",
            "sample": f"{s['streams']} of {cfg.C} streams of one batch row (T={cfg.T}): latest-k k={cfg.k} + "
                      f"segmented-sum fwd+bwd, = {s['tokens_equiv']:.0f} token-equivalents; "
                      f"{steps} timed steps, {warmup} warm-up",
            "sec_per_step": dt}


# ---------------------------------------------------------------- GPU arm
def kernel_bytes(cfg) -> dict:
    """Algorithmic bytes per launch of each compute entry point."""
    import torch
    N, D, k = cfg.N, cfg.D, cfg.k
    e = torch.finfo(cfg.dtype).bits // 8
    addr = 8 * (1 if cfg.addressing != "model" else 2)
    return {
        "ravel_tape_build": N * addr,
        "ravel_latestk_fwd_tape": N * (D * e + k * D * e + k),
        "ravel_latestk_bwd": N * (k * D * e + D * e),
        "ravel_segsum_fwd_tape": N * (2 * D * e + 1),
        "ravel_segsum_bwd": N * (2 * D * e),
    }


def gpu_uuid(dev) -> str:
    import torch
    try:
        return "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        return str(dev.index or 0)


def run_decode(dev) -> dict:
    import torch
    from ravel_lm_b200 import RavelLayerCache
    from ravel_lm_b200.workloads import DECODE
    S, H, A, D, dt = DECODE["streams"], DECODE["H"], DECODE["A"], DECODE["D"], DECODE["dtype"]
    steps = DECODE["steps"]
    g = torch.Generator(device=dev).manual_seed(1004)
    P = DECODE["prefill"]
    pa = torch.randint(0, A, (S, P, H), generator=g, device=dev)
    pp = torch.randn(S, P, H, D, generator=g, device=dev).to(dt)
    # prefill of 4096 prior writes: token by token (one write per position, as the
    # reference's generate() does) and in bulk (one sort + one copy); same state
    cache = RavelLayerCache.empty(S, H, A, D, device=dev, dtype=dt)
    bulk = RavelLayerCache.empty(S, H, A, D, device=dev, dtype=dt)
    bulk.prefill(pa, pp)  # warm-up (kernel loading)
    bulk.values.zero_()
    bulk.filled.zero_()
    torch.cuda.synchronize(dev)
    p0, p1, p2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
    p0.record()
    for t in range(P):
        cache.write(pa[:, t], pp[:, t])
    p1.record()
    bulk.prefill(pa, pp)
    p2.record()
    torch.cuda.synchronize(dev)
    prefill_tok_us, prefill_bulk_us = p0.elapsed_time(p1) * 1000.0, p1.elapsed_time(p2) * 1000.0
    if not (torch.equal(bulk.filled, cache.filled) and torch.equal(bulk.values, cache.values)):
        raise RuntimeError("bulk prefill differs from token-by-token prefill")
    del bulk, pa, pp
    ra = torch.randint(0, A, (steps, S, H), generator=g, device=dev)
    pay = torch.randn(steps, S, H, D, generator=g, device=dev).to(dt)
    torch.cuda.synchronize(dev)
    # eager: one read + one write launch per step through the API
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for i in range(16):
        cache.read(ra[i])
        cache.write(ra[i], pay[i])
    e0.record()
    for i in range(steps):
        cache.read(ra[i])
        cache.write(ra[i], pay[i])
    e1.record()
    torch.cuda.synchronize(dev)
    eager_us = e0.elapsed_time(e1) * 1000.0 / steps
    # graph: the 1024 fused read+write steps captured once and replayed
    stream = torch.cuda.Stream(dev)
    stream.wait_stream(torch.cuda.current_stream(dev))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        cache.step(ra[0], ra[0], pay[0])
        with torch.cuda.graph(graph, stream=stream):
            for i in range(steps):
                cache.step(ra[i], ra[i], pay[i])
    torch.cuda.current_stream(dev).wait_stream(stream)
    graph.replay()
    torch.cuda.synchronize(dev)
    g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 3
    g0.record()
    for _ in range(reps):
        graph.replay()
    g1.record()
    torch.cuda.synchronize(dev)
    graph_us = g0.elapsed_time(g1) * 1000.0 / (steps * reps)
    del graph
    step_bytes = S * H * (2 * 8 + 4 * D * 2 + 3)
    return {"config": "cfg4: 256 streams x 16 heads, A=4096 uniform, D=64 bf16, cache prefilled by 4096 writes",
            "us_per_step_graph": graph_us, "us_per_step_eager": eager_us,
            "prefill_us_token_by_token": prefill_tok_us, "prefill_us_bulk": prefill_bulk_us,
            "bytes_per_step": step_bytes, "gbs_graph": step_bytes / (graph_us * 1e-6) / 1e9,
            "target_us": 10.0}


def main():
    args = parse()
    from ravel_lm_b200.workloads import CONFIGS
    cfg = CONFIGS[args.config]
    if args.batch is not None:
        cfg = cfg.with_batch(args.batch)
    rank, world, local = (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
                          int(os.environ.get("LOCAL_RANK", "0")))

    if args.impl == "reference":
        if rank != 0:
            return
        cb = run_cpu_baseline(cfg, args.steps, args.warmup, args.cpu_streams)
        line = {"metric": METRIC, "value": cb["value"], "unit": "tokens/s", "impl": "reference",
                "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": cb["sec_per_step"] * 1000.0, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": DTYPE_NAMES[str(cfg.dtype)],
                "data": "synthetic", "config": workload_config(cfg, 1),
                "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
                "e2e": {"value": cb["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    import torch
    import ravel_lm_b200._lib as L
    from ravel_lm_b200 import causal_last_k_lookup, causal_sum_lookup
    from ravel_lm_b200.ravel_memory import clear_tape_cache
    from ravel_lm_b200.workloads import make_inputs

    rank, world, local = dist_setup()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    seed = 1000 + cfg.cfg + 7919 * rank
    x = make_inputs(cfg, seed=seed, device=dev)
    if args.ops == "ss":  # the latest-k gradient is not needed
        x["g_vals"] = None
        torch.cuda.empty_cache()
    w, r = x["write"], x["read"]
    p = x["payload"].requires_grad_(True)
    gv, gs = x["g_vals"], x["g_sums"]
    A, k = cfg.A, cfg.k

    def step():
        # Each step stands for a new batch: forget the tape of the previous step
        # (only the latest-k -> sum reuse inside one step is legitimate).
        clear_tape_cache()
        p.grad = None
        outs, grads = [], []
        if args.ops in ("all", "lk"):
            vals, _m = causal_last_k_lookup(w, p, r, address_space=A, k=k)
            outs.append(vals)
            grads.append(gv)
        if args.ops in ("all", "ss"):
            sums, _s = causal_sum_lookup(w, p, r, address_space=A)
            outs.append(sums)
            grads.append(gs)
        torch.autograd.backward(outs, grads)

    # The clock sampler starts before the warm-up, so that the warm-up steps, not
    # an idle pause, come right before the timed region (an idle GPU drops its
    # clocks and the first timed step would pay for the ramp back up).
    clocks = ClockSampler(gpu_uuid(dev))
    clocks.start()
    time.sleep(0.3)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    assert L.device_error(stream) == 0

    records = defaultdict(list)
    # events made before the timed region, so that timing each entry point adds
    # only two event records per call to the host's work
    pool = [torch.cuda.Event(enable_timing=True) for _ in range(2 * 16 * args.steps)]
    used = [0]

    def hook(name, thunk):
        i = used[0]
        if i + 2 > len(pool):
            return thunk()
        used[0] = i + 2
        e0, e1 = pool[i], pool[i + 1]
        e0.record()
        rc = thunk()
        e1.record()
        records[name].append((e0, e1))
        return rc

    barrier(world)
    torch.cuda.synchronize(dev)
    launches0 = L.kernel_launches()
    L.set_call_hook(hook)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(args.steps):
        step()
    t1.record()
    torch.cuda.synchronize(dev)
    L.set_call_hook(None)
    launches = L.kernel_launches() - launches0
    barrier(world)
    clk = clocks.stop()
    ms_local = t0.elapsed_time(t1) / args.steps
    ms = max_over_ranks(ms_local, world)
    assert L.device_error(stream) == 0, "device error word set"

    peaks = measured_peaks()
    kb = kernel_bytes(cfg)
    kernels = {}
    for name, evs in records.items():
        times = [a.elapsed_time(b) for a, b in evs]
        avg_ms = sum(times) / len(times)
        ent = {"launches": len(times), "avg_us": avg_ms * 1000.0, "share": sum(times) / (ms_local * args.steps)}
        if name in kb:
            gbs = kb[name] / (avg_ms * 1e-3) / 1e9
            ent.update({"bytes": kb[name], "gbs": gbs, "frac": gbs / peaks["hbm_gbs"]})
        kernels[name] = ent
    dom = max((n for n in kernels if n in kb), key=lambda n: kernels[n]["avg_us"] * kernels[n]["launches"])
    traffic = load_traffic(dom, cfg)
    roofline = {"bound": "hbm", "kernel": dom, "achieved": kernels[dom]["gbs"], "peak": peaks["hbm_gbs"],
                "unit": "GB/s", "frac": kernels[dom]["frac"], "traffic": traffic,
                "peak_source": f"{peaks['source']} (MEASURED_PEAKS.json hbm_gbs)" if peaks["source"] == "measured"
                else "fallback 6.65 TB/s"}
    step_bytes = sum(kb.values())  # one tape per step: the sum reuses the latest-k tape
    tokens = cfg.tokens * world
    value = tokens / (ms * 1e-3)

    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(cfg, x, dev, args.e2e_steps, world)
    general = None
    if not args.no_general and cfg.addressing == "zipf":
        general = run_general(cfg, x, dev, world)
    ref_gpu = None
    if world == 1 and not args.no_reference_gpu:
        ref_gpu = run_reference_gpu(cfg, x, dev, steps=5, warmup=args.warmup)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cb = run_cpu_baseline(cfg, 1, 1, args.cpu_streams)
        cpu = {k2: cb[k2] for k2 in ("value", "unit", "cores", "kind", "sample")}
    decode = None
    if not args.no_decode:
        del x, p, gv, gs
        torch.cuda.empty_cache()
        decode = run_decode(dev)

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": DTYPE_NAMES[str(cfg.dtype)],
            "data": "synthetic", "config": workload_config(cfg, world),
            "tokens_per_sec_per_gpu": value / world,
            "step_roofline": {"algorithmic_bytes": step_bytes, "achieved_gbs": step_bytes / (ms * 1e-3) / 1e9,
                              "frac": step_bytes / (ms * 1e-3) / 1e9 / peaks["hbm_gbs"], "peak": peaks["hbm_gbs"]},
            "roofline": roofline, "kernels": kernels, "e2e": e2e, "cpu_baseline": cpu, "decode": decode,
            "general_path": general, "reference_gpu": ref_gpu,
            "clocks": clk, "gpu_launches": launches,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        barrier(world)
        dist.destroy_process_group()


def workload_config(cfg, world) -> dict:
    return {"workload": f"cfg{cfg.cfg}: latest-k (k={cfg.k}) + causal segmented-sum, forward + backward",
            "B_per_gpu": cfg.B, "T": cfg.T, "H": cfg.C, "D": cfg.D, "A": cfg.A, "k": cfg.k,
            "addresses": cfg.addressing + (f" s={cfg.zipf_s}" if cfg.zipf_s else ""),
            "payload_dtype": str(cfg.dtype).replace("torch.", ""), "global_batch": cfg.B * world,
            "parallelism": f"batch x head streams sharded over {world} GPU(s), no collective",
            "l2": "inputs larger than L2 (no flush needed)"}


def load_traffic(kernel: str, cfg):
    """DRAM bytes per launch of the dominant kernel from the committed ncu summary, if present."""
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None
    try:
        d = json.loads(p.read_text())
        ent = d.get(f"cfg{cfg.cfg}", {}).get(kernel)
        return None if ent is None else float(ent)
    except (ValueError, OSError):
        return None


def run_reference_gpu(cfg, x, dev, steps: int = 5, warmup: int = 3) -> dict:
    """The reference's own causal_last_k_lookup + causal_sum_lookup (torch CUDA ops,
    ravel_memory.py:52-241) on the same CUDA inputs, forward + backward through
    autograd: the GPU comparator of the benchmark plan.  It runs from an installed
    copy of the reference under baseline/_ref (pip install --no-deps --target
    baseline/_ref <reference>), never from the reference's source tree."""
    import torch
    ref = ROOT / "baseline" / "_ref"
    if not (ref / "ravel_lm" / "ravel_memory.py").exists():
        return {"unavailable": "baseline/_ref holds no installed reference"}
    sys.path.insert(0, str(ref))
    try:
        from ravel_lm.ravel_memory import causal_last_k_lookup as ref_lk, causal_sum_lookup as ref_ss
    except Exception as exc:  # an install that does not import is reported, not fatal
        return {"unavailable": f"import of the installed reference failed: {exc}"[:200]}
    finally:
        sys.path.remove(str(ref))
    w, r = x["write"], x["read"]
    p = x["payload"].detach().clone().requires_grad_(True)
    gv, gs = x["g_vals"], x["g_sums"]

    def step():
        p.grad = None
        vals, _m = ref_lk(w, p, r, address_space=cfg.A, k=cfg.k)
        sums, _s = ref_ss(w, p, r, address_space=cfg.A)
        torch.autograd.backward([vals, sums], [gv, gs])

    for _ in range(warmup):
        step()
    torch.cuda.synchronize(dev)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(steps):
        step()
    t1.record()
    torch.cuda.synchronize(dev)
    ms = t0.elapsed_time(t1) / steps
    del p
    torch.cuda.empty_cache()
    return {"path": "reference ravel_lm.ravel_memory on CUDA tensors (torch ops), forward + backward",
            "ms_per_step": ms, "value": cfg.tokens / (ms * 1e-3), "unit": "tokens/s", "steps": steps,
            "warmup": warmup}


def run_general(cfg, x, dev, world, steps: int = 5) -> dict:
    """The same step with reads drawn apart from the writes (the path of the model's
    learned read heads, model.py:367-384): independent Zipf reads of the same shape."""
    import torch
    import ravel_lm_b200._lib as L
    from ravel_lm_b200 import causal_last_k_lookup, causal_sum_lookup
    from ravel_lm_b200.ravel_memory import clear_tape_cache
    from ravel_lm_b200.workloads import zipf_ranks
    g = torch.Generator(device=dev).manual_seed(2000 + cfg.cfg)
    w = x["write"]
    r = zipf_ranks(cfg.A, cfg.zipf_s, tuple(w.shape), g)
    p = x["payload"].detach().requires_grad_(True)
    gv, gs = x["g_vals"], x["g_sums"]
    records = defaultdict(list)

    def hook(name, thunk):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        rc = thunk()
        e1.record()
        records[name].append((e0, e1))
        return rc

    def step():
        clear_tape_cache()
        p.grad = None
        vals, _m = causal_last_k_lookup(w, p, r, address_space=cfg.A, k=cfg.k)
        sums, _s = causal_sum_lookup(w, p, r, address_space=cfg.A)
        torch.autograd.backward([vals, sums], [gv, gs])

    for _ in range(2):
        step()
    torch.cuda.synchronize(dev)
    L.set_call_hook(hook)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(steps):
        step()
    t1.record()
    torch.cuda.synchronize(dev)
    L.set_call_hook(None)
    ms = max_over_ranks(t0.elapsed_time(t1) / steps, world)
    per = {n: sum(a.elapsed_time(b) for a, b in v) / len(v) * 1000.0 for n, v in records.items()}
    return {"reads": f"independent Zipf(s={cfg.zipf_s}) reads of the same shape", "ms_per_step": ms,
            "value": cfg.tokens * world / (ms * 1e-3), "unit": "tokens/s", "steps": steps,
            "kernels_us": per}


def run_e2e(cfg, x, dev, steps, world):
    """The same step through the public API from pinned host buffers, with copies in the timed region."""
    import torch
    from ravel_lm_b200 import causal_last_k_lookup, causal_sum_lookup
    from ravel_lm_b200.ravel_memory import clear_tape_cache
    host = {n: x[n].detach().to("cpu").pin_memory() for n in ("write", "payload", "g_vals", "g_sums")}
    if x["read"] is not None:
        host["read"] = x["read"].to("cpu").pin_memory()
    B, T, C, D, k = cfg.B, cfg.T, cfg.C, cfg.D, cfg.k
    out = {"vals": torch.empty(B, T, C, k, D, dtype=cfg.dtype).pin_memory(),
           "mask": torch.empty(B, T, C, k, dtype=torch.bool).pin_memory(),
           "sums": torch.empty(B, T, C, D, dtype=cfg.dtype).pin_memory(),
           "smask": torch.empty(B, T, C, dtype=torch.bool).pin_memory(),
           "grad": torch.empty(B, T, C, D, dtype=cfg.dtype).pin_memory()}
    h2d = sum(t.numel() * t.element_size() for t in host.values())
    d2h = sum(t.numel() * t.element_size() for t in out.values())

    # Three streams, as a serving or training pipeline runs them: step i+1's inputs
    # cross PCIe (host->device) while step i's results cross back (device->host);
    # PCIe is full duplex.  Every step still copies all of its own inputs from
    # pinned host memory and all of its results back, inside the timed region.
    s_in, s_cmp, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev), torch.cuda.Stream(dev)

    def one():
        with torch.cuda.stream(s_in):
            w = host["write"].to(dev, non_blocking=True)
            r = host["read"].to(dev, non_blocking=True) if "read" in host else None
            p = host["payload"].to(dev, non_blocking=True)
            gv = host["g_vals"].to(dev, non_blocking=True)
            gs = host["g_sums"].to(dev, non_blocking=True)
            ev_in = torch.cuda.Event()
            ev_in.record(s_in)
        with torch.cuda.stream(s_cmp):
            s_cmp.wait_event(ev_in)
            for t in (w, r, p, gv, gs):
                if t is not None:
                    t.record_stream(s_cmp)
            clear_tape_cache()
            p.requires_grad_(True)
            vals, mask = causal_last_k_lookup(w, p, r, address_space=cfg.A, k=k)
            sums, smask = causal_sum_lookup(w, p, r, address_space=cfg.A)
            torch.autograd.backward([vals, sums], [gv, gs])
            res = (vals.detach(), mask, sums.detach(), smask, p.grad)
            ev_cmp = torch.cuda.Event()
            ev_cmp.record(s_cmp)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_cmp)
            for t in res:
                t.record_stream(s_out)
            for name, t in zip(("vals", "mask", "sums", "smask", "grad"), res):
                out[name].copy_(t, non_blocking=True)

    def drain():
        torch.cuda.current_stream(dev).wait_stream(s_out)
        torch.cuda.synchronize(dev)

    one()
    drain()
    barrier(world)
    cur = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(cur)
    s_in.wait_stream(cur)
    for _ in range(steps):
        one()
    cur.wait_stream(s_out)
    e1.record(cur)
    torch.cuda.synchronize(dev)
    ms = max_over_ranks(e0.elapsed_time(e1) / steps, world)
    return {"value": cfg.tokens * world / (ms * 1e-3), "unit": "tokens/s", "ms_per_step": ms,
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": steps,
            "path": "pinned host -> ravel_lm_b200.causal_last_k_lookup/causal_sum_lookup (+autograd) -> pinned host",
            "overlap": "copies in and out on their own streams; step i+1 host->device overlaps step i device->host"}


if __name__ == "__main__":
    main()
