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
(``e2e``) and its copy-only floor, the reference's CPU code timed on the host
(``cpu_baseline``, rank 0 at N=1), decode microseconds per step for
configuration 4, the configuration-5 model step, strong scaling under
torchrun, and the SM clocks sampled during the timed region.

``--impl reference`` times the reference's own CPU implementation: its
``ravel_lm.ravel_memory`` functions on CPU tensors with every host core
(torch threads), from the installed copy under baseline/_ref, on a bounded
sample of the same workload; the C restatement in oracle/ (OpenMP) is timed
beside it as ``cpu_port``, and replaces it when the install does not import.
Under torchrun only rank 0 works.
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
    ap.add_argument("--config", type=int, default=3, choices=[1, 2, 3, 5])
    ap.add_argument("--e2e-steps", type=int, default=8)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-decode", action="store_true")
    ap.add_argument("--no-general", action="store_true",
                    help="skip the extra timing of the general path (reads drawn apart from the writes)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-model", action="store_true",
                    help="skip the whole-model training step of configuration 5 (needs baseline/_ref)")
    ap.add_argument("--no-strong", action="store_true",
                    help="under torchrun: skip the strong-scaling run of the fixed configuration-3 problem")
    ap.add_argument("--no-reference-gpu", action="store_true",
                    help="skip timing the reference's own functions on CUDA tensors (needs baseline/_ref)")
    ap.add_argument("--cpu-streams", type=int, default=8, help="streams in the CPU baseline sample")
    ap.add_argument("--batch", type=int, default=None, help="override B per GPU (small profiling cases)")
    ap.add_argument("--ops", choices=["all", "lk", "ss"], default="all",
                    help="ops in a step (profiling a single op; the benchmark runs all)")
    ap.add_argument("--only", choices=["fused_read", "decode", "config1", "config5_op", "general", "model"], default=None,
                    help="run one side measurement alone and print its JSON (profiling)")
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
    gv = x["g_vals"][:, :, :C].contiguous() if "g_vals" in x else None
    gs = x["g_sums"][:, :, :C].contiguous() if "g_sums" in x else None
    code = {torch.bfloat16: "bf16", torch.float16: "f16"}.get(p.dtype)
    pbits = p.view(torch.int16).numpy().view(np.uint16) if code else p.numpy()
    return dict(w=w, r=r, p=p, pbits=pbits, code=code, gv=gv, gs=gs, streams=C, T=cfg.T,
                tokens_equiv=cfg.T * C / cfg.C)


def cpu_step(oracle, s, cfg):
    """LK fwd + SS fwd + LK bwd + SS bwd of the CPU port on the sample (LK fwd only for forward-only configs)."""
    vals, mask, src, tape = oracle.latestk_fwd(s["w"], s["pbits"], s["r"], address_space=cfg.A, k=cfg.k,
                                               dtype=s["code"])
    if not cfg.backward:
        return vals.sum()
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
    what = (f"latest-k k={cfg.k} + segmented-sum fwd+bwd" if cfg.backward else f"latest-k k={cfg.k} fwd")
    return {"value": s["tokens_equiv"] / dt, "unit": "tokens/s", "cores": oracle.num_threads(), "kind": "port",
            "sample": f"{s['streams']} of {cfg.C} streams of one batch row (T={cfg.T}): {what}, "
                      f"= {s['tokens_equiv']:.0f} token-equivalents; {steps} timed steps, {warmup} warm-up",
            "sec_per_step": dt}


def import_reference():
    """The installed reference (baseline/_ref, a pip --target install of ravel-lm), or None."""
    ref = ROOT / "baseline" / "_ref"
    if not (ref / "ravel_lm" / "ravel_memory.py").exists():
        return None
    if str(ref) not in sys.path:
        sys.path.insert(0, str(ref))
    import ravel_lm.ravel_memory as mem
    return mem


def run_reference_torch_cpu(cfg, steps: int, warmup: int, n_streams: int) -> dict:
    """The reference's own torch code (ravel_memory.py:52-241) on the host cores, on the same
    bounded sample as the CPU port: latest-k + sum forward and backward through autograd."""
    import torch
    try:
        mem = import_reference()
    except Exception as exc:  # an install that does not import is reported, not fatal
        return {"unavailable": f"import of the installed reference failed: {exc}"[:200]}
    if mem is None:
        return {"unavailable": "baseline/_ref holds no installed reference"}
    cores = os.cpu_count() or 1
    old_threads = torch.get_num_threads()
    torch.set_num_threads(cores)
    s = cpu_sample(cfg, n_streams)
    w = torch.from_numpy(s["w"])
    r = None if s["r"] is None else torch.from_numpy(s["r"])
    p = s["p"].clone().requires_grad_(cfg.backward)

    def step():
        p.grad = None
        vals, _ = mem.causal_last_k_lookup(w, p, r, address_space=cfg.A, k=cfg.k)
        if not cfg.backward:
            return
        sums, _ = mem.causal_sum_lookup(w, p, r, address_space=cfg.A)
        torch.autograd.backward([vals, sums], [s["gv"], s["gs"]])

    for _ in range(warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    dt = (time.perf_counter() - t0) / max(steps, 1)
    torch.set_num_threads(old_threads)
    return {"value": s["tokens_equiv"] / dt, "unit": "tokens/s", "cores": cores, "kind": "reference",
            "sample": f"{s['streams']} of {cfg.C} streams of one batch row (T={cfg.T}), "
                      f"= {s['tokens_equiv']:.0f} token-equivalents: the reference's causal_last_k_lookup"
                      f"{' + causal_sum_lookup forward + backward (autograd)' if cfg.backward else ' forward'} "
                      f"on CPU tensors, torch {torch.__version__} with {cores} threads; "
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
        # the latest-k gradient added to the sum's: reads that gradient too
        "ravel_latestk_bwd_accumulate": N * (k * D * e + 2 * D * e),
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
    wa = torch.randint(0, A, (steps, S, H), generator=g, device=dev)  # independent write addresses
    pay = torch.randn(steps, S, H, D, generator=g, device=dev).to(dt)
    torch.cuda.synchronize(dev)

    def timed(fn, n):
        for i in range(16):
            fn(i)
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(n):
            fn(i)
        e1.record()
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) * 1000.0 / n

    def graphed(rd, wr):
        """The 1024 fused read+write steps captured once and replayed: µs per step."""
        stream = torch.cuda.Stream(dev)
        stream.wait_stream(torch.cuda.current_stream(dev))
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            cache.step(rd[0], wr[0], pay[0])
            with torch.cuda.graph(graph, stream=stream):
                for i in range(steps):
                    cache.step(rd[i], wr[i], pay[i])
        torch.cuda.current_stream(dev).wait_stream(stream)
        graph.replay()
        torch.cuda.synchronize(dev)
        reps = 3
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record()
        for _ in range(reps):
            graph.replay()
        g1.record()
        torch.cuda.synchronize(dev)
        del graph
        return g0.elapsed_time(g1) * 1000.0 / (steps * reps)

    # eager: one read + one write launch per step through the API (what model.py:421,424 calls)
    eager_us = timed(lambda i: (cache.read(ra[i]), cache.write(ra[i], pay[i])), steps)
    # eager: the one-launch step, with new output tensors and into reused ones
    step_us = timed(lambda i: cache.step(ra[i], ra[i], pay[i]), steps)
    obuf = (torch.empty(S, H, D, dtype=dt, device=dev), torch.empty(S, H, dtype=torch.bool, device=dev))
    step_out_us = timed(lambda i: cache.step(ra[i], ra[i], pay[i], out=obuf), steps)
    graph_us = graphed(ra, ra)
    graph_ind_us = graphed(ra, wa)
    step_bytes = S * H * (2 * 8 + 4 * D * 2 + 3)
    out = {"config": "cfg4: 256 streams x 16 heads, A=4096 uniform, D=64 bf16, cache prefilled by 4096 writes",
           "us_per_step_graph": graph_us, "us_per_step_graph_independent_rw": graph_ind_us,
           "us_per_step_eager": eager_us, "us_per_step_eager_one_launch": step_us,
           "us_per_step_eager_one_launch_reused_out": step_out_us,
           "prefill_us_token_by_token": prefill_tok_us, "prefill_us_bulk": prefill_bulk_us,
           "bytes_per_step": step_bytes, "gbs_graph": step_bytes / (graph_us * 1e-6) / 1e9,
           "target_us": 10.0}
    # the reference's own cache (gather / scatter_, ravel_memory.py:271-292) on the same GPU
    try:
        mem = import_reference()
    except Exception as exc:
        mem, out["reference"] = None, f"unavailable: {exc}"[:200]
    if mem is not None:
        rc = mem.RavelLayerCache(values=cache.values.clone(), filled=cache.filled.clone())
        out["us_per_step_reference_eager"] = timed(lambda i: (rc.read(ra[i]), rc.write(ra[i], pay[i])), steps)
        stream = torch.cuda.Stream(dev)
        stream.wait_stream(torch.cuda.current_stream(dev))
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            rc.read(ra[0])
            rc.write(ra[0], pay[0])
            with torch.cuda.graph(graph, stream=stream):
                for i in range(steps):
                    rc.read(ra[i])
                    rc.write(ra[i], pay[i])
        torch.cuda.current_stream(dev).wait_stream(stream)
        out["us_per_step_reference_graph"] = timed(lambda i: graph.replay(), 3) / steps
        del graph, rc
    return out


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
        # the reference's own torch code on the host cores when its install imports, else the C port
        cb = run_reference_torch_cpu(cfg, args.steps, args.warmup, args.cpu_streams)
        port = run_cpu_baseline(cfg, 3, 1, args.cpu_streams)
        if "unavailable" in cb:
            cb, port = port, {"unavailable": cb["unavailable"]}
        line = {"metric": METRIC, "value": cb["value"], "unit": "tokens/s", "impl": "reference",
                "cpu_port": {k: port[k] for k in ("value", "unit", "cores", "kind", "sample", "unavailable")
                             if k in port},
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
    if args.only is not None:
        dev = torch.device("cuda", local)
        fn = {"fused_read": run_fused_read, "decode": run_decode, "config1": run_cfg1, "config5_op": run_cfg5_op,
              "general": lambda d: run_general(cfg, make_inputs(cfg, seed=1000 + cfg.cfg, device=d), d, world,
                                               steps=args.steps),
              "model": lambda d: run_model(d, rank, world)}[args.only]
        res = fn(dev)
        if rank == 0:
            print(json.dumps({"only": args.only, "result": res}), flush=True)
        if world > 1:
            import torch.distributed as dist
            barrier(world)
            dist.destroy_process_group()
        return
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    seed = 1000 + cfg.cfg + 7919 * rank
    x = make_inputs(cfg, seed=seed, device=dev)
    if args.ops == "ss":  # the latest-k gradient is not needed
        x["g_vals"] = None
        torch.cuda.empty_cache()
    w, r = x["write"], x["read"]
    p = x["payload"].requires_grad_(cfg.backward)
    gv, gs = x.get("g_vals"), x.get("g_sums")
    A, k = cfg.A, cfg.k

    def step():
        # Each step stands for a new batch: forget the tape of the previous step
        # (only the latest-k -> sum reuse inside one step is legitimate).
        clear_tape_cache()
        if not cfg.backward:  # configuration 1: the latest-1 forward alone
            return causal_last_k_lookup(w, p, r, address_space=A, k=k)
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

    barrier(world)
    torch.cuda.synchronize(dev)
    launches0 = L.kernel_launches()
    # every entry point's own GPU time, recorded by the library around its work
    # (two cudaEventRecord calls per call; nothing on the Python side)
    L.timing_start(16 * args.steps)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(args.steps):
        step()
    t1.record()
    torch.cuda.synchronize(dev)
    records = defaultdict(list)
    for name, t in L.timing_stop():
        records[name].append(t)
    launches = L.kernel_launches() - launches0
    barrier(world)
    clk = clocks.stop()
    ms_local = t0.elapsed_time(t1) / args.steps
    ms = max_over_ranks(ms_local, world)
    assert L.device_error(stream) == 0, "device error word set"

    peaks = measured_peaks()
    kb = kernel_bytes(cfg)
    kernels = {}
    for name, times in records.items():
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
    step_bytes = sum(kb[n] for n in kb if n in kernels)  # one tape per step: the sum reuses the latest-k tape
    tokens = cfg.tokens * world
    value = tokens / (ms * 1e-3)

    step_graph = run_graph_step(step, dev, world)
    e2e = copy_bound = e2e_train = None
    if not args.no_e2e and cfg.backward:
        e2e = run_e2e(cfg, x, dev, args.e2e_steps, world)
        copy_bound = run_copy_bound(e2e, dev, args.e2e_steps, world)
        e2e_train = run_e2e_training(cfg, x, dev, args.e2e_steps, world)
    general = None
    if not args.no_general and cfg.addressing == "zipf" and cfg.backward:
        general = run_general(cfg, x, dev, world)
    strong = None
    if world > 1 and not args.no_strong and cfg.cfg == 3:
        strong = run_strong(cfg, dev, rank, world)
    ref_gpu = cfg1 = fused_read = None
    if world == 1 and not args.no_reference_gpu:
        if cfg.backward:
            ref_gpu = run_reference_gpu(cfg, x, dev, steps=5, warmup=args.warmup)
        cfg1 = run_cfg1(dev)
        fused_read = run_fused_read(dev)
    cfg5_op = run_cfg5_op(dev) if world == 1 and args.config != 5 else None
    del x, p, gv, gs
    torch.cuda.empty_cache()
    model = None
    if not args.no_model:
        model = run_model(dev, rank, world)
    decode = None
    if not args.no_decode:
        decode = run_decode(dev)
    cpu = port = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cb = run_reference_torch_cpu(cfg, 3, 1, args.cpu_streams)
        pb = run_cpu_baseline(cfg, 3, 1, args.cpu_streams)
        if "unavailable" in cb:
            cb, pb = pb, {"unavailable": cb["unavailable"]}
        cpu = {k2: cb[k2] for k2 in ("value", "unit", "cores", "kind", "sample")}
        port = {k2: pb[k2] for k2 in ("value", "unit", "cores", "kind", "sample", "unavailable") if k2 in pb}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": DTYPE_NAMES[str(cfg.dtype)],
            "data": "synthetic", "config": workload_config(cfg, world),
            "tokens_per_sec_per_gpu": value / world,
            "step_graph": step_graph,
            "step_roofline": {"algorithmic_bytes": step_bytes, "achieved_gbs": step_bytes / (ms * 1e-3) / 1e9,
                              "frac": step_bytes / (ms * 1e-3) / 1e9 / peaks["hbm_gbs"], "peak": peaks["hbm_gbs"]},
            "roofline": roofline, "kernels": kernels, "e2e": e2e, "e2e_copy_bound": copy_bound,
            "e2e_training": e2e_train,
            "cpu_baseline": cpu, "cpu_port": port, "decode": decode,
            "general_path": general, "reference_gpu": ref_gpu, "config1": cfg1, "strong_scaling": strong,
            "config5_op": cfg5_op, "config5_model": model, "fused_read_linear": fused_read, "clocks": clk,
            "gpu_launches": launches,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        barrier(world)
        dist.destroy_process_group()


def workload_config(cfg, world) -> dict:
    what = "latest-k (k={}) + causal segmented-sum, forward + backward" if cfg.backward else "latest-k (k={}), forward"
    return {"workload": f"cfg{cfg.cfg}: " + what.format(cfg.k),
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
    def step():
        clear_tape_cache()
        p.grad = None
        vals, _m = causal_last_k_lookup(w, p, r, address_space=cfg.A, k=cfg.k)
        sums, _s = causal_sum_lookup(w, p, r, address_space=cfg.A)
        torch.autograd.backward([vals, sums], [gv, gs])

    for _ in range(2):
        step()
    torch.cuda.synchronize(dev)
    L.timing_start(16 * steps)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(steps):
        step()
    t1.record()
    torch.cuda.synchronize(dev)
    records = defaultdict(list)
    for name, t in L.timing_stop():
        records[name].append(t)
    ms = max_over_ranks(t0.elapsed_time(t1) / steps, world)
    per = {n: sum(v) / len(v) * 1000.0 for n, v in records.items()}
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


def run_graph_step(step, dev, world, reps: int = 10) -> dict:
    """The same step captured once in a CUDA graph and replayed (no host launch work): the
    kernel-bound step time, which host-bound small configurations hide in eager mode."""
    import torch
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(side):
        step()
        with torch.cuda.graph(graph, stream=side):
            step()
    torch.cuda.current_stream(dev).wait_stream(side)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize(dev)
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize(dev)
    ms = max_over_ranks(e0.elapsed_time(e1) / reps, world)
    del graph
    return {"ms_per_step": ms, "replays": reps}


def run_e2e_training(cfg, x, dev, steps, world):
    """A training step of the operator end to end: each step's batch (write addresses and payload)
    crosses from pinned host memory, the forward outputs are consumed on the device by a fixed
    probe loss L = <values, G1> + <sums, G2> (G1, G2 device-resident like a next layer's weights;
    its gradients are exactly G1 and G2, the upstream gradients of the device-timed step), and the
    loss and the payload gradient -- the step's results for its caller -- cross back."""
    import torch
    from ravel_lm_b200 import causal_last_k_lookup, causal_sum_lookup
    from ravel_lm_b200.ravel_memory import clear_tape_cache

    class ProbeLoss(torch.autograd.Function):
        @staticmethod
        def forward(ctx, t, g):
            ctx.save_for_backward(g)
            return torch.dot(t.reshape(-1), g.reshape(-1)).float()  # one pass in the payload dtype

        @staticmethod
        def backward(ctx, go):
            (g,) = ctx.saved_tensors
            return g * go.to(g.dtype), None

    G1, G2 = x["g_vals"], x["g_sums"]
    host = {"write": x["write"].to("cpu").pin_memory(), "payload": x["payload"].detach().to("cpu").pin_memory()}
    if x["read"] is not None:
        host["read"] = x["read"].to("cpu").pin_memory()
    out_loss = torch.empty(1, dtype=torch.float32).pin_memory()
    out_grad = torch.empty(tuple(x["payload"].shape), dtype=cfg.dtype).pin_memory()
    h2d = sum(t.numel() * t.element_size() for t in host.values())
    d2h = out_loss.numel() * 4 + out_grad.numel() * out_grad.element_size()
    s_in, s_cmp, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev), torch.cuda.Stream(dev)

    def one():
        with torch.cuda.stream(s_in):
            w = host["write"].to(dev, non_blocking=True)
            r = host["read"].to(dev, non_blocking=True) if "read" in host else None
            p = host["payload"].to(dev, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(s_in)
        with torch.cuda.stream(s_cmp):
            s_cmp.wait_event(ev)
            for t in (w, r, p):
                if t is not None:
                    t.record_stream(s_cmp)
            clear_tape_cache()
            p.requires_grad_(True)
            vals, _ = causal_last_k_lookup(w, p, r, address_space=cfg.A, k=cfg.k)
            sums, _ = causal_sum_lookup(w, p, r, address_space=cfg.A)
            loss = ProbeLoss.apply(vals, G1) + ProbeLoss.apply(sums, G2)
            loss.backward()
            res = (loss.detach().reshape(1), p.grad)
            ev2 = torch.cuda.Event()
            ev2.record(s_cmp)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev2)
            for t in res:
                t.record_stream(s_out)
            out_loss.copy_(res[0], non_blocking=True)
            out_grad.copy_(res[1], non_blocking=True)

    one()
    torch.cuda.current_stream(dev).wait_stream(s_out)
    torch.cuda.synchronize(dev)
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
            "path": "pinned host batch (addresses, payload) -> causal_last_k_lookup/causal_sum_lookup -> probe "
                    "loss <values, G1> + <sums, G2> on the device -> backward -> pinned host loss + payload gradient",
            "overlap": "copies in and out on their own streams; step i+1 host->device overlaps step i device->host"}


def run_copy_bound(e2e: dict, dev, steps: int, world: int) -> dict:
    """The end-to-end number's floor: the same bytes per step copied host->device and
    device->host (pinned, on two streams, as the end-to-end pipeline runs them) with no compute."""
    import torch
    hin = torch.empty(e2e["h2d_bytes_per_step"], dtype=torch.uint8).pin_memory()
    hout = torch.empty(e2e["d2h_bytes_per_step"], dtype=torch.uint8).pin_memory()
    din = torch.empty_like(hin, device=dev)
    dout = torch.empty_like(hout, device=dev)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

    def one():
        with torch.cuda.stream(s_in):
            din.copy_(hin, non_blocking=True)
        with torch.cuda.stream(s_out):
            hout.copy_(dout, non_blocking=True)

    one()
    torch.cuda.synchronize(dev)
    barrier(world)
    cur = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(cur)
    s_in.wait_stream(cur)
    s_out.wait_stream(cur)
    for _ in range(steps):
        one()
    cur.wait_stream(s_in)
    cur.wait_stream(s_out)
    e1.record(cur)
    torch.cuda.synchronize(dev)
    ms = max_over_ranks(e0.elapsed_time(e1) / steps, world)
    del din, dout
    torch.cuda.empty_cache()
    return {"ms_per_step": ms, "tokens_per_s": e2e["value"] * e2e["ms_per_step"] / ms,
            "h2d_gbs": e2e["h2d_bytes_per_step"] / (ms * 1e-3) / 1e9,
            "d2h_gbs": e2e["d2h_bytes_per_step"] / (ms * 1e-3) / 1e9,
            "e2e_frac_of_bound": ms / e2e["ms_per_step"],
            "what": "pinned host<->device copies of the end-to-end step's bytes, both directions at once, no compute"}


def run_strong(cfg, dev, rank: int, world: int, steps: int = 10, warmup: int = 3) -> dict:
    """Strong scaling: the fixed single-GPU problem (global batch cfg.B) split over the ranks
    with sharding.sharded_lookup (batch rows, or heads when B < world), each rank holding only
    its own slice.  Also times replicated outputs (one NCCL all-gather per output)."""
    import torch
    from ravel_lm_b200.ravel_memory import clear_tape_cache
    from ravel_lm_b200.sharding import gather_outputs, shard_streams, sharded_lookup
    from ravel_lm_b200.workloads import make_inputs
    sh = shard_streams(cfg.B, cfg.C, world, rank)
    x = make_inputs(cfg, seed=1000 + cfg.cfg, device=dev)  # identical global problem on every rank
    w, p0 = sh.take(x["write"]), sh.take(x["payload"])
    r = sh.take(x["read"])
    gv, gs = sh.take(x["g_vals"]), sh.take(x["g_sums"])
    del x
    torch.cuda.empty_cache()
    p = p0.requires_grad_(True)
    kw = dict(address_space=cfg.A, world=world, rank=rank, full_shape=(cfg.B, cfg.C))

    def step():
        clear_tape_cache()
        p.grad = None
        vals, _ = sharded_lookup(w, p, r, k=cfg.k, **kw)
        sums, _ = sharded_lookup(w, p, r, use_sum=True, **kw)
        torch.autograd.backward([vals, sums], [gv, gs])

    for _ in range(warmup):
        step()
    torch.cuda.synchronize(dev)
    barrier(world)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(steps):
        step()
    t1.record()
    torch.cuda.synchronize(dev)
    ms = max_over_ranks(t0.elapsed_time(t1) / steps, world)
    # replicated outputs: every rank receives the full [B, T, C, ...] results
    with torch.no_grad():
        vals, vmask = sharded_lookup(w, p, r, k=cfg.k, **kw)
        sums, smask = sharded_lookup(w, p, r, use_sum=True, **kw)
    outs = (vals, vmask, sums, smask)
    for o in outs:
        gather_outputs(o, sh)
    torch.cuda.synchronize(dev)
    barrier(world)
    g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    g0.record()
    for o in outs:
        gather_outputs(o, sh)
    g1.record()
    torch.cuda.synchronize(dev)
    gms = max_over_ranks(g0.elapsed_time(g1), world)
    full_bytes = sum(o.numel() * o.element_size() for o in outs) * world
    recv = full_bytes * (world - 1) / world
    return {"global_batch": cfg.B, "streams_per_rank": sh.streams, "split": "heads" if sh.splits_heads else "batch",
            "ms_per_step": ms, "value": cfg.tokens / (ms * 1e-3), "unit": "tokens/s",
            "replicate_ms": gms, "replicate_bytes": full_bytes,
            "replicate_recv_gbs_per_rank": recv / (gms * 1e-3) / 1e9,
            "what": "fixed cfg3 problem split over the ranks; latest-k + sum fwd+bwd per rank; replicate = "
                    "all_gather_into_tensor of values, masks, sums, sum masks + local reorder"}


def run_cfg1(dev, reps: int = 200) -> dict:
    """Configuration 1 (latest-1 forward, fp32, B8 T256 H4 D16): ours against the kernel the
    reference dispatches to on CUDA for it (Triton v2, triton_latest1.py:86-154), µs per call."""
    import torch
    from ravel_lm_b200 import causal_last_k_lookup
    from ravel_lm_b200.ravel_memory import clear_tape_cache
    from ravel_lm_b200.workloads import CONFIGS, make_inputs
    cfg = CONFIGS[1]
    x = make_inputs(cfg, seed=1001, device=dev)
    w, p = x["write"], x["payload"]

    def timed(fn):
        for _ in range(10):
            fn()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) * 1000.0 / reps

    def ours():
        clear_tape_cache()
        return causal_last_k_lookup(w, p, address_space=cfg.A, k=1)

    out = {"config": "cfg1: B8 T256 H4 D16 fp32, k=1, Zipf(1.1) over 256, forward", "us_ours_eager": timed(ours)}
    # one CUDA graph per call (what a captured model step pays)
    stream = torch.cuda.Stream(dev)
    stream.wait_stream(torch.cuda.current_stream(dev))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        ours()
        with torch.cuda.graph(graph, stream=stream):
            ours()
    torch.cuda.current_stream(dev).wait_stream(stream)
    out["us_ours_graph"] = timed(graph.replay)
    del graph
    try:
        mem = import_reference()
    except Exception as exc:
        mem, out["reference"] = None, f"unavailable: {exc}"[:200]
    if mem is not None:
        import ravel_lm.triton_latest1 as tl1
        if tl1.can_use_triton_latest1_v2(w, p, None, address_space=cfg.A, k=1, write_mask=None):
            try:
                out["us_reference_triton_v2"] = timed(
                    lambda: mem.causal_last_k_lookup(w, p, address_space=cfg.A, k=1))
                vr, mr = mem.causal_last_k_lookup(w, p, address_space=cfg.A, k=1)
                vo, mo = ours()
                out["values_equal_to_reference"] = bool(torch.equal(vr, vo) and torch.equal(mr, mo))
            except Exception as exc:  # a Triton build failure on this stack is reported, not fatal
                out["reference"] = f"Triton v2 failed: {exc}"[:200]
        else:
            out["reference"] = "Triton v2 not eligible here (no triton)"
        old = tl1._HAS_TRITON
        tl1._HAS_TRITON = False
        try:
            out["us_reference_torch"] = timed(lambda: mem.causal_last_k_lookup(w, p, address_space=cfg.A, k=1))
        finally:
            tl1._HAS_TRITON = old
    return out


def run_cfg5_op(dev, steps: int = 50) -> dict:
    """Configuration 5's operator step (latest-k k=2 + sum, forward + backward, learned read heads
    apart from the writes, B8 T1024 H8 D32 fp32) through the public API: eager ms per step with
    nothing else on the host, each entry point's GPU time (recorded by the library), and the same
    step replayed from a CUDA graph.  The small shape that host work, not HBM, decides."""
    import torch
    import ravel_lm_b200._lib as L
    from collections import defaultdict
    from ravel_lm_b200 import causal_last_k_lookup, causal_sum_lookup
    from ravel_lm_b200.ravel_memory import clear_tape_cache
    from ravel_lm_b200.workloads import CONFIGS, make_inputs
    cfg = CONFIGS[5]
    x = make_inputs(cfg, device=dev)
    w, r = x["write"], x["read"]
    p = x["payload"].detach().requires_grad_(True)
    gv, gs = x["g_vals"], x["g_sums"]

    def step():
        clear_tape_cache()
        p.grad = None
        v, _ = causal_last_k_lookup(w, p, r, address_space=cfg.A, k=cfg.k)
        s_, _ = causal_sum_lookup(w, p, r, address_space=cfg.A)
        torch.autograd.backward([v, s_], [gv, gs])

    def timed(n):
        for _ in range(10):
            step()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n):
            step()
        e1.record()
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) / n

    # host-bound: the median of three runs, since other work on the host moves single runs;
    # the objects earlier measurements left behind are collected first
    import gc
    gc.collect()
    runs = sorted(timed(steps) for _ in range(3))
    ms = runs[1]
    L.timing_start(16 * steps)
    ms_timed = timed(steps)
    per = defaultdict(list)
    for name, t in L.timing_stop()[-5 * steps:]:
        per[name].append(t)
    graph = run_graph_step(step, dev, 1, reps=steps)
    return {"config": "cfg5 operator: B8 T1024 H8 D32 fp32, k=2 + sum, learned reads apart from writes, fwd + bwd",
            "ms_per_step_eager": ms, "ms_per_step_eager_runs": runs, "tokens_per_s_eager": cfg.tokens / (ms * 1e-3),
            "ms_per_step_eager_entry_timing": ms_timed,
            "entry_us": {n: sum(v) / len(v) * 1000.0 for n, v in per.items()},
            "ms_per_step_graph": graph["ms_per_step"], "target_ms_eager": 0.2}


def run_fused_read(dev, reps: int = 20) -> dict:
    """The memory layer's read-out at configuration 5's layer shapes (8 x 1024 tokens, 8 heads,
    D 32 fp32, k 2 + sum read, fuse 768 -> 256, gate residual; learned read heads): the unfused
    chain (latest-k forward, sum forward, cat, cuBLAS Linear, gate residual) against
    memory_read_linear (the gather inside a tcgen05 GEMM), forward only, per call; and the
    fused GEMM kernel's own time with its algorithmic FLOPs and bytes."""
    import torch
    import ravel_lm_b200._lib as L
    from ravel_lm_b200 import causal_last_k_lookup, causal_sum_lookup
    from ravel_lm_b200.fused import memory_read_linear
    from ravel_lm_b200.ravel_memory import clear_tape_cache
    from ravel_lm_b200.workloads import CONFIGS, make_inputs
    cfg = CONFIGS[5]
    x0 = make_inputs(cfg, seed=1005, device=dev, grads=False)
    w, r, p = x0["write"], x0["read"], x0["payload"]
    B, T, C, D, k = cfg.B, cfg.T, cfg.C, cfg.D, cfg.k
    N, K = 256, C * (k + 1) * D
    g = torch.Generator(device=dev).manual_seed(77)
    W = torch.randn(N, K, generator=g, device=dev) * K ** -0.5
    x = torch.randn(B, T, N, generator=g, device=dev)
    gate = torch.randn(B, T, N, generator=g, device=dev)

    def unfused():
        clear_tape_cache()
        vals, _ = causal_last_k_lookup(w, p, r, address_space=cfg.A, k=k)
        sums, _ = causal_sum_lookup(w, p, r, address_space=cfg.A)
        rows = torch.cat([vals.reshape(B, T, -1), sums.reshape(B, T, -1)], -1)
        return x + torch.sigmoid(gate) * torch.nn.functional.linear(rows, W)

    def fused():
        clear_tape_cache()
        return memory_read_linear(w, p, r, W, address_space=cfg.A, k=k, use_sum_read=True, x=x, gate_lin=gate)

    def timed(fn):
        for _ in range(5):
            fn()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) * 1000.0 / reps

    with torch.no_grad():
        out = {"config": "cfg5 layer: B8 T1024 H8 D32 fp32, k=2 + sum read, fuse 768->256, gate residual",
               "us_unfused": timed(unfused), "us_fused": timed(fused)}
        diff = (fused() - unfused()).abs().max().item()
        L.timing_start(16 * reps)
        for _ in range(reps):
            fused()
        torch.cuda.synchronize(dev)
        recs = [t for name, t in L.timing_stop() if name == "ravel_gather_gemm"]
    us = sum(recs) / len(recs) * 1000.0
    M = B * T
    flops = 2.0 * M * N * K
    # payload rows read once + sums + source table + weight + x, gate, out
    nbytes = (M * C * D * 4) * 2 + M * C * k * 4 + N * K * 4 + 3 * M * N * 4
    out.update({"us_gemm_kernel": us, "gemm_tflops": flops / (us * 1e-6) / 1e12,
                "gemm_gbs": nbytes / (us * 1e-6) / 1e9, "gemm_algorithmic_bytes": nbytes, "gemm_flops": flops,
                "max_abs_diff_vs_unfused": diff,
                "precision": "fused: TF32 tensor-core inputs, fp32 accumulation; unfused: cuBLAS fp32"})
    return out


def model_config(RavelConfig):
    """Configuration 5's model: a random-init 6-layer RavelLM with both lookups in every layer."""
    return RavelConfig(vocab_size=1024, block_size=1024, d_model=256, n_layers=6, address_space=1024,
                       n_literal_heads=4, n_learned_heads=4, n_codebooks=2, codebook_size=32, payload_dim=32,
                       last_k=2, use_sum_read=True, memory_every=1, dropout=0.0)


def run_model(dev, rank: int, world: int, steps: int = 8, warmup: int = 3) -> dict:
    """Configuration 5: the reference's own RavelLM (from baseline/_ref, unchanged) trained on
    8 sequences of 1024 tokens per GPU, with this operator dropped in for ravel_lm.ravel_memory
    (the import of model.py:11) and, for comparison, with the stock operator.  One step =
    forward, backward, the deferred weight gradients (deferred.flush_deferred), a gradient
    all-reduce over NCCL when world > 1 (data parallel), and an AdamW step.  ``ours_fused``
    also replaces every memory layer's forward by ravel_lm_b200.layer.memory_layer_forward
    (token-hashed tape, read-out GEMM and gate residual on the tensor cores)."""
    import torch
    import ravel_lm_b200._lib as L
    import ravel_lm_b200.ravel_memory as mine
    from ravel_lm_b200.workloads import zipf_ranks
    try:
        mem = import_reference()
        if mem is None:
            return {"unavailable": "baseline/_ref holds no installed reference"}
        import ravel_lm.deferred as deferred
        import ravel_lm.model as model_mod
        from ravel_lm.config import RavelConfig
    except Exception as exc:
        return {"unavailable": f"import of the installed reference failed: {exc}"[:200]}
    cfg = model_config(RavelConfig)
    B, T = 8, 1024
    torch.manual_seed(0)  # same initial weights on every rank
    model = model_mod.RavelLM(cfg).to(dev)
    params = [q for q in model.parameters() if q.requires_grad]
    opt = torch.optim.AdamW(params, lr=1e-4, fused=True)
    g = torch.Generator(device=dev).manual_seed(5000 + rank)
    toks = zipf_ranks(cfg.vocab_size, 1.1, (B, T + 1), g)
    x, y = toks[:, :-1].contiguous(), toks[:, 1:].contiguous()
    names = ("causal_last_k_lookup", "causal_sum_lookup", "RavelLayerCache")
    stock = {n: getattr(model_mod, n) for n in names}
    import types

    from ravel_lm_b200.layer import memory_layer_forward
    layers = [blk.memory for blk in model.blocks if blk.memory is not None]

    def use(impl):
        for n in names:
            setattr(model_mod, n, stock[n] if impl == "stock" else getattr(mine, n))
        for layer in layers:
            if impl == "ours_fused":
                layer.forward = types.MethodType(memory_layer_forward, layer)
            elif "forward" in layer.__dict__:
                del layer.forward

    def step():
        mine.clear_tape_cache()
        opt.zero_grad(set_to_none=True)
        loss = model(x, y)["loss"]
        loss.backward()
        deferred.flush_deferred()
        if world > 1:
            import torch.distributed as dist
            for q in params:
                if q.grad is None:
                    q.grad = torch.zeros_like(q)
            grads = [q.grad for q in params]
            flat = torch._utils._flatten_dense_tensors(grads)
            dist.all_reduce(flat)
            flat.div_(world)
            for gq, v in zip(grads, torch._utils._unflatten_dense_tensors(flat, grads)):
                gq.copy_(v)
        opt.step()
        return loss

    out = {"config": "cfg5: RavelLM vocab 1024, d_model 256, 6 layers, 4 literal + 4 learned heads (2x32 codes), "
                     "A 1024, payload 32 fp32, last_k 2 + sum read; 8 x 1024 tokens per GPU",
           "parallelism": f"data parallel over {world} GPU(s), NCCL all-reduce of gradients" if world > 1
           else "1 GPU", "global_batch": B * world}
    for impl in ("ours", "ours_fused", "stock"):
        use(impl)
        try:
            for _ in range(warmup):
                step()
            torch.cuda.synchronize(dev)
            barrier(world)
            if impl != "stock":
                L.timing_start(64 * steps)
            t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            t0.record()
            for _ in range(steps):
                loss = step()
            t1.record()
            torch.cuda.synchronize(dev)
            ops = [t for _name, t in L.timing_stop()] if impl != "stock" else []
            ms = max_over_ranks(t0.elapsed_time(t1) / steps, world)
            ent = {"ms_per_step": ms, "value": B * T * world / (ms * 1e-3), "unit": "tokens/s",
                   "loss": float(loss.detach())}
            if ops:
                op_ms = sum(ops) / steps
                ent["operator_ms_per_step"] = op_ms
                ent["operator_share"] = op_ms / (t0.elapsed_time(t1) / steps)
            out[impl] = ent
        finally:
            use("stock")
            L.timing_stop()
    del model, opt
    torch.cuda.empty_cache()
    return out


if __name__ == "__main__":
    main()
