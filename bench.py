"""Prefill-attention benchmark (one JSON line on rank 0).

Default workload ("reuse_prefill"): KVBoost's prefix-reuse prefill op --
batch 4, 32 query heads over 8 KV heads (GQA 4), head_dim 128, bf16, a cached
prefix of 7 chunks x 128 = 896 tokens plus a 256-token suffix (kv_len 1152,
bottom-right causal offset 896), all N(0,1) from a seed.  One step = one
launch of the prefill kernel over one such batch.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME]
    python bench.py --impl reference ...   # the CPU restatement on host cores

Timing: K steps are captured in one CUDA graph and replayed between two
events on the launching stream (W warm-up steps replayed first).  The steps
rotate over enough distinct input sets that the inputs touched (>126 MB) do
not fit in L2, so every step reads cold data.  With N > 1 (torchrun) every
rank runs its own batch (weak scaling, no collective on the data path); the
elapsed time is the max over ranks.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

L2_BYTES = 126 * 1024 * 1024

WORKLOADS = {
    # name: (B, Hq, Hkv, Sq, P (cached prefix), D, dtype)
    "reuse_prefill": dict(B=4, Hq=32, Hkv=8, Sq=256, P=896, D=128, dtype="bf16",
                          desc="prefix-reuse prefill op: B4 Hq32/Hkv8 D128 bf16, "
                               "7 cached chunks (896) + 256 new tokens"),
    "causal_op": dict(B=2, Hq=16, Hkv=16, Sq=1024, P=0, D=64, dtype="bf16",
                      desc="single causal op: B2 H16 S1024 D64 bf16"),
}

# dram__bytes_read.sum + dram__bytes_write.sum of one prefill launch from the
# committed ncu capture (profiles/prefill_dense_reuse_b4h32kv8_d128.md).
NCU_TRAFFIC_BYTES = {"reuse_prefill": 27335168}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="kvboost", choices=["kvboost", "reference"])
    ap.add_argument("--workload", default="reuse_prefill", choices=sorted(WORKLOADS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=10)
    return ap.parse_args()


def flops_of(w):
    from oracle.attention import attention_flops
    kv = w["P"] + w["Sq"]
    return attention_flops([w["Sq"]] * w["B"], [kv] * w["B"], w["Hq"], w["D"], causal=True)


def bytes_of(w):
    s = 2
    kv = w["P"] + w["Sq"]
    return w["B"] * (2 * w["Hq"] * w["Sq"] * w["D"] * s + 2 * w["Hkv"] * kv * w["D"] * s)


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["bf16_tflops"]), float(d["hbm_gbs"]), "measured"
    return 1590.0, 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, FileNotFoundError):
            self.proc = None
        time.sleep(0.25)
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in getattr(self, "lines", []):
            parts = [x.strip() for x in l.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def cpu_baseline(w, budget_s=12.0, sample_batches=1):
    """The oracle (numpy float32, all host threads) on `sample_batches` batch elements."""
    import numpy as np
    from oracle.attention import attention, attention_flops
    try:
        from threadpoolctl import threadpool_limits
        limiter = threadpool_limits(limits=os.cpu_count())
    except Exception:  # pragma: no cover
        limiter = None
    g = np.random.default_rng(0)
    b = sample_batches
    kv = w["P"] + w["Sq"]
    q = g.standard_normal((b, w["Hq"], w["Sq"], w["D"]), dtype=np.float32)
    k = g.standard_normal((b, w["Hkv"], kv, w["D"]), dtype=np.float32)
    v = g.standard_normal((b, w["Hkv"], kv, w["D"]), dtype=np.float32)
    scale = 1.0 / math.sqrt(w["D"])
    fl = attention_flops([w["Sq"]] * b, [kv] * b, w["Hq"], w["D"], True)
    n, t0 = 0, time.perf_counter()
    while True:
        attention(q, k, v, scale, True, compute_dtype=np.float32)
        n += 1
        el = time.perf_counter() - t0
        if el > budget_s or n >= 50:
            break
    if limiter is not None:
        limiter.unregister() if hasattr(limiter, "unregister") else None
    return {"value": fl * n / el / 1e12, "unit": "TFLOP/s", "cores": os.cpu_count(),
            "kind": "port",
            "sample": f"{n} x {b} of {w['B']} batch elements of the workload, numpy float32 "
                      f"oracle (oracle/attention.py), {el:.1f} s"}


def run_reference(args, w):
    """--impl reference: the CPU restatement timed on the host (rank 0 only)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import numpy as np
    from oracle.attention import attention, attention_flops
    kv = w["P"] + w["Sq"]
    g = np.random.default_rng(0)
    q = g.standard_normal((1, w["Hq"], w["Sq"], w["D"]), dtype=np.float32)
    k = g.standard_normal((1, w["Hkv"], kv, w["D"]), dtype=np.float32)
    v = g.standard_normal((1, w["Hkv"], kv, w["D"]), dtype=np.float32)
    scale = 1.0 / math.sqrt(w["D"])
    fl = attention_flops([w["Sq"]], [kv], w["Hq"], w["D"], True)
    for _ in range(max(0, args.warmup)):
        attention(q, k, v, scale, True, compute_dtype=np.float32)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        attention(q, k, v, scale, True, compute_dtype=np.float32)
    el = time.perf_counter() - t0
    val = fl * args.steps / el / 1e12
    line = {
        "impl": "reference", "metric": "prefill attention TFLOP/s", "value": val,
        "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": el / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": args.workload, "desc": w["desc"], "sample": "1 batch element per step"},
        "cpu_baseline": {"value": val, "unit": "TFLOP/s", "cores": os.cpu_count(), "kind": "port",
                         "sample": "1 of %d batch elements per step, numpy float32 oracle "
                                   "(no runnable reference CUDA path exists)" % w["B"]},
        "e2e": {"value": val, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    w = WORKLOADS[args.workload]
    if args.impl == "reference":
        run_reference(args, w)
        return

    import torch
    import torch.distributed as dist
    from kvboost_b200 import ops

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))

    dtype = torch.bfloat16 if w["dtype"] == "bf16" else torch.float16
    B, Hq, Hkv, Sq, P, D = w["B"], w["Hq"], w["Hkv"], w["Sq"], w["P"], w["D"]
    kv = P + Sq
    scale = 1.0 / math.sqrt(D)
    per_set = bytes_of(w)
    R = max(2, math.ceil(2 * L2_BYTES / per_set))
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    sets = []
    for _ in range(R):
        q = torch.randn(B, Hq, Sq, D, generator=g, device=dev, dtype=torch.float32).to(dtype)
        k = torch.randn(B, Hkv, kv, D, generator=g, device=dev, dtype=torch.float32).to(dtype)
        v = torch.randn(B, Hkv, kv, D, generator=g, device=dev, dtype=torch.float32).to(dtype)
        o = torch.empty(B, Hq, Sq, D, device=dev, dtype=dtype)
        sets.append((q, k, v, o))

    def step(i):
        q, k, v, o = sets[i % R]
        ops.prefill_attention(q, k, v, scale, True, out=o, return_lse=False)

    # one eager call (allocates the status word), then capture
    step(0)
    torch.cuda.synchronize()
    stream = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(stream):
        gw, gt = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
        with torch.cuda.graph(gw, stream=stream):
            for i in range(args.warmup):
                step(i)
        with torch.cuda.graph(gt, stream=stream):
            for i in range(args.steps):
                step(i)
    torch.cuda.synchronize()

    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        with torch.cuda.stream(stream):
            gw.replay()
            if world > 1:
                dist.barrier()
            torch.cuda.synchronize()
            ev0.record(stream)
            gt.replay()
            ev1.record(stream)
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
    ms = ev0.elapsed_time(ev1)
    if world > 1:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    status = ops.read_status(dev)
    fl = flops_of(w)
    per_launch_s = ms / 1e3 / args.steps
    value = world * fl * args.steps / (ms / 1e3) / 1e12
    tok_s = world * B * Sq * args.steps / (ms / 1e3)

    # ---- e2e: public API with pinned host buffers, copies inside the timed region
    hq = torch.randn(B, Hq, Sq, D, dtype=torch.float32).to(dtype).pin_memory()
    hk = torch.randn(B, Hkv, kv, D, dtype=torch.float32).to(dtype).pin_memory()
    hv = torch.randn(B, Hkv, kv, D, dtype=torch.float32).to(dtype).pin_memory()
    ho = torch.empty(B, Hq, Sq, D, dtype=dtype).pin_memory()
    h2d = sum(t.numel() * t.element_size() for t in (hq, hk, hv))
    d2h = ho.numel() * ho.element_size()

    def e2e_step():
        dq, dk, dv = (t.to(dev, non_blocking=True) for t in (hq, hk, hv))
        o, _ = ops.prefill_attention(dq, dk, dv, scale, True, return_lse=False)
        ho.copy_(o, non_blocking=True)

    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.e2e_steps):
        e2e_step()
    e1.record()
    torch.cuda.synchronize()
    ems = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ems], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ems = float(t.item())
    e2e_value = world * fl * args.e2e_steps / (ems / 1e3) / 1e12

    peak_tf, peak_bw, peak_src = measured_peaks()
    achieved = fl / per_launch_s / 1e12
    traffic = NCU_TRAFFIC_BYTES.get(args.workload)
    line = {
        "metric": "prefill attention TFLOP/s", "value": value, "unit": "TFLOP/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": w["dtype"], "data": "synthetic",
        "config": {"workload": args.workload, "desc": w["desc"], "batch": B, "q_heads": Hq,
                   "kv_heads": Hkv, "q_len": Sq, "kv_len": kv, "head_dim": D,
                   "parallelism": f"independent batches x{world}" if world > 1 else "single",
                   "l2": f"inputs rotate over {R} sets ({R * per_set / 2**20:.0f} MiB > L2)",
                   "timing": "CUDA graph of K launches between events"},
        "tokens_per_s": tok_s,
        "e2e": {"value": e2e_value, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": ems / args.e2e_steps},
        "gpu_launches": args.steps,
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak_tf,
                     "unit": "TFLOP/s", "frac": achieved / peak_tf, "traffic": traffic,
                     "peak_source": f"{peak_src} bf16 (burst)",
                     "algorithmic_bytes": bytes_of(w)},
        "clocks": clk.summary(),
        "device_status": status,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(w)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        del gw, gt
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
