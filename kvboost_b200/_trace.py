"""Phase timelines of the dense prefill kernel, from a traced build (pipeline studies).

    python -m kvboost_b200._trace            # on an sm_100a device, nvcc on PATH

Builds a copy of the library with ``-DKVB_TRACE`` (per-CTA clock64 stamps at each
phase of the first 16 key tiles, softmax sub-phases included, and global-timer stamps at CTA entry, after the
dependent-launch wait and at CTA end), loads it instead of the shipped library,
and prints:

* the steady-state chain of one query slot per key tile (softmax, MMA warp
  reaction, PV and next S) for a long causal prefill and the prefix-reuse prefill;
* per-CTA fixed costs of the prefix-reuse prefill (first S, first tile, last tile,
  epilogue), by the CTAs' key-tile count;
* the launch-level timeline of the last of 20 back-to-back launches in a CUDA
  graph: when its CTAs enter, pass the wait and end, relative to the wait.

The stamps add a few instructions per phase; durations are in SM cycles (clock64)
or microseconds (global timer).  The shipped library is never built with them.
"""

from __future__ import annotations

import ctypes
import math
import os
import sys
import tempfile


def _load_traced():
    from . import _build
    out = os.path.join(tempfile.mkdtemp(prefix="kvb_trace_"), "_kvb_attn_trace.so")
    _build.build_traced(out)
    os.environ["KVB_LIB"] = out
    from . import _lib
    lib = _lib.load()
    lib.kvb_debug_set_trace.argtypes = [ctypes.c_void_p]
    return lib


def _inputs(torch, B, Hq, Hkv, Sq, Skv, D, n=1, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return [(torch.randn(B, Hq, Sq, D, device="cuda", generator=g).bfloat16(),
             torch.randn(B, Hkv, Skv, D, device="cuda", generator=g).bfloat16(),
             torch.randn(B, Hkv, Skv, D, device="cuda", generator=g).bfloat16())
            for _ in range(n)]


def _traced_rows(torch, lib, launch):
    buf = torch.zeros(4096 * 512, dtype=torch.int64, device="cuda")
    lib.kvb_debug_set_trace(buf.data_ptr())
    launch()
    torch.cuda.synchronize()
    lib.kvb_debug_set_trace(None)
    t = buf.view(4096, 512).cpu()
    return t[t[:, 0] != 0]


def steady_chain(torch, lib, shape):
    from . import ops
    q, k, v = _inputs(torch, *shape)[0]
    D = shape[-1]
    for _ in range(3):
        ops.prefill_attention(q, k, v, 1 / math.sqrt(D), True, return_lse=False)
    rows = _traced_rows(torch, lib, lambda: ops.prefill_attention(q, k, v, 1 / math.sqrt(D), True,
                                                                  return_lse=False))
    med = lambda x: round(float(x.double().median()))
    out = {}
    for j in range(2, 12):
        r = rows[(rows[:, 64 + j] > 0) & (rows[:, 80 + j] > 0) & (rows[:, 96 + j] > 0)
                 & (rows[:, 64 + j + 1] > 0)]
        if len(r) == 0:
            continue
        if j == 4:   # every softmax warp of slot 0 stamps its P arrival at tile 4
            last = r[:, 8:16].max(1).values
            out["tile 4 arrivals"] = {
                "first_to_last_warp": med(last - r[:, 8:16].min(1).values),
                "last_warp_to_mma_awake": med(r[:, 112 + j] - last),
                "last_warp_to_pv_issued": med(r[:, 96 + j] - last)}
        if (r[:, 256 + j] > 0).all() and (r[:, 320 + j] > 0).all():
            # softmax sub-phases of row 0 (both column halves), from S visible
            out[f"{j} softmax phases"] = {
                "exp_done_h0": med(r[:, 256 + j] - r[:, 64 + j]),
                "exp_done_h1": med(r[:, 304 + j] - r[:, 64 + j]),
                "pair_decided": med(r[:, 272 + j] - r[:, 64 + j]),
                "p_stored_h0": med(r[:, 288 + j] - r[:, 64 + j]),
                "p_stored_h1": med(r[:, 320 + j] - r[:, 64 + j]),
                "arrived_w0": med(r[:, 80 + j] - r[:, 64 + j])}
        out[j] = {"softmax": med(r[:, 80 + j] - r[:, 64 + j]),
                  "p_to_mma_awake": med(r[:, 112 + j] - r[:, 80 + j]),
                  "p_to_pv_issued": med(r[:, 96 + j] - r[:, 80 + j]),
                  "pv_issued_to_next_s_seen": med(r[:, 64 + j + 1] - r[:, 96 + j]),
                  "period": med(r[:, 64 + j + 1] - r[:, 64 + j])}
    return out


def fixed_costs(torch, lib, shape):
    from . import ops
    q, k, v = _inputs(torch, *shape)[0]
    D = shape[-1]
    for _ in range(3):
        ops.prefill_attention(q, k, v, 1 / math.sqrt(D), True, return_lse=False)

    def five():
        for _ in range(5):
            ops.prefill_attention(q, k, v, 1 / math.sqrt(D), True, return_lse=False)
    rows = _traced_rows(torch, lib, five)
    med = lambda x: round(float(x.double().median()))
    ntile = (rows[:, 64:80] > 0).sum(1)
    out = {}
    for n in sorted(set(ntile.tolist())):
        s = rows[ntile == n]
        out[n] = {"ctas": len(s), "wait_to_first_s": med(s[:, 64] - s[:, 0]),
                  "first_tile": med(s[:, 65] - s[:, 64]) if n > 1 else None,
                  "steady_tile": med((s[:, 64 + n - 1] - s[:, 65]) / max(1, n - 2)) if n > 2
                  else None,
                  "last_s_to_epilogue": med(s[:, 2] - s[:, 64 + n - 1]),
                  "epilogue_to_end": med(s[:, 3] - s[:, 2]), "total": med(s[:, 3] - s[:, 0])}
    return out


def launch_timeline(torch, lib, shape, launches=20):
    from . import ops
    D = shape[-1]
    sets = _inputs(torch, *shape, n=8)
    outs = [torch.empty_like(s[0]) for s in sets]
    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        ops.prefill_attention(*sets[0], 1 / math.sqrt(D), True, out=outs[0], return_lse=False)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(st):
        with torch.cuda.graph(graph, stream=st):
            for i in range(launches):
                ops.prefill_attention(*sets[i % 8], 1 / math.sqrt(D), True, out=outs[i % 8],
                                      return_lse=False)
    with torch.cuda.stream(st):
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        graph.replay()
        e1.record(st)
    torch.cuda.synchronize()
    per_launch_us = e0.elapsed_time(e1) / launches * 1000
    def replay():
        with torch.cuda.stream(st):
            graph.replay()
    rows = _traced_rows(torch, lib, replay)
    rel = rows[:, 5].min()
    us = lambda x: [round(float(v) / 1000, 2) for v in (x.min(), x.double().median(), x.max())]
    out = {"us_per_launch": round(per_launch_us, 2), "ctas": len(rows),
           "entry_minus_wait_us(min/med/max)": us(rows[:, 4] - rel),
           "wait_spread_us": us(rows[:, 5] - rel),
           "end_minus_wait_us": us(rows[:, 6] - rel)}
    ntile = (rows[:, 64:80] > 0).sum(1)
    for n in sorted(set(ntile.tolist())):
        r = rows[ntile == n]
        out[f"{n}_tiles: entry_minus_wait / end_minus_wait"] = (us(r[:, 4] - rel),
                                                                us(r[:, 6] - rel))
    return out


def main():
    import torch
    if not torch.cuda.is_available():
        sys.exit("needs an sm_100a device")
    lib = _load_traced()
    reuse = (4, 32, 8, 256, 1152, 128)
    for shape in ((1, 32, 8, 4096, 4096, 128), reuse):
        print("steady chain per key tile, slot 0, shape (B, Hq, Hkv, q, kv, D) =", shape)
        for j, d in steady_chain(torch, lib, shape).items():
            print(" ", j, d)
    print("fixed costs per CTA (cycles), by key tiles, shape", reuse)
    for n, d in fixed_costs(torch, lib, reuse).items():
        print(" ", n, d)
    for shape in (reuse, (2, 16, 16, 1024, 1024, 64)):
        print("launch timeline, shape", shape)
        for key, val in launch_timeline(torch, lib, shape).items():
            print(" ", key, val)


if __name__ == "__main__":
    main()
