"""Prefill-attention benchmark (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME]
    python bench.py --impl reference ...   # the CPU restatement on host cores

Workloads (seeded N(0,1) inputs with the shapes of the configs the
reference's metric is defined on; the public datasets are not available):

* ``reuse_prefill`` (default) -- prefix-reuse prefill op: batch 4, 32 query
  heads over 8 KV heads, head_dim 128, bf16, 7 cached chunks x 128 = 896
  tokens + 256 new tokens (kv_len 1152, bottom-right offset 896).
* ``causal_op`` -- single causal op: batch 2, 16 heads, S 1024, D 64, bf16.
* ``varlen_d96`` -- 64 requests, suffix ~ U{16..512}, prefix ~ 128*U{0..64},
  32 heads MHA, D 96, fp16, packed varlen.
* ``ttft_reuse`` -- TTFT at 75% prefix reuse through the engine
  (``generate_batch``) on a random-init Qwen2.5-3B-architecture decoder, 8
  prompts x 4096 tokens sharing a warmed 3072-token prefix (its own timing
  loop; see ``run_ttft``).
* ``paged_long`` -- 32768-token int8 paged prefix (KIVI per 128-token chunk,
  16-token blocks of an 8192-block pool at a seeded permutation) + 2048 new
  tokens, 64 query / 8 KV heads, D 128, bf16.  With N GPUs the KV heads are
  split across ranks (strong scaling; each rank holds its heads' pool shard).

* ``decode`` -- decode attention of the Qwen2.5-3B-architecture model: batch 8, 16 query / 2
  KV heads, D 128, one query row over 4096 keys (split-key kernel + merge launch).
* ``quantize_store`` -- quantise-on-store of the Qwen2.5-3B-architecture warm: 24 chunks x
  128 tokens x 36 layers x 2 KV heads x D 128 bf16 into the int8 block pool
  (GB/s; one launch per chunk).
* ``cacheblend`` -- CacheBlend repair of a 3072-position stitched prefix of the
  Qwen2.5-3B-architecture model (deviation over 36 layers, top 15 %, patch; GB/s; 3 launches).
* ``long_causal`` -- long causal prefill (KV encoding of a 16384-token prompt): batch 1,
  32 query / 8 KV heads, D 128, bf16, q = kv = 16384.
* ``short_suffix`` -- reuse-dominated short-suffix prefill: 16 new tokens over a
  32768-token reused prefix, batch 8, 16 query / 2 KV heads, D 128 (the Qwen2.5-3B-architecture
  model's seam shape; split-key kernel through ``prefill_attention``; GB/s).

One step = one kernel launch over one batch (the last two: one chunk store per
chunk, and the repair's three launches).  K steps are captured in one
CUDA graph and replayed between two events on the launching stream after
0.5 s of untimed replays and W graph-replayed warm-up steps.  The e2e leg
(host inputs, copies inside the region) runs steps that share no device state
on two streams in turn, so one step's uploads overlap the previous step's
kernel and download.  Steps rotate over enough input sets that the
bytes touched exceed L2 (126 MB).  With N > 1 (torchrun) the elapsed time is
the max over ranks; only that scalar crosses ranks (no data-path collective).
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
# what the CPU legs run, per workload family
TORCH_PATH = ("the reference's CPU dispatch restated as its own torch calls (oracle/sdpa_ref.py, "
              "bit-identical to its outputs): SDPA in the inputs' dtype")
NUMPY_PATH = "the reference's arithmetic restated in numpy (oracle/)"
# Untimed replays of the warm-up graph before the timed region, so that the
# timed steps run at the clocks the GPU holds under load rather than during
# its ramp from idle.
PREWARM_S = 0.5

# dram__bytes_read.sum + dram__bytes_write.sum of one launch from the committed
# ncu captures (profiles/*.md), per workload.  varlen_d96: the 16-request capture
# (1 029.9 MB) scaled to the full launch by algorithmic bytes (3 535.4 / 1 004.1 MB).
NCU_TRAFFIC_BYTES = {"reuse_prefill": 27328000, "varlen_d96": 3626150000,
                     # the batched 24-chunk launch (staged kernels): 113.4 MB read + 30.7 MB written
                     # (the rest of the pool writes still in L2 at the end)
                     "quantize_store": 113353728 + 30690304,
                     # per step: deviation 113 267 968 + 3 780 096, select 47 616,
                     # patch 16 965 632 + 14 080 (read + write)
                     "cacheblend": 134075392,
                     # split-key kernel, 33 647 616 read (the merged partials stay in L2)
                     "decode": 33647616,
                     # split-key kernel (dual CTAs merging in-kernel): 269 853 952 read
                     # + 11 240 192 written
                     "short_suffix": 281094144}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="kvboost", choices=["kvboost", "reference"])
    ap.add_argument("--workload", default="reuse_prefill",
                    choices=["reuse_prefill", "causal_op", "varlen_d96", "paged_long",
                             "ttft_reuse", "paged_long_cp", "decode", "quantize_store",
                             "cacheblend", "short_suffix", "long_causal"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sharded", action="store_true",
                    help="skip the long paged prefill sharded over the ranks that the "
                         "default workload's line carries beside its own number")
    ap.add_argument("--varlen-split", default="replicate", choices=["replicate", "lpt"],
                    help="varlen_d96 with N > 1: every rank runs the whole batch (weak "
                         "scaling) or the 64 requests are placed longest-first over the "
                         "ranks (strong scaling, no collective)")
    ap.add_argument("--kv-bits", type=int, default=16, choices=[16, 8],
                    help="ttft_reuse: the engine's chunk store (8: KIVI int8 block pool, "
                         "quantised on store, dequantised on assembly)")
    ap.add_argument("--recompute", default="selective", choices=["selective", "cacheblend", "none"],
                    help="ttft_reuse: seam repair of the single-prompt generate() timed "
                         "beside the batch (generate_batch itself repairs no seams)")
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--cp-gather", default="peers", choices=["peers", "nccl"],
                    help="paged_long_cp: read peers' shards in place over NVLink inside the "
                         "dequantise kernel (peers) or all-gather them with NCCL first")
    ap.add_argument("--small", action="store_true",
                    help="a reduced case of the workload for profiler captures (paged_long: "
                         "8192-token prefix + 1024 new tokens; varlen_d96: first 16 requests)")
    return ap.parse_args()


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["bf16_tflops"]), float(d["hbm_gbs"]), "measured"
    return 1590.0, 6650.0, "fallback"


# ───────────────────────────────────────────────────────────── workloads ──

class Dense:
    """Dense ``[B, H, S, D]`` prefill (configs 1 and 2)."""

    def __init__(self, name, B, Hq, Hkv, Sq, P, D, dtype, desc):
        self.name, self.B, self.Hq, self.Hkv, self.Sq, self.P, self.D = name, B, Hq, Hkv, Sq, P, D
        self.dtype_name, self.desc = dtype, desc
        self.kv = P + Sq
        self.scaling = "weak"
        self.bound = "tensor"
        self.e2e_overlap = True   # e2e steps share no device state

    def flops(self):
        from oracle.attention import attention_flops
        return attention_flops([self.Sq] * self.B, [self.kv] * self.B, self.Hq, self.D)

    def bytes(self):
        return self.B * 2 * (2 * self.Hq * self.Sq * self.D + 2 * self.Hkv * self.kv * self.D)

    def tokens(self):
        return self.B * self.Sq

    def config(self):
        return {"batch": self.B, "q_heads": self.Hq, "kv_heads": self.Hkv, "q_len": self.Sq,
                "kv_len": self.kv, "head_dim": self.D}

    def setup(self, torch, dev, rank, world):
        from kvboost_b200 import ops
        dt = torch.bfloat16 if self.dtype_name == "bf16" else torch.float16
        self.dt = dt
        g = torch.Generator(device=dev).manual_seed(1234 + rank)
        R = max(2, math.ceil(2 * L2_BYTES / self.bytes()))
        self.sets_desc = f"inputs rotate over {R} sets ({R * self.bytes() / 2**20:.0f} MiB > L2)"
        sets = []
        for _ in range(R):
            q = torch.randn(self.B, self.Hq, self.Sq, self.D, generator=g, device=dev).to(dt)
            k = torch.randn(self.B, self.Hkv, self.kv, self.D, generator=g, device=dev).to(dt)
            v = torch.randn(self.B, self.Hkv, self.kv, self.D, generator=g, device=dev).to(dt)
            sets.append((q, k, v, torch.empty_like(q)))
        scale = 1.0 / math.sqrt(self.D)

        def step(i):
            q, k, v, o = sets[i % R]
            ops.prefill_attention(q, k, v, scale, True, out=o, return_lse=False)
        return step

    def e2e(self, torch, dev):
        """Through the function a patched HF attention module calls
        (``flash_attn_ext.kvboost_attention_forward``, the registry entry): Q/K/V
        uploaded from pinned host memory every step, HF's bottom-right bool mask
        (built once, as HF builds one mask per forward for every layer; ``None``
        with ``is_causal`` when q == kv, as HF passes it), O read back."""
        from kvboost_b200.flash_attn_ext import kvboost_attention_forward
        hq = torch.randn(self.B, self.Hq, self.Sq, self.D).to(self.dt).pin_memory()
        hk = torch.randn(self.B, self.Hkv, self.kv, self.D).to(self.dt).pin_memory()
        hv = torch.randn(self.B, self.Hkv, self.kv, self.D).to(self.dt).pin_memory()
        ho = [torch.empty(self.B, self.Sq, self.Hq, self.D, dtype=self.dt).pin_memory()
              for _ in range(2)]
        scale = 1.0 / math.sqrt(self.D)
        mask = None
        if self.Sq != self.kv:
            mask = torch.ones(self.Sq, self.kv, dtype=torch.bool, device=dev).tril(self.kv - self.Sq)
            mask = mask[None, None].expand(self.B, 1, self.Sq, self.kv)

        def step(slot=0):
            dq, dk, dv = (t.to(dev, non_blocking=True) for t in (hq, hk, hv))
            o, _ = kvboost_attention_forward(None, dq, dk, dv, mask, scaling=scale, is_causal=True)
            ho[slot].copy_(o, non_blocking=True)
        h2d = sum(t.numel() * t.element_size() for t in (hq, hk, hv))
        return step, h2d, ho[0].numel() * ho[0].element_size()

    def gpu_sdpa(self, torch, dev):
        """The reference's GPU fallback on the same shapes: its ``torch_flash`` tier
        runs ``F.scaled_dot_product_attention`` with K/V repeated to the query heads
        and the bottom-right bool mask HF builds (``flash_attn_ext.py:86-103``)."""
        import torch.nn.functional as F
        g = torch.Generator(device=dev).manual_seed(77)
        q = torch.randn(self.B, self.Hq, self.Sq, self.D, generator=g, device=dev).to(self.dt)
        k = torch.randn(self.B, self.Hkv, self.kv, self.D, generator=g, device=dev).to(self.dt)
        v = torch.randn(self.B, self.Hkv, self.kv, self.D, generator=g, device=dev).to(self.dt)
        rep = self.Hq // self.Hkv
        mask = torch.ones(self.Sq, self.kv, dtype=torch.bool, device=dev).tril(self.kv - self.Sq)

        def run():
            kk = k.repeat_interleave(rep, 1) if rep > 1 else k
            vv = v.repeat_interleave(rep, 1) if rep > 1 else v
            F.scaled_dot_product_attention(q, kk, vv, attn_mask=mask, scale=1.0 / math.sqrt(self.D))
        return run

    # the CPU sample: this many batch elements and query heads of one step
    cpu_batch = None
    cpu_heads = None

    def cpu_sample(self, np):
        """The reference's CPU path (``oracle.sdpa_ref``: torch SDPA in the inputs' dtype,
        K/V expanded to the query heads, HF's bottom-right mask) on ``cpu_batch``
        batch elements x ``cpu_heads`` query heads (with their KV heads) of one step."""
        import torch
        from oracle import sdpa_ref
        from oracle.attention import attention_flops
        nb = self.cpu_batch or self.B
        nh = self.cpu_heads or self.Hq
        group = self.Hq // self.Hkv
        nkv = max(1, nh // group)
        dt = torch.bfloat16 if self.dtype_name == "bf16" else torch.float16
        g = torch.Generator().manual_seed(0)
        q = torch.randn(nb, nh, self.Sq, self.D, generator=g).to(dt)
        k = torch.randn(nb, nkv, self.kv, self.D, generator=g).to(dt)
        v = torch.randn(nb, nkv, self.kv, self.D, generator=g).to(dt)
        fl = attention_flops([self.Sq] * nb, [self.kv] * nb, nh, self.D)
        scale = 1.0 / math.sqrt(self.D)

        def run():
            sdpa_ref.reuse_prefill(q, k, v, scale)
        what = ("the whole step" if (nb, nh) == (self.B, self.Hq)
                else f"{nb} of {self.B} batch elements x {nh} of {self.Hq} query heads")
        return run, fl, what


class Decode(Dense):
    """Decode attention of the Qwen2.5-3B-architecture model at its 4096-token context: batch 8, 16
    query heads over 2 KV heads, D 128, bf16, one query row per head
    (``decode_attention``: GQA heads packed per key tile, keys split over CTAs).
    HBM-bound: every launch streams the 8 x 2 x 4096 keys and values once."""

    def __init__(self):
        super().__init__("decode", 8, 16, 2, 1, 4095, 128, "bf16",
                         "decode attention: B8 Hq16/Hkv2 D128 bf16, 1 query row over 4096 keys")
        self.bound = "hbm"
        self.launches_per_step = 2    # split-key kernel + merge of its partials

    def setup(self, torch, dev, rank, world):
        from kvboost_b200 import ops
        self.dt = torch.bfloat16
        g = torch.Generator(device=dev).manual_seed(4321 + rank)
        R = max(2, math.ceil(2 * L2_BYTES / self.bytes()))
        self.sets_desc = f"inputs rotate over {R} sets ({R * self.bytes() / 2**20:.0f} MiB > L2)"
        sets = []
        for _ in range(R):
            q = torch.randn(self.B, self.Hq, self.Sq, self.D, generator=g, device=dev).to(self.dt)
            k = torch.randn(self.B, self.Hkv, self.kv, self.D, generator=g, device=dev).to(self.dt)
            v = torch.randn(self.B, self.Hkv, self.kv, self.D, generator=g, device=dev).to(self.dt)
            sets.append((q, k, v, torch.empty_like(q)))
        scale = 1.0 / math.sqrt(self.D)
        ops.decode_attention(*sets[0][:3], scale, True, out=sets[0][3], return_lse=False)

        def step(i):
            q, k, v, o = sets[i % R]
            ops.decode_attention(q, k, v, scale, True, out=o, return_lse=False)
        return step

    def e2e(self, torch, dev):
        from kvboost_b200 import ops
        hq = torch.randn(self.B, self.Hq, self.Sq, self.D).to(self.dt).pin_memory()
        hk = torch.randn(self.B, self.Hkv, self.kv, self.D).to(self.dt).pin_memory()
        hv = torch.randn(self.B, self.Hkv, self.kv, self.D).to(self.dt).pin_memory()
        ho = [torch.empty(self.B, self.Hq, self.Sq, self.D, dtype=self.dt).pin_memory()
              for _ in range(2)]
        scale = 1.0 / math.sqrt(self.D)

        def step(slot=0):
            dq, dk, dv = (t.to(dev, non_blocking=True) for t in (hq, hk, hv))
            o, _ = ops.decode_attention(dq, dk, dv, scale, True, return_lse=False)
            ho[slot].copy_(o, non_blocking=True)
        h2d = sum(t.numel() * t.element_size() for t in (hq, hk, hv))
        return step, h2d, ho[0].numel() * ho[0].element_size()


class LongCausal(Dense):
    """Long causal prefill: the KV encoding of one 16384-token prompt (q = kv), 32 query
    heads over 8 KV heads, D 128, bf16.  Tensor-bound; many waves of query-tile pairs."""

    def __init__(self):
        super().__init__("long_causal", 1, 32, 8, 16384, 0, 128, "bf16",
                         "long causal prefill: B1 Hq32/Hkv8 D128 bf16, q = kv = 16384")

    def gpu_sdpa(self, torch, dev):
        """The reference's torch tier for q == kv without a mask
        (``flash_attn_ext.py:86-95``): SDPA with ``is_causal`` over K/V repeated to the
        query heads."""
        import torch.nn.functional as F
        g = torch.Generator(device=dev).manual_seed(77)
        q = torch.randn(self.B, self.Hq, self.Sq, self.D, generator=g, device=dev).to(self.dt)
        k = torch.randn(self.B, self.Hkv, self.kv, self.D, generator=g, device=dev).to(self.dt)
        v = torch.randn(self.B, self.Hkv, self.kv, self.D, generator=g, device=dev).to(self.dt)
        rep = self.Hq // self.Hkv

        def run():
            F.scaled_dot_product_attention(q, k.repeat_interleave(rep, 1), v.repeat_interleave(rep, 1),
                                           is_causal=True, scale=1.0 / math.sqrt(self.D))
        return run

    cpu_heads = 1      # one query head of the full causal square: ~0.2 s on the host


class ShortSuffix(Dense):
    """Reuse-dominated short-suffix prefill: the selective-recompute seam shape of the
    Qwen2.5-3B-architecture model (16 query heads over 2 KV heads, D 128, bf16, 16 new tokens) over a
    32 768-token reused prefix, batch 8, through ``prefill_attention`` (which takes the
    split-key kernel for it).  HBM-bound: every launch streams the reused K/V once."""

    def __init__(self):
        super().__init__("short_suffix", 8, 16, 2, 16, 32768, 128, "bf16",
                         "short-suffix reuse prefill: B8 Hq16/Hkv2 D128 bf16, 16 new tokens "
                         "over a 32768-token reused prefix (split-key kernel)")
        self.bound = "hbm"
        self.launches_per_step = 2    # split-key kernel + merge of its 128-row partials
        self.cpu_batch = 1

    def setup(self, torch, dev, rank, world):
        from kvboost_b200 import ops
        self.dt = torch.bfloat16
        g = torch.Generator(device=dev).manual_seed(99 + rank)
        R = max(2, math.ceil(2 * L2_BYTES / self.bytes()))
        self.sets_desc = f"inputs rotate over {R} sets ({R * self.bytes() / 2**20:.0f} MiB > L2)"
        sets = []
        for _ in range(R):
            q = torch.randn(self.B, self.Hq, self.Sq, self.D, generator=g, device=dev).to(self.dt)
            k = torch.randn(self.B, self.Hkv, self.kv, self.D, generator=g, device=dev).to(self.dt)
            v = torch.randn(self.B, self.Hkv, self.kv, self.D, generator=g, device=dev).to(self.dt)
            sets.append((q, k, v, torch.empty_like(q)))
        scale = 1.0 / math.sqrt(self.D)

        def step(i):
            q, k, v, o = sets[i % R]
            ops.prefill_attention(q, k, v, scale, True, out=o, return_lse=False)
        return step

    def e2e(self, torch, dev):
        """The reused prefix's K/V is device-resident (the chunk store); each step
        uploads the suffix's Q and its 16 new K/V rows into the cache tail, runs the
        public op and reads O back."""
        from kvboost_b200 import ops
        g = torch.Generator().manual_seed(17)
        hq = torch.randn(self.B, self.Hq, self.Sq, self.D, generator=g).to(self.dt).pin_memory()
        hk = torch.randn(self.B, self.Hkv, self.Sq, self.D, generator=g).to(self.dt).pin_memory()
        hv = torch.randn(self.B, self.Hkv, self.Sq, self.D, generator=g).to(self.dt).pin_memory()
        caches = [(torch.randn(self.B, self.Hkv, self.kv, self.D, device=dev).to(self.dt),
                   torch.randn(self.B, self.Hkv, self.kv, self.D, device=dev).to(self.dt))
                  for _ in range(2)]   # one per e2e stream slot
        ho = [torch.empty(self.B, self.Hq, self.Sq, self.D, dtype=self.dt).pin_memory()
              for _ in range(2)]
        scale = 1.0 / math.sqrt(self.D)

        def step(slot=0):
            dk, dv = caches[slot]
            dk[:, :, self.P:].copy_(hk, non_blocking=True)
            dv[:, :, self.P:].copy_(hv, non_blocking=True)
            dq = hq.to(dev, non_blocking=True)
            o, _ = ops.prefill_attention(dq, dk, dv, scale, True, return_lse=False)
            ho[slot].copy_(o, non_blocking=True)
        h2d = sum(t.numel() * t.element_size() for t in (hq, hk, hv))
        return step, h2d, ho[0].numel() * ho[0].element_size()


class Varlen:
    """Packed varlen reuse prefill: 64 requests, 32 heads MHA, head_dim 96, fp16."""

    def __init__(self, small=False):
        import torch
        self.name, self.Hq, self.Hkv, self.D, self.dtype_name = "varlen_d96", 32, 32, 96, "fp16"
        g = torch.Generator().manual_seed(0)
        self.sq, self.pre = [], []
        for _ in range(64):
            self.sq.append(int(torch.randint(16, 513, (1,), generator=g)))
            self.pre.append(128 * int(torch.randint(0, 65, (1,), generator=g)))
        if small:
            self.sq, self.pre = self.sq[:16], self.pre[:16]
        self.skv = [a + b for a, b in zip(self.sq, self.pre)]
        self.desc = ("varlen: 64 requests, suffix U{16..512}, prefix 128*U{0..64}, "
                     "32 heads MHA, D96, fp16")
        self.scaling = "weak"
        self.bound = "hbm"
        self.e2e_overlap = True

    def flops(self):
        from oracle.attention import attention_flops
        return attention_flops(self.sq, self.skv, self.Hq, self.D)

    def bytes(self):
        return 2 * self.D * (2 * self.Hq * sum(self.sq) + 2 * self.Hkv * sum(self.skv))

    def tokens(self):
        return getattr(self, "all_tokens", sum(self.sq))

    def work(self):
        """Per-rank share of the job's FLOPs (the value line multiplies by N)."""
        return getattr(self, "all_flops", None) or self.flops()

    def shard(self, rank, world):
        """Keep this rank's requests of a longest-processing-time-first placement of
        the batch over ``world`` ranks (every rank computes the same placement)."""
        from kvboost_b200.sharding import lpt_partition, request_cost
        from oracle.attention import attention_flops
        self.all_flops = attention_flops(self.sq, self.skv, self.Hq, self.D) / world
        self.all_tokens = sum(self.sq)
        if world > len(self.sq):
            raise SystemExit(f"varlen_d96 --varlen-split lpt: {len(self.sq)} requests cannot "
                             f"give each of {world} ranks one")
        costs = [request_cost(a, b, self.Hq, self.Hkv, self.D) for a, b in zip(self.sq, self.skv)]
        mine = lpt_partition(costs, world)[rank]
        self.sq = [self.sq[i] for i in mine]
        self.pre = [self.pre[i] for i in mine]
        self.skv = [self.skv[i] for i in mine]
        self.scaling = "strong"
        self.desc += f"; requests placed longest-first over {world} ranks"

    def config(self):
        return {"requests": len(self.sq), "q_heads": self.Hq, "kv_heads": self.Hkv, "head_dim": self.D,
                "total_q": sum(self.sq), "total_kv": sum(self.skv)}

    def _packed(self, torch, dev, g):
        import numpy as np
        cu_q = torch.tensor(np.concatenate([[0], np.cumsum(self.sq)]), dtype=torch.int32, device=dev)
        cu_k = torch.tensor(np.concatenate([[0], np.cumsum(self.skv)]), dtype=torch.int32, device=dev)
        q = torch.randn(sum(self.sq), self.Hq, self.D, generator=g, device=dev).half()
        k = torch.randn(sum(self.skv), self.Hkv, self.D, generator=g, device=dev).half()
        v = torch.randn(sum(self.skv), self.Hkv, self.D, generator=g, device=dev).half()
        return q, k, v, cu_q, cu_k

    def setup(self, torch, dev, rank, world):
        from kvboost_b200 import ops
        g = torch.Generator(device=dev).manual_seed(4 + rank)
        R = 2  # one set is already > L2; two keep consecutive steps on distinct data
        self.sets_desc = f"inputs rotate over {R} sets ({R * self.bytes() / 2**30:.1f} GiB > L2)"
        sets = [self._packed(torch, dev, g) for _ in range(R)]
        outs = [torch.empty_like(s[0]) for s in sets]

        def step(i):
            q, k, v, cq, ck = sets[i % R]
            ops.prefill_attention_varlen(q, k, v, cq, ck, max(self.sq), max(self.skv),
                                         1.0 / math.sqrt(self.D), True, out=outs[i % R],
                                         return_lse=False)
        return step

    def e2e(self, torch, dev):
        from kvboost_b200 import ops
        q, k, v, cq, ck = self._packed(torch, "cpu", torch.Generator().manual_seed(9))
        hq, hk, hv = (t.pin_memory() for t in (q, k, v))
        ho = [torch.empty_like(hq).pin_memory() for _ in range(2)]
        cq, ck = cq.to(dev), ck.to(dev)

        def step(slot=0):
            dq, dk, dv = (t.to(dev, non_blocking=True) for t in (hq, hk, hv))
            o, _ = ops.prefill_attention_varlen(dq, dk, dv, cq, ck, max(self.sq), max(self.skv),
                                                1.0 / math.sqrt(self.D), True, return_lse=False)
            ho[slot].copy_(o, non_blocking=True)
        h2d = sum(t.numel() * t.element_size() for t in (hq, hk, hv))
        return step, h2d, ho[0].numel() * ho[0].element_size()

    def cpu_sample(self, np):
        """The reference's CPU path per request (``oracle.sdpa_ref``: fp16 SDPA with the
        request's bottom-right mask, MHA) on the first 8 of the 64 requests."""
        import torch
        from oracle import sdpa_ref
        from oracle.attention import attention_flops
        n = 8
        sq, skv = self.sq[:n], self.skv[:n]
        g = torch.Generator().manual_seed(0)
        reqs = [tuple(torch.randn(1, self.Hq, m, self.D, generator=g).half() for m in (a, b, b))
                for a, b in zip(sq, skv)]
        fl = attention_flops(sq, skv, self.Hq, self.D)

        def run():
            for q, k, v in reqs:
                sdpa_ref.reuse_prefill(q, k, v, 1.0 / math.sqrt(self.D))
        return run, fl, f"the first {n} of {len(self.sq)} requests"


class PagedLong:
    """Paged int8 reuse: 32K-token prefix + 2048 new tokens, KV heads split over ranks."""

    def __init__(self, small=False):
        self.name = "paged_long"
        self.B, self.Hq, self.Hkv, self.D, self.Sq, self.P = 1, 64, 8, 128, 2048, 32768
        self.num_blocks = 8192
        if small:
            self.Sq, self.P, self.num_blocks = 1024, 8192, 2048
        self.dtype_name = "bf16"
        self.desc = ("paged int8 reuse: P 32768 (KIVI int8, 16-token blocks, 8192-block pool, "
                     "seeded permutation) + 2048 new tokens, Hq64/Hkv8, D128, bf16")
        self.scaling = "strong"
        self.bound = "tensor"
        self.world = 1
        self.launches_per_step = 2    # dequantise-once materialise + attention
        self.e2e_overlap = True

    def local_heads(self, rank, world):
        if self.Hkv % world:
            raise SystemExit(f"paged_long splits 8 KV heads; --gpus {world} does not divide 8")
        hk = self.Hkv // world
        return hk, hk * (self.Hq // self.Hkv)

    def flops(self):
        from oracle.attention import attention_flops
        _, hq = self.local_heads(0, self.world)
        return attention_flops([self.Sq], [self.P + self.Sq], hq, self.D)

    def bytes(self):
        hk, hq = self.local_heads(0, self.world)
        nblk = self.P // 16
        pool = nblk * hk * (2 * 16 * self.D + 4 * 16 + 4 * self.D)   # int8 K/V + fp32 scales
        return pool + 2 * (2 * hq * self.Sq * self.D + 2 * hk * self.Sq * self.D)

    def tokens(self):
        return self.Sq

    def config(self):
        return {"batch": 1, "q_heads": self.Hq, "kv_heads": self.Hkv, "head_dim": self.D,
                "prefix_tokens": self.P, "q_len": self.Sq, "pool_blocks": self.num_blocks,
                "block_size": 16, "kv_storage": "int8 KIVI, fp32 copies of fp16 scales"}

    def _pool(self, torch, dev, hk, seed):
        from kvboost_b200.paged import DeviceBlockAllocator, quantize_chunk_int8
        g = torch.Generator(device=dev).manual_seed(seed)
        alloc = DeviceBlockAllocator(1, hk, self.D, self.num_blocks, device=dev)
        perm = torch.randperm(self.num_blocks, generator=torch.Generator().manual_seed(seed))
        table = perm[: self.P // 16].tolist()
        for c in range(self.P // 128):
            k = torch.randn(1, hk, 128, self.D, generator=g, device=dev).to(torch.bfloat16).half()
            v = torch.randn(1, hk, 128, self.D, generator=g, device=dev).to(torch.bfloat16).half()
            alloc.write_chunk_int8(0, table[8 * c: 8 * c + 8], *quantize_chunk_int8(k, v))
        bt = torch.tensor([table], dtype=torch.int32, device=dev)
        return alloc, bt

    def setup(self, torch, dev, rank, world):
        from kvboost_b200.paged import paged_prefill_attention
        self.world = world
        hk, hq = self.local_heads(rank, world)
        R = 2
        sets = []
        for r in range(R):
            alloc, bt = self._pool(torch, dev, hk, seed=100 + 7 * rank + r)
            g = torch.Generator(device=dev).manual_seed(200 + rank + r)
            q = torch.randn(1, hq, self.Sq, self.D, generator=g, device=dev).to(torch.bfloat16)
            kn = torch.randn(1, hk, self.Sq, self.D, generator=g, device=dev).to(torch.bfloat16)
            vn = torch.randn(1, hk, self.Sq, self.D, generator=g, device=dev).to(torch.bfloat16)
            sets.append((q, kn, vn, alloc, bt, torch.empty_like(q)))
        self.sets_desc = (f"{R} pools x {self.bytes() / 2**20:.0f} MiB touched per step > L2; "
                          f"rank holds KV heads {rank * hk}..{(rank + 1) * hk - 1}")
        self.e2e_set = sets[0]

        def step(i):
            q, kn, vn, alloc, bt, o = sets[i % R]
            paged_prefill_attention(q, kn, vn, alloc, 0, bt, self.P, out=o, return_lse=False)
        return step

    def e2e(self, torch, dev):
        """Suffix Q/K/V and the block table come from pinned host memory; the int8
        pool is the device-resident chunk cache."""
        from kvboost_b200.paged import paged_prefill_attention
        q, kn, vn, alloc, bt, _ = self.e2e_set
        hq, hk_, hv = (t.cpu().pin_memory() for t in (q, kn, vn))
        hbt = bt.cpu().pin_memory()
        ho = [torch.empty_like(hq).pin_memory() for _ in range(2)]

        def step(slot=0):
            dq, dk, dv, dbt = (t.to(dev, non_blocking=True) for t in (hq, hk_, hv, hbt))
            o, _ = paged_prefill_attention(dq, dk, dv, alloc, 0, dbt, self.P, return_lse=False)
            ho[slot].copy_(o, non_blocking=True)
        h2d = sum(t.numel() * t.element_size() for t in (hq, hk_, hv, hbt))
        return step, h2d, ho[0].numel() * ho[0].element_size()

    def cpu_sample(self, np):
        """One KV-head group (1 KV head, its 8 query heads) of the full step through the
        reference's host path (``oracle.sdpa_ref``): ``dequantize_kv`` of the int8
        chunks (float16 product), ``read_kv`` through the block table, the suffix
        appended, K/V expanded to the query heads, SDPA with the bottom-right mask."""
        import torch
        from oracle import sdpa_ref
        from oracle.attention import attention_flops
        g = torch.Generator().manual_seed(0)
        nblk, grp = self.P // 16, self.Hq // self.Hkv
        pool_q = torch.randint(-127, 128, (self.num_blocks, 2, 1, 16, self.D), generator=g,
                               dtype=torch.int8)
        k_scale = (torch.rand(self.num_blocks, 1, 16, 1, generator=g) / 40 + 1e-3).half()
        v_scale = (torch.rand(self.num_blocks, 1, 1, self.D, generator=g) / 40 + 1e-3).half()
        table = torch.randperm(self.num_blocks, generator=g)[:nblk].tolist()
        q = torch.randn(1, grp, self.Sq, self.D, generator=g).bfloat16()
        kn = torch.randn(1, 1, self.Sq, self.D, generator=g).bfloat16()
        vn = torch.randn(1, 1, self.Sq, self.D, generator=g).bfloat16()
        fl = attention_flops([self.Sq], [self.P + self.Sq], grp, self.D)

        def run():
            used = pool_q[table]      # the reused chunks' blocks, dequantised, in table order
            pool = torch.stack([sdpa_ref.dequantize_int8(used[:, 0], k_scale[table]),
                                sdpa_ref.dequantize_int8(used[:, 1], v_scale[table])], 1)
            k, v = sdpa_ref.read_kv(pool.bfloat16(), range(nblk), self.P)
            K = torch.cat([k[None], kn], dim=2)
            V = torch.cat([v[None], vn], dim=2)
            sdpa_ref.reuse_prefill(q, K, V, 1.0 / math.sqrt(self.D))
        return run, fl, f"1 of {self.Hkv} KV-head groups ({grp} query heads)"


class QuantizeStore:
    """Quantise-on-store of freshly encoded chunks (``kvb_quantize_store``): the Qwen2.5-3B-architecture
    model's warm of a 3072-token prefix -- 24 chunks of 128 tokens, 36 layers, 2 KV
    heads, D 128 -- each chunk's bf16 K/V read as the model's cache holds them
    ([1, H, S, D] views of [1, S, H, D] projections), KIVI int8 + scales written into
    its 8 blocks of the int8 pool.  One launch stores the 24 chunks, all layers
    (``store_chunks_int8``, as the engine's warm does)."""

    metric, unit, unit_scale, dtype_name = "quantize-on-store GB/s", "GB/s", 1e9, "bf16->int8"

    def __init__(self):
        self.name, self.L, self.H, self.S, self.D, self.chunks = "quantize_store", 36, 2, 128, 128, 24
        self.nblk = self.S // 16
        self.desc = ("quantise-on-store: 24 chunks x 128 tokens, 36 layers, 2 KV heads, D 128, "
                     "bf16 model-cache K/V -> KIVI int8 16-token blocks + fp16/fp32 scales")
        self.scaling, self.bound = "weak", "hbm"
        self.launches_per_step = 1

    def chunk_bytes(self):
        L, H, S, D, n = self.L, self.H, self.S, self.D, self.nblk
        return (L * H * S * D * 2 * 2            # bf16 K and V read
                + L * H * n * 16 * D * 2         # int8 K and V rows written
                + L * H * n * 16 * 6             # K scales, fp16 + fp32
                + n * L * H * D * 6)             # V scales in every block, fp16 + fp32

    def bytes(self):
        return self.chunks * self.chunk_bytes()

    work = bytes

    def flops(self):
        return 0

    def tokens(self):
        return self.chunks * self.S

    def config(self):
        return {"chunks": self.chunks, "chunk_tokens": self.S, "layers": self.L,
                "kv_heads": self.H, "head_dim": self.D, "block_size": 16}

    def _chunks(self, torch, dev, g):
        out = []
        for _ in range(self.chunks):
            raw = [torch.randn(2, 1, self.S, self.H, self.D, generator=g, device=dev)
                   .to(torch.bfloat16) for _ in range(self.L)]
            out.append(([r[0].transpose(1, 2) for r in raw], [r[1].transpose(1, 2) for r in raw]))
        return out

    def setup(self, torch, dev, rank, world):
        from kvboost_b200.paged import DeviceBlockAllocator
        g = torch.Generator(device=dev).manual_seed(99 + rank)
        R = max(2, math.ceil(2 * L2_BYTES / self.bytes()))
        self.alloc = DeviceBlockAllocator(self.L, self.H, self.D, R * self.chunks * self.nblk,
                                          device=dev)
        sets = []
        for _ in range(R):
            chunks = self._chunks(torch, dev, g)
            blocks = [self.alloc.allocate(self.nblk) for _ in range(self.chunks)]
            sets.append(self.alloc.prepare_chunks_int8(
                [(b, ks, vs) for (ks, vs), b in zip(chunks, blocks)]))
        torch.cuda.synchronize()
        self.sets_desc = f"inputs rotate over {R} sets ({R * self.bytes() / 2**20:.0f} MiB > L2)"

        def step(i):
            self.alloc.launch_prepared(sets[i % R])
        return step

    def e2e(self, torch, dev):
        """Each chunk's K/V from pinned host memory, stored, and its int8 blocks and
        scales read back to pinned host memory."""
        g = torch.Generator().manual_seed(5)
        hk = torch.randn(self.L, self.H, self.S, self.D, generator=g).to(torch.bfloat16).pin_memory()
        hv = torch.randn(self.L, self.H, self.S, self.D, generator=g).to(torch.bfloat16).pin_memory()
        blocks = self.alloc.allocate(self.nblk) if self.alloc.free_blocks >= self.nblk else \
            list(range(self.nblk))
        idx = torch.tensor(blocks, device=dev)
        hp = torch.empty(self.L, self.nblk, 2, self.H, 16, self.D, dtype=torch.int8).pin_memory()

        def step():
            for _ in range(self.chunks):
                dk, dv = hk.to(dev, non_blocking=True), hv.to(dev, non_blocking=True)
                self.alloc.store_chunk_int8(blocks, dk, dv)
                hp.copy_(torch.stack([p[idx] for p in self.alloc.pools]), non_blocking=True)
        h2d = self.chunks * 2 * hk.numel() * 2
        return step, h2d, self.chunks * hp.numel()
    # (e2e: one chunk per call through the public single-chunk store, the
    # reference's store granularity)

    def gpu_reference(self, torch, dev):
        """The reference's store arithmetic as torch ops on this GPU
        (``_quantize_int8`` per layer, then the block scatter of ``write_chunk_int8``)."""
        from kvboost_b200.paged import quantize_chunk_int8
        chunks = self._chunks(torch, dev, torch.Generator(device=dev).manual_seed(3))
        blocks = list(range(self.nblk))

        def run():
            for ks, vs in chunks:
                for layer in range(self.L):
                    self.alloc.write_chunk_int8(layer, blocks, *quantize_chunk_int8(ks[layer],
                                                                                    vs[layer]))
        return run, "torch ops: _quantize_int8 per layer + write_chunk_int8 scatter"

    cpu_path = NUMPY_PATH

    def cpu_sample(self, np):
        """One chunk, all layers: the reference's bf16 quantisation arithmetic (numpy)."""
        from oracle.kv_quant import quantize_int8_model_dtype, round_to_bf16
        g = np.random.default_rng(0)
        k = round_to_bf16(g.standard_normal((self.L, self.H, self.S, self.D), dtype=np.float32))
        v = round_to_bf16(g.standard_normal((self.L, self.H, self.S, self.D), dtype=np.float32))

        def run():
            for layer in range(self.L):
                quantize_int8_model_dtype(k[layer], v[layer], "bf16")
        return run, self.chunk_bytes(), "1 of 24 chunks (all 36 layers)"


class CacheBlendRepair:
    """CacheBlend repair of one Qwen2.5-3B-architecture prompt's stitched prefix (``kvb_cacheblend_fwd``):
    3072 cached positions, 36 layers, 2 KV heads, D 128, bf16; cosine deviation of
    cached vs full-context K over all layers, top 15 % above 0.01, patch of those
    positions' K and V.  Cached K/V stacked [L, H, S, D] (the assembled prefix), the
    full-context K/V as the model's cache holds them."""

    metric, unit, unit_scale, dtype_name = "CacheBlend repair GB/s", "GB/s", 1e9, "bf16"

    def __init__(self):
        self.name, self.L, self.H, self.S, self.D = "cacheblend", 36, 2, 3072, 128
        self.k = max(1, int(self.S * 0.15))
        self.desc = ("CacheBlend repair: 3072 cached positions, 36 layers, 2 KV heads, D 128, "
                     "bf16, top 15% above 0.01 patched")
        self.scaling, self.bound = "weak", "hbm"
        self.launches_per_step = 3

    def bytes(self):
        L, H, S, D, k = self.L, self.H, self.S, self.D, self.k
        return (2 * L * H * S * D * 2     # cached K and full-context K read (deviation)
                + S * 4 * 7               # deviation written, read by the select passes
                + k * 4                   # chosen positions
                + 2 * k * L * H * D * 2 * 2)  # K and V rows at k positions: read fresh, write cached

    work = bytes

    def flops(self):
        return 0

    def tokens(self):
        return self.S

    def config(self):
        return {"cached_positions": self.S, "layers": self.L, "kv_heads": self.H,
                "head_dim": self.D, "recompute_ratio": 0.15, "min_deviation": 0.01,
                "patched_positions": self.k}

    def _inputs(self, torch, dev, g):
        ck = torch.randn(self.L, self.H, self.S, self.D, generator=g, device=dev).to(torch.bfloat16)
        cv = torch.randn(self.L, self.H, self.S, self.D, generator=g, device=dev).to(torch.bfloat16)
        mags = torch.rand(self.S, generator=g, device=dev).view(1, self.S, 1, 1)
        raw = [(ck[l].transpose(0, 1)[None] + mags * torch.randn(1, self.S, self.H, self.D,
               generator=g, device=dev)).to(torch.bfloat16).contiguous() for l in range(self.L)]
        fk = [r.transpose(1, 2) for r in raw]
        fv = [torch.randn(1, self.S, self.H, self.D, generator=g, device=dev).to(torch.bfloat16)
              .transpose(1, 2) for _ in range(self.L)]
        return ck, cv, fk, fv

    def setup(self, torch, dev, rank, world):
        from kvboost_b200.cacheblend import cacheblend_fwd
        g = torch.Generator(device=dev).manual_seed(17 + rank)
        R = max(2, math.ceil(2 * L2_BYTES / (4 * self.L * self.H * self.S * self.D * 2)))
        sets = [self._inputs(torch, dev, g) for _ in range(R)]
        self.sets_desc = (f"inputs rotate over {R} sets "
                          f"({R * 4 * self.L * self.H * self.S * self.D * 2 / 2**20:.0f} MiB > L2)")
        self.e2e_set = sets[0]

        def step(i):
            cacheblend_fwd(*sets[i % R], 0.15, 0.01, patch=True)
        return step

    def e2e(self, torch, dev):
        """Cached and full-context K/V from pinned host memory; the chosen positions
        and count read back."""
        from kvboost_b200.cacheblend import cacheblend_fwd
        ck, cv, fk, fv = self.e2e_set
        hck, hcv = ck.cpu().pin_memory(), cv.cpu().pin_memory()
        hfk = torch.stack([t[0] for t in fk]).cpu().pin_memory()
        hfv = torch.stack([t[0] for t in fv]).cpu().pin_memory()
        hsel = torch.empty(self.k + 1, dtype=torch.int32).pin_memory()

        def step():
            d = [t.to(dev, non_blocking=True) for t in (hck, hcv, hfk, hfv)]
            _, sel, cnt = cacheblend_fwd(*d, 0.15, 0.01, patch=True)
            hsel[:self.k].copy_(sel, non_blocking=True)
            hsel[self.k:].copy_(cnt, non_blocking=True)
        h2d = sum(t.numel() * 2 for t in (hck, hcv, hfk, hfv))
        return step, h2d, hsel.numel() * 4

    def gpu_reference(self, torch, dev):
        """The reference's steps as torch ops on this GPU (``cacheblend.py:141-197``)."""
        import torch.nn.functional as F
        ck, cv, fk, fv = self._inputs(torch, dev, torch.Generator(device=dev).manual_seed(4))

        def run():
            devs = []
            for l in range(self.L):
                a = ck[l].permute(1, 0, 2).reshape(1, self.S, -1)
                b = fk[l][0].permute(1, 0, 2).reshape(1, self.S, -1)
                devs.append(1.0 - F.cosine_similarity(a, b, dim=-1))
            mean = torch.stack(devs).mean(0).squeeze(0)
            above = mean > 0.01
            masked = mean.clone()
            masked[~above] = -1.0
            _, top = masked.topk(min(self.k, int(above.sum().item())))
            idx = top.sort().values
            for l in range(self.L):
                ck[l][:, idx] = fk[l][0][:, idx]
                cv[l][:, idx] = fv[l][0][:, idx]
        return run, "torch ops: cosine_similarity per layer, mean, topk, index copy"

    cpu_path = NUMPY_PATH

    def cpu_sample(self, np):
        """The whole repair through the oracle (numpy; the reference's CPU steps)."""
        from oracle import cacheblend as ocb
        g = np.random.default_rng(0)
        ck = g.standard_normal((self.L, self.H, self.S, self.D), dtype=np.float32)
        fk = ck + g.standard_normal((self.L, self.H, self.S, self.D), dtype=np.float32) * 0.3
        cv = g.standard_normal((self.L, self.H, self.S, self.D), dtype=np.float32)
        fv = g.standard_normal((self.L, self.H, self.S, self.D), dtype=np.float32)

        def run():
            dev = ocb.deviation(ck, fk)
            ocb.patch(ck, cv, fk, fv, ocb.select(dev, self.k, 0.01))
        return run, self.bytes(), "the full repair of one prompt"


class TtftReuse:
    """TTFT at 75% prefix reuse through the engine on a random-init
    Qwen2.5-3B-architecture decoder (36 layers, hidden 2048, 16 q / 2 KV heads,
    D 128, MLP 11008, vocab 151936, bf16).  8 prompts x 4096 seeded token ids share
    a 3072-token prefix (24 chunks) warmed first; each step is one
    ``generate_batch`` call with a fresh 1024-token suffix per prompt and greedy
    decode of 64 tokens.  With N GPUs every rank serves its own batch (replicas)."""

    name = "ttft_reuse"
    B, PREFIX, SUFFIX, NEW = 8, 3072, 1024, 64
    LAYERS, HQ, HKV, D, HIDDEN, MLP, VOCAB = 36, 16, 2, 128, 2048, 11008, 151936
    dtype_name = "bf16"
    scaling = "weak"
    desc = ("TTFT at 75% reuse: random-init Qwen2.5-3B architecture (36 layers, hidden 2048, "
            "Hq16/Hkv2, D128, MLP 11008, vocab 151936, bf16), 8 prompts x 4096 tokens sharing "
            "a warmed 3072-token prefix, greedy decode of 64 tokens")

    def attn_flops(self):
        """Algorithmic FLOPs of one layer's suffix-prefill attention (one launch)."""
        from oracle.attention import attention_flops
        return attention_flops([self.SUFFIX] * self.B, [self.PREFIX + self.SUFFIX] * self.B,
                               self.HQ, self.D)

    def config(self):
        return {"batch": self.B, "prompt_tokens": self.PREFIX + self.SUFFIX,
                "shared_prefix": self.PREFIX, "suffix_tokens": self.SUFFIX,
                "new_tokens": self.NEW, "layers": self.LAYERS, "q_heads": self.HQ,
                "kv_heads": self.HKV, "head_dim": self.D, "hidden": self.HIDDEN,
                "intermediate": self.MLP, "vocab": self.VOCAB}

    def cpu_sample(self, np):
        """Attention of the suffix prefill for one prompt, one layer and one KV-head
        group (8 query heads over 1 KV head) through the reference's CPU dispatch
        (``oracle.sdpa_ref``, bf16); the projection to the whole batch multiplies by
        prompts x layers x KV heads."""
        import torch
        from oracle import sdpa_ref
        from oracle.attention import attention_flops
        g = torch.Generator().manual_seed(0)
        grp = self.HQ // self.HKV
        q = torch.randn(1, grp, self.SUFFIX, self.D, generator=g).bfloat16()
        k = torch.randn(1, 1, self.PREFIX + self.SUFFIX, self.D, generator=g).bfloat16()
        v = torch.randn(1, 1, self.PREFIX + self.SUFFIX, self.D, generator=g).bfloat16()
        fl = attention_flops([self.SUFFIX], [self.PREFIX + self.SUFFIX], grp, self.D)

        def run():
            sdpa_ref.reuse_prefill(q, k, v, 1.0 / math.sqrt(self.D))
        return run, fl, "suffix-prefill attention of 1 prompt x 1 layer x 1 KV-head group"

    def projection(self):
        return self.B * self.LAYERS * self.HKV

    def model(self, torch, dev):
        from transformers import Qwen2Config, Qwen2ForCausalLM
        cfg = Qwen2Config(vocab_size=self.VOCAB, hidden_size=self.HIDDEN,
                          intermediate_size=self.MLP, num_hidden_layers=self.LAYERS,
                          num_attention_heads=self.HQ, num_key_value_heads=self.HKV,
                          max_position_embeddings=32768, rms_norm_eps=1e-6, rope_theta=1e6,
                          tie_word_embeddings=True, initializer_range=0.02,
                          attn_implementation="sdpa")
        torch.manual_seed(0)
        old = torch.get_default_dtype()
        torch.set_default_dtype(torch.bfloat16)
        try:
            with torch.device(dev):
                m = Qwen2ForCausalLM(cfg)
        finally:
            torch.set_default_dtype(old)
        with torch.no_grad():   # weights N(0, 0.02), norms 1, biases 0
            for n, p in m.named_parameters():
                if p.dim() >= 2:
                    p.normal_(0.0, 0.02)
        return m.eval()

    def prompts(self, step, rank):
        import numpy as np
        g = np.random.default_rng(1000 + rank)
        prefix = g.integers(0, self.VOCAB, self.PREFIX).tolist()
        h = np.random.default_rng(10_000 * (rank + 1) + step)
        return prefix, [prefix + h.integers(0, self.VOCAB, self.SUFFIX).tolist()
                        for _ in range(self.B)]


def run_cp(args, torch, dist, rank, world, local, dev):
    """The paged int8 32K-prefix workload with the prefix chunks placed round-robin across the ranks (chunk c on
    rank c % N): every step all-gathers the int8 pool shards and the suffix K/V
    (NCCL over NVLink), dequantises prefix + suffix once, and runs this rank's
    zig-zag query chunks over all 64 query heads.  Strong scaling: the work of one
    prefill is split N ways."""
    import numpy as np
    from kvboost_b200 import context_parallel as cp
    from kvboost_b200 import ops
    from kvboost_b200.paged import DeviceBlockAllocator, block_table_tensor, quantize_chunk_int8
    from oracle.attention import attention_flops
    P, Sq, Hq, Hkv, D = (8192, 1024, 64, 8, 128) if args.small else (32768, 2048, 64, 8, 128)
    C = P // 128
    peers = args.cp_gather == "peers"
    g = torch.Generator(device=dev).manual_seed(300 + rank)
    rows = 2 * (Sq // (2 * world))
    if peers:
        shards = cp.PeerShardBuffer(C, world, Hkv, D, Sq, torch.bfloat16, dev,
                                    symmetric=world > 1)
        local_pool = shards.alloc
    else:
        local_pool = cp.make_shard_allocator(C, world, Hkv, D, dev)
    for slot, c in enumerate(cp.local_chunk_slots(C, world, rank)):
        k = torch.randn(1, Hkv, 128, D, generator=g, device=dev).to(torch.bfloat16).half()
        v = torch.randn(1, Hkv, 128, D, generator=g, device=dev).to(torch.bfloat16).half()
        local_pool.write_chunk_int8(0, list(range(slot * 8, slot * 8 + 8)), *quantize_chunk_int8(k, v))
    full_pool = None if peers else DeviceBlockAllocator(1, Hkv, D, world * local_pool.num_blocks,
                                                        device=dev)
    q = torch.randn(1, Hq, rows, D, generator=g, device=dev).to(torch.bfloat16)
    kl = torch.randn(1, Hkv, rows, D, generator=g, device=dev).to(torch.bfloat16)
    vl = torch.randn(1, Hkv, rows, D, generator=g, device=dev).to(torch.bfloat16)
    if peers:   # this rank's suffix rows live in its shard buffer
        shards.suffix_k.copy_(kl[0])
        shards.suffix_v.copy_(vl[0])
    out = torch.empty_like(q)
    kv_pad = (P + Sq + 127) // 128 * 128
    ws = torch.empty(2 * Hkv * kv_pad * D, dtype=torch.bfloat16, device=dev)
    table = block_table_tensor([cp.gathered_block_table(C, world)], dev)
    index = cp.zigzag_token_index(Sq, world).to(dev)
    if world > 1:
        torch.cuda.synchronize()
        dist.barrier()

    def step():
        if peers:
            cp.cp_reuse_prefill_peers(q, shards, P, rank, None, out, ws, table)
        elif world > 1:
            cp.cp_reuse_prefill(q, kl, vl, local_pool, full_pool, P, Sq, None, None, out, ws,
                                table, index)
        else:   # one rank: the shard is the whole pool, the suffix is local
            cp.cp_rank_prefill(q, local_pool, kl, vl, P, Sq, 1, 0, None, out, ws, table)

    def timed(n):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n):
            step()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([ms], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    timed(max(3, args.warmup))
    with ClockSampler(local) as clk:
        ms = timed(args.steps)
    fl_total = attention_flops([Sq], [P + Sq], Hq, D)
    value = fl_total * args.steps / (ms / 1e3) / 1e12
    # one untimed step with events around each phase (same stream)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    if world > 1:
        dist.barrier()
    ev[0].record()
    if peers:
        shards.barrier()
    elif world > 1:
        cp.gather_pool(local_pool, full_pool)
        kf, vf = cp.gather_suffix_kv(kl, vl, Sq, None, index)
    else:
        kf, vf = kl, vl
    ev[1].record()
    from kvboost_b200.paged import paged_materialize
    if peers:
        K, V = cp.materialize_from_peers(shards.bases, shards.shard_blocks, shards.zz_rows, Hkv,
                                         D, torch.bfloat16, table, P, Sq,
                                         world * shards.shard_blocks, ws)
    else:
        K, V = paged_materialize(full_pool if world > 1 else local_pool, 0, table, P, kf, vf,
                                 workspace=ws)
    ev[2].record()
    c = Sq // (2 * world)
    for j, (s0, e0_) in enumerate(cp.zigzag_chunks(Sq, world, rank)):
        ops.prefill_attention(q[:, :, j * c:(j + 1) * c], K[:, :, :P + e0_], V[:, :, :P + e0_],
                              None, True, out=out[:, :, j * c:(j + 1) * c], return_lse=False)
    ev[3].record()
    torch.cuda.synchronize()
    phases = [ev[i].elapsed_time(ev[i + 1]) for i in range(3)]
    peak_tf, _, peak_src = measured_peaks()
    rank_fl = fl_total / world       # zig-zag chunks give every rank the same causal work
    achieved = rank_fl / (phases[2] / 1e3) / 1e12
    gathered_bytes = (world - 1) * (local_pool.pools[0].numel() + 4 * local_pool.k_scale[0].numel()
                                    + 4 * local_pool.v_scale[0].numel()
                                    + 2 * 2 * kl.numel())
    line = {
        "metric": "prefill attention TFLOP/s", "value": value, "unit": "TFLOP/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "paged_long_cp" + (" (small)" if args.small else ""),
                   "desc": f"paged int8 reuse, prefix chunks round-robin over {world} ranks: "
                           f"P {P} + {Sq} new tokens, Hq{Hq}/Hkv{Hkv}, D{D}, bf16; per step "
                           + ("one kernel reads every rank's shard over NVLink and dequantises"
                              if peers else "NCCL all-gather of pool shards + suffix K/V, "
                              "dequantise once") + ", zig-zag query chunks",
                   "parallelism": f"context parallel x{world} (zig-zag query chunks)",
                   "l2": "pool, workspace and outputs > L2",
                   "timing": "CUDA events around K eager steps, max over ranks"},
        "tokens_per_s": Sq * args.steps / (ms / 1e3),
        "phase_ms": {"gather" if not peers else "barrier": phases[0],
                     "materialize" if not peers else "materialize_from_peers": phases[1],
                     "prefill": phases[2]},
        "gathered_bytes_per_rank": gathered_bytes,
        "cp_gather": args.cp_gather,
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0,
                "note": "inputs are device-resident shards by construction of this workload"},
        "gpu_launches": 3 * args.steps,   # materialise + two prefill launches per step
        "roofline": {"bound": "tensor", "kernel": "dense prefill over the rank's query chunks",
                     "achieved": achieved, "peak": peak_tf, "unit": "TFLOP/s",
                     "frac": achieved / peak_tf, "traffic": None,
                     "peak_source": f"{peak_src} bf16 dense (burst)"},
        "clocks": clk.summary(),
        "device_status": ops.read_status(dev),
    }
    if rank == 0:
        print(json.dumps(line), flush=True)


def run_ttft(args, torch, dist, rank, world, local, dev):
    """TTFT at 75% reuse through the engine (ms, lower is better)."""
    import numpy as np
    from kvboost_b200 import _lib, ops
    from kvboost_b200.engine import KVBoost
    w = TtftReuse()
    eng = KVBoost(w.model(torch, dev), None, recompute_strategy=args.recompute,
                  max_cache_bytes=48 << 30, kv_cache_bits=args.kv_bits, device=str(dev))
    prefix, _ = w.prompts(0, rank)
    eng.warm(prefix)

    def allmax(x):
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # device-side prefill: the cached prefix broadcast + 8 x 1024-token suffix forward
    # (36 layers) + argmax, inputs resident, CUDA events on the current stream
    keys, values, cached, _ = eng._assemble(prefix + [0], repair_seams=False)
    _, pr = w.prompts(10**6, rank)
    x = torch.tensor([p[cached:] for p in pr], device=dev)
    pos = torch.arange(cached, cached + w.SUFFIX, device=dev)[None].expand(w.B, -1)

    def prefill():
        cache = eng._cache_from(keys, values, w.B)
        out = eng._forward(x, pos, cache)
        return out.logits[:, -1].argmax(-1)

    for _ in range(max(3, args.warmup)):
        prefill()
    torch.cuda.synchronize()
    # attention kernel launches timed inside one forward (events on the launching stream)
    times = []
    orig = ops.prefill_attention

    def timed(*a, **k):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        r = orig(*a, **k)
        e1.record()
        times.append((e0, e1))
        return r
    ops.prefill_attention = timed
    try:
        prefill()
    finally:
        ops.prefill_attention = orig
    torch.cuda.synchronize()
    attn_ms = [a.elapsed_time(b) for a, b in times]
    dev_ms = []
    with ClockSampler(local) as clk:
        for _ in range(args.steps):
            if world > 1:
                dist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            prefill()
            e1.record()
            torch.cuda.synchronize()
            dev_ms.append(allmax(e0.elapsed_time(e1)))
    # end to end: generate_batch from host token ids to host tokens
    c0 = _lib.calls_ok
    ttft, total = [], []
    for s in range(args.warmup + args.e2e_steps):
        _, pr = w.prompts(s + 1, rank)
        if world > 1:
            dist.barrier()
        res = eng.generate_batch(pr, max_new_tokens=w.NEW)
        assert all(r.cached_tokens == w.PREFIX for r in res)
        if s >= args.warmup:
            ttft.append(allmax(res[0].ttft_ms))
            total.append(allmax(res[0].total_ms))
    launches = (_lib.calls_ok - c0) // (args.warmup + args.e2e_steps)
    # one prompt through generate(): the seam repair of --recompute runs here
    single = []
    for s in range(args.warmup + args.e2e_steps):
        _, pr = w.prompts(2000 + s, rank)
        if world > 1:
            dist.barrier()
        r = eng.generate(pr[0], max_new_tokens=1)
        assert r.cached_tokens == w.PREFIX
        if s >= args.warmup:
            single.append(allmax(r.ttft_ms))
    # the same engine on stock SDPA, for the kernel's share of TTFT
    from kvboost_b200.flash_attn_ext import install_flash_attention, uninstall_flash_attention
    uninstall_flash_attention(eng.model)
    sdpa = []
    for s in range(3):
        _, pr = w.prompts(500 + s, rank)
        res = eng.generate_batch(pr, max_new_tokens=1)
        sdpa.append(allmax(res[0].ttft_ms))
    install_flash_attention(eng.model)

    peak_tf, _, peak_src = measured_peaks()
    per_launch = statistics.mean(attn_ms) / 1e3
    afl = w.attn_flops()
    value = statistics.mean(dev_ms)
    e2e = statistics.mean(ttft)
    line = {
        "metric": "TTFT at 75% prefix reuse", "value": value, "unit": "ms",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": value, "higher_is_better": False, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded token ids, random-init)",
        "config": {"workload": w.name, "desc": w.desc, **w.config(),
                   "parallelism": f"replicas x{world}" if world > 1 else "single",
                   "l2": "model weights 6.2 GB and per-layer K/V > L2",
                   "timing": "value: CUDA events around the batched suffix prefill (cached "
                             "prefix resident); e2e: generate_batch wall clock to the first "
                             "token on the host"},
        "prefill_tokens_per_s": world * w.B * (w.PREFIX + w.SUFFIX) / (value / 1e3),
        "computed_tokens_per_s": world * w.B * w.SUFFIX / (value / 1e3),
        "e2e": {"value": e2e, "unit": "ms", "h2d_bytes_per_step": w.B * w.SUFFIX * 8,
                "d2h_bytes_per_step": w.B * w.NEW * 8, "total_ms": statistics.mean(total),
                "ttft_ms_sdpa_engine": statistics.mean(sdpa),
                "ttft_ms_samples": [round(x, 2) for x in ttft],
                "ttft_ms_single_prompt_generate": statistics.mean(single),
                "kv_cache_bits": args.kv_bits, "recompute_single_prompt": args.recompute,
                "prompt_tokens_per_s": world * w.B * (w.PREFIX + w.SUFFIX) / (e2e / 1e3)},
        "gpu_launches": launches,
        "roofline": {"bound": "tensor", "kernel": "suffix-prefill attention (per layer)",
                     "achieved": afl / per_launch / 1e12, "peak": peak_tf, "unit": "TFLOP/s",
                     "frac": afl / per_launch / 1e12 / peak_tf, "traffic": None,
                     "peak_source": f"{peak_src} bf16 dense (burst)",
                     "algorithmic_flops": afl, "attention_ms_per_prefill": sum(attn_ms),
                     "attention_share_of_prefill": sum(attn_ms) / statistics.mean(dev_ms)},
        "clocks": clk.summary(),
        "device_status": ops.read_status(dev),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cores = cpu_threads()
        run, sfl, sample = w.cpu_sample(np)
        _, n, el = time_cpu(run, sfl)
        line["cpu_baseline"] = {
            "value": el / n * w.projection() * 1e3, "unit": "ms (suffix-prefill attention only)",
            "cores": cores, "kind": "port", "cpu": cpu_model(),
            "sample": f"{n} x {sample}, {TORCH_PATH}, {el:.1f} s; projected x"
                      f"{w.projection()} (prompts x layers x KV heads)"}
    if rank == 0:
        print(json.dumps(line), flush=True)


def make_workload(name, small=False):
    if name == "reuse_prefill":
        return Dense(name, 4, 32, 8, 256, 896, 128, "bf16",
                     "prefix-reuse prefill op: B4 Hq32/Hkv8 D128 bf16, 7 cached chunks (896) + "
                     "256 new tokens")
    if name == "causal_op":
        return Dense(name, 2, 16, 16, 1024, 0, 64, "bf16", "single causal op: B2 H16 S1024 D64 bf16")
    if name == "varlen_d96":
        return Varlen(small)
    if name == "ttft_reuse":
        return TtftReuse()
    if name == "decode":
        return Decode()
    if name == "quantize_store":
        return QuantizeStore()
    if name == "cacheblend":
        return CacheBlendRepair()
    if name == "short_suffix":
        return ShortSuffix()
    if name == "long_causal":
        return LongCausal()
    return PagedLong(small)


# ─────────────────────────────────────────────────────────── helpers ──

class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

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
        for l in self.lines:
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


def time_cpu(run, fl, budget_s=10.0, max_iters=100000):
    """Repeat a bounded CPU sample for about ``budget_s`` seconds."""
    run()  # warm
    n, t0 = 0, time.perf_counter()
    while True:
        run()
        n += 1
        el = time.perf_counter() - t0
        if el > budget_s or n >= max_iters:
            return fl * n / el / 1e12, n, el


def cpu_threads():
    """All host threads for the CPU legs (torch intra-op and BLAS pools)."""
    n = os.cpu_count()
    try:
        from threadpoolctl import threadpool_limits
        threadpool_limits(limits=n)
    except Exception:  # pragma: no cover
        pass
    import torch
    torch.set_num_threads(n)
    return n


def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"



def run_reference(args):
    """--impl reference: the reference's CPU path on all host threads (its own torch
    calls for attention, ``oracle/sdpa_ref.py``; numpy restatements for the store and
    CacheBlend workloads)."""
    if int(os.environ.get("RANK", "0")) != 0:
        return
    import numpy as np
    w = make_workload(args.workload)
    cores = cpu_threads()
    run, fl, sample = w.cpu_sample(np)
    for _ in range(max(0, args.warmup)):
        run()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        run()
    el = time.perf_counter() - t0
    if isinstance(w, TtftReuse):
        val = el / args.steps * w.projection() * 1e3
        sample += f", projected x{w.projection()} (prompts x layers x KV heads)"
        line = {
            "impl": "reference", "metric": "TTFT at 75% prefix reuse", "value": val,
            "unit": "ms", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": val, "higher_is_better": False, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": args.workload, "desc": w.desc,
                       "sample": sample + " per step; attention of the suffix prefill only"},
            "cpu_baseline": {"value": val, "unit": "ms (suffix-prefill attention only)",
                             "cores": cores, "kind": "port", "cpu": cpu_model(),
                             "sample": sample + ", " + TORCH_PATH},
            "e2e": {"value": val, "unit": "ms", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }
        print(json.dumps(line), flush=True)
        return
    metric = getattr(w, "metric", "prefill attention TFLOP/s")
    munit, mscale = getattr(w, "unit", "TFLOP/s"), getattr(w, "unit_scale", 1e12)
    val = fl * args.steps / el / mscale
    line = {
        "impl": "reference", "metric": metric, "value": val,
        "unit": munit, "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": el / args.steps * 1e3, "higher_is_better": True, "scaling": w.scaling,
        "vs_baseline": None,
        "dtype": getattr(w, "dtype_name", "f32") if getattr(w, "cpu_path", TORCH_PATH) == TORCH_PATH
        else "f32",
        "data": "synthetic",
        "config": {"workload": args.workload, "desc": w.desc, "sample": sample + " per step"},
        "cpu_baseline": {"value": val, "unit": munit, "cores": cores, "kind": "port",
                         "cpu": cpu_model(),
                         "sample": sample + " per step, " + getattr(w, "cpu_path", TORCH_PATH)},
        "e2e": {"value": val, "unit": munit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def time_graph_steps(torch, dist, step, steps, warmup, dev, world, stream, prewarm_s=0.2):
    """K steps captured in one CUDA graph, replayed between two events on ``stream``
    after untimed replays and the W warm-up steps; returns the max over ranks of
    the elapsed milliseconds."""
    with torch.cuda.stream(stream):
        step(0)
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        gw, gt = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
        with torch.cuda.graph(gw, stream=stream):
            for i in range(warmup):
                step(i)
        with torch.cuda.graph(gt, stream=stream):
            for i in range(steps):
                step(i)
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        t_end = time.time() + prewarm_s
        while time.time() < t_end:
            gt.replay()
            gw.replay()
            stream.synchronize()
        gw.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        gt.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    del gw, gt
    return ms


def sharded_paged_line(torch, dist, rank, world, dev, steps=20, warmup=3):
    """The long paged int8 reuse prefill (32K-token prefix, 2048 new tokens, 64/8 heads)
    sharded over the job's ranks by KV head (each rank holds its heads' pool shard;
    no collective), beside the headline line: per-step time (max over ranks), the
    whole job's TFLOP/s, and the same prefill on one GPU (rank 0 alone, all 8 KV
    heads) for the speed-up and the strong-scaling efficiency."""
    from oracle.attention import attention_flops
    full = PagedLong()
    fl_all = attention_flops([full.Sq], [full.P + full.Sq], full.Hq, full.D)
    stream = torch.cuda.Stream(device=dev)
    w = PagedLong()
    ms_n = time_graph_steps(torch, dist, w.setup(torch, dev, rank, world), steps, warmup, dev,
                            world, stream) / steps
    del w
    torch.cuda.empty_cache()
    ms_1 = ms_n if world == 1 else None
    if world > 1:
        dist.barrier()
    if rank == 0 and world > 1:
        w1 = PagedLong()
        ms_1 = time_graph_steps(torch, dist, w1.setup(torch, dev, 0, 1), steps, warmup, dev, 1,
                                stream) / steps
        del w1
        torch.cuda.empty_cache()
    if world > 1:
        dist.barrier()
    out = {"workload": "paged_long (" + full.desc + ")",
           "parallelism": f"KV heads split over {world} ranks, no collective",
           "scaling": "strong", "n_gpus": world, "ms_per_step": ms_n,
           "value": fl_all / (ms_n / 1e3) / 1e12, "unit": "TFLOP/s",
           "prefill_tokens_per_s": full.Sq / (ms_n / 1e3)}
    if ms_1 is not None:
        out["one_gpu_ms_per_step"] = ms_1
        out["speedup_vs_one_gpu"] = ms_1 / ms_n
        out["strong_scaling_efficiency"] = ms_1 / ms_n / world
    return out


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
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
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=180))

    if args.workload in ("ttft_reuse", "paged_long_cp"):
        (run_ttft if args.workload == "ttft_reuse" else run_cp)(args, torch, dist, rank, world,
                                                                 local, dev)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return

    w = make_workload(args.workload, args.small)
    if args.workload == "varlen_d96" and args.varlen_split == "lpt" and world > 1:
        w.shard(rank, world)
    step = w.setup(torch, dev, rank, world)
    stream = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(stream):
        step(0)  # eager call on the capture stream: status word and workspaces before capture
    torch.cuda.synchronize()
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
    # Untimed replays until the GPU's clocks are at their loaded level (a few
    # hundred ms), then the W warm-up steps and the K timed steps.  The timed
    # graph is among the untimed replays: a graph's first replay also uploads
    # it to the device, which is not a step's work.
    with torch.cuda.stream(stream):
        t_end = time.time() + PREWARM_S
        while time.time() < t_end:
            gt.replay()
            gw.replay()
            stream.synchronize()
    with ClockSampler(local) as clk:
        with torch.cuda.stream(stream):
            gw.replay()
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
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
    fl = w.flops()                     # per rank per step
    metric = getattr(w, "metric", "prefill attention TFLOP/s")
    munit, mscale = getattr(w, "unit", "TFLOP/s"), getattr(w, "unit_scale", 1e12)
    work = w.work() if hasattr(w, "work") else fl
    per_launch_s = ms / 1e3 / args.steps
    value = world * work * args.steps / (ms / 1e3) / mscale
    units = w.tokens() * (world if w.scaling == "weak" else 1)
    tok_s = units * args.steps / (ms / 1e3)

    # ---- e2e through the public op with pinned host buffers ------------------
    # Steps whose calls share no device state run on two streams in turn, as a
    # serving loop would: step i+1's host-to-device copies overlap step i's
    # kernel and device-to-host copy.  Every step's copies stay in the region.
    e2e_step, h2d, d2h = w.e2e(torch, dev)
    overlap = getattr(w, "e2e_overlap", False)
    e2e_streams = [torch.cuda.Stream(device=dev) for _ in range(2)] if overlap else None

    def run_e2e(n):
        if not overlap:
            for _ in range(n):
                e2e_step()
            return
        cur = torch.cuda.current_stream(dev)
        for st in e2e_streams:
            st.wait_stream(cur)
        for i in range(n):
            with torch.cuda.stream(e2e_streams[i % 2]):
                e2e_step(i % 2)
        for st in e2e_streams:
            cur.wait_stream(st)

    run_e2e(4)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    run_e2e(args.e2e_steps)
    e1.record()
    torch.cuda.synchronize()
    ems = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ems], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ems = float(t.item())
    e2e_value = world * work * args.e2e_steps / (ems / 1e3) / mscale

    peak_tf, peak_bw, peak_src = measured_peaks()
    if w.bound == "tensor":
        achieved, peak, unit = fl / per_launch_s / 1e12, peak_tf, "TFLOP/s"
        psrc = f"{peak_src} bf16 dense (burst)"
    else:
        achieved, peak, unit = w.bytes() / per_launch_s / 1e9, peak_bw, "GB/s"
        psrc = f"{peak_src} HBM copy"
    cfg = {"workload": w.name + (" (small profiling case)" if args.small else ""),
           "desc": w.desc, **w.config(),
           "parallelism": ((f"requests placed longest-first over {world} ranks"
                            if hasattr(w, "all_flops") else f"KV heads split over {world} ranks")
                           if w.scaling == "strong"
                           else f"independent batches x{world}") if world > 1 else "single",
           "l2": w.sets_desc,
           "timing": f"CUDA graph of K launches between events, after {PREWARM_S} s of untimed replays"}
    line = {
        "metric": metric, "value": value, "unit": munit,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": w.scaling,
        "vs_baseline": None, "dtype": w.dtype_name, "data": "synthetic", "config": cfg,
        "tokens_per_s": tok_s,
        "e2e": {"value": e2e_value, "unit": munit, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": ems / args.e2e_steps,
                "streams": 2 if overlap else 1},
        "gpu_launches": args.steps * getattr(w, "launches_per_step", 1),
        "roofline": {"bound": w.bound, "achieved": achieved, "peak": peak, "unit": unit,
                     "frac": achieved / peak, "traffic": NCU_TRAFFIC_BYTES.get(w.name),
                     "peak_source": psrc, "algorithmic_flops": fl, "algorithmic_bytes": w.bytes()},
        "clocks": clk.summary(),
        "device_status": status,
    }
    if hasattr(w, "gpu_sdpa"):
        run = w.gpu_sdpa(torch, dev)
        for _ in range(3):
            run()
        torch.cuda.synchronize()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n_sdpa = 20
        s0.record()
        for _ in range(n_sdpa):
            run()
        s1.record()
        torch.cuda.synchronize()
        sms = s0.elapsed_time(s1) / n_sdpa
        line["gpu_reference_sdpa"] = {
            "value": fl / (sms / 1e3) / 1e12, "unit": "TFLOP/s", "ms_per_step": sms,
            "what": "the reference's torch_flash tier on this GPU: F.scaled_dot_product_attention "
                    "with repeat_interleave'd K/V and the bottom-right bool mask, same shapes"}
    if hasattr(w, "gpu_reference"):
        run, what = w.gpu_reference(torch, dev)
        for _ in range(3):
            run()
        torch.cuda.synchronize()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n_ref = 5
        s0.record()
        for _ in range(n_ref):
            run()
        s1.record()
        torch.cuda.synchronize()
        rms = s0.elapsed_time(s1) / n_ref
        line["gpu_reference_torch"] = {"value": work / (rms / 1e3) / mscale, "unit": munit,
                                       "ms_per_step": rms, "what": "the reference's steps on this GPU: " + what}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        import numpy as np
        cores = cpu_threads()
        run, sfl, sample = w.cpu_sample(np)
        v, n, el = time_cpu(run, sfl)
        v = v * 1e12 / mscale
        line["cpu_baseline"] = {"value": v, "unit": munit, "cores": cores, "kind": "port",
                                "cpu": cpu_model(),
                                "sample": f"{n} x {sample}, {getattr(w, 'cpu_path', TORCH_PATH)}, "
                                          f"{el:.1f} s"}
    del gw, gt
    if args.workload == "reuse_prefill" and not args.no_sharded and not args.small \
            and 8 % world == 0:
        try:   # every rank takes the same steps; a failure here must not cost the line
            line["sharded_paged_long"] = sharded_paged_line(torch, dist, rank, world, dev)
        except Exception as e:  # pragma: no cover - reported in the line
            line["sharded_paged_long"] = {"error": repr(e)[:300]}
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
