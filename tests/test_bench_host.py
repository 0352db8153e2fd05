"""Host: the bench's workload definitions and its reference arm (no GPU).

Algorithmic FLOPs and bytes are the roofline's numerators, so they are checked
against the counts written out for each workload: FLOPs = 4 * D * Hq per visible
(query, key) pair under bottom-right causality, bytes = Q + O + K + V once.
"""

import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


def _pairs(sq, skv):
    return sq * (skv - sq) + sq * (sq + 1) // 2


@pytest.mark.parametrize("name,B,Hq,Hkv,Sq,Skv,D", [
    ("reuse_prefill", 4, 32, 8, 256, 1152, 128),
    ("causal_op", 2, 16, 16, 1024, 1024, 64),
    ("long_causal", 1, 32, 8, 16384, 16384, 128),
    ("short_suffix", 8, 16, 2, 16, 32784, 128),
    ("decode", 8, 16, 2, 1, 4096, 128),
])
def test_dense_workload_counts(name, B, Hq, Hkv, Sq, Skv, D):
    w = bench.make_workload(name)
    assert w.flops() == 4 * D * Hq * B * _pairs(Sq, Skv)
    assert w.bytes() == B * 2 * (2 * Hq * Sq * D + 2 * Hkv * Skv * D)
    cfg = w.config()
    assert (cfg["batch"], cfg["q_heads"], cfg["kv_heads"], cfg["q_len"], cfg["kv_len"],
            cfg["head_dim"]) == (B, Hq, Hkv, Sq, Skv, D)


def test_reuse_prefill_headline_counts():
    w = bench.make_workload("reuse_prefill")
    assert w.flops() == 17188257792          # 17.19 GFLOP
    assert w.bytes() == 35651584             # 35.65 MB
    assert w.bound == "tensor" and w.scaling == "weak"


def test_varlen_lengths_are_seeded_and_bounded():
    a, b = bench.make_workload("varlen_d96"), bench.make_workload("varlen_d96")
    assert a.sq == b.sq and a.pre == b.pre and len(a.sq) == 64
    assert all(16 <= s <= 512 for s in a.sq)
    assert all(p % 128 == 0 and 0 <= p <= 8192 for p in a.pre)


def test_launch_counts_claimed():
    # kernels per step that the bench line claims in gpu_launches
    assert getattr(bench.make_workload("reuse_prefill"), "launches_per_step", 1) == 1
    assert bench.make_workload("decode").launches_per_step == 2
    assert bench.make_workload("short_suffix").launches_per_step == 2
    assert bench.make_workload("paged_long").launches_per_step == 2


def test_cpu_samples_are_bounded():
    import numpy as np
    for name in ("reuse_prefill", "long_causal", "short_suffix"):
        run, fl, sample = bench.make_workload(name).cpu_sample(np)
        assert fl > 0 and sample
        # torch SDPA runs at >= 0.3 TFLOP/s on 8 host cores: well under a second
        assert fl < 1e11


def test_reference_arm_prints_one_line():
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                          "--workload", "causal_op", "--steps", "1", "--warmup", "0"],
                         capture_output=True, text=True, timeout=300, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["value"] > 0 and d["unit"] == "TFLOP/s"
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
