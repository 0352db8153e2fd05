"""The one-line drop-in into the unmodified KVBoost package.

``kvboost_b200.flash_attn_ext.inject_into_reference()`` registers the sm_100a op
as ``kvboost._flash_attn_cuda``; the reference's import-time probe
(``src/kvboost/flash_attn_ext.py:37-39``) then reports tier ``"kvboost_cuda"``
and its dispatcher ``_kvboost_flash_attn`` calls ``flash_attn_fwd`` for CUDA
16-bit inputs without a mask (``:80-84``), while CPU tensors keep its vanilla
SDPA path (``:97-103``).

The reference package is found through ``KVBOOST_REF_SRC`` (its ``src``
directory) or the stock install under ``baseline/_ref``; without either the
tests skip.  Each check runs in a child process so the reference's ``kvboost``
never enters this test session's modules.
"""

import os
import subprocess
import sys
import textwrap

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _reference_path():
    for p in (os.environ.get("KVBOOST_REF_SRC"), os.path.join(ROOT, "baseline", "_ref")):
        if p and os.path.isfile(os.path.join(p, "kvboost", "flash_attn_ext.py")):
            return p
    pytest.skip("the reference package is not available (KVBOOST_REF_SRC or baseline/_ref)")


def _run(body: str):
    ref = _reference_path()
    code = textwrap.dedent(f"""
        import sys
        sys.path.insert(0, {ROOT!r})
        from kvboost_b200.flash_attn_ext import inject_into_reference
        inject_into_reference()
        sys.path.insert(0, {ref!r})
        import kvboost
        import kvboost.flash_attn_ext as fae
        import kvboost_b200._flash_attn_cuda as ours
        assert kvboost.get_flash_attn_tier() == "kvboost_cuda", kvboost.get_flash_attn_tier()
        assert fae._flash_attn_cuda is ours
    """) + textwrap.dedent(body)
    res = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=600,
                         cwd=ROOT)
    assert res.returncode == 0, res.stdout + res.stderr
    return res.stdout


def test_reference_reports_kvboost_cuda_and_keeps_cpu_path():
    out = _run("""
        import math, torch
        from oracle import sdpa_ref
        g = torch.Generator().manual_seed(0)
        q, k, v = (torch.randn(1, 4, 64, 64, generator=g).bfloat16() for _ in range(3))
        o = fae._kvboost_flash_attn(q, k, v, 0.125, True)
        assert torch.equal(o, sdpa_ref.kvboost_flash_attn_cpu(q, k, v, 0.125, True))
        print("ok")
    """)
    assert out.strip().endswith("ok")


@pytest.mark.gpu
def test_reference_dispatcher_runs_the_sm100_op():
    import torch
    if not torch.cuda.is_available() or torch.cuda.get_device_capability()[0] != 10:
        pytest.skip("needs an sm_100 (B200) device")
    out = _run("""
        import math, numpy as np, torch
        from oracle import attention as oattn
        calls = []
        fwd = ours.flash_attn_fwd
        def counting(*a, **k):
            calls.append(a[0].shape)
            return fwd(*a, **k)
        ours.flash_attn_fwd = counting
        g = torch.Generator().manual_seed(1)
        # the single causal op: B2 H16 S1024 D64 bf16, no mask -> the CUDA tier
        q, k, v = (torch.randn(2, 16, 1024, 64, generator=g).bfloat16() for _ in range(3))
        o = fae._kvboost_flash_attn(q.cuda(), k.cuda(), v.cuda(), 0.125, True)
        torch.cuda.synchronize()
        assert len(calls) == 1, calls
        ref, _ = oattn.attention(q.float().numpy(), k.float().numpy(), v.float().numpy(), 0.125,
                                 True, compute_dtype=np.float32)
        err = float(np.abs(o.float().cpu().numpy() - ref).max())
        assert err <= 2e-2, err
        # with a mask the reference keeps its torch tier: no call reaches the op
        m = torch.ones(1024, 1024, dtype=torch.bool, device="cuda").tril()
        fae._kvboost_flash_attn(q.cuda(), k.cuda(), v.cuda(), 0.125, True, attn_mask=m)
        assert len(calls) == 1
        print("ok", err)
    """)
    assert "ok" in out
