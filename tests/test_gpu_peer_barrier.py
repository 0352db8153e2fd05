"""GPU: the bounded cross-GPU barrier (``kvb_peer_barrier``) on one device.

Two ranks' signal arrays both live on this GPU and only rank 0's barrier
kernel runs; rank 1's arrival is a word the test writes (or never writes).
So one kernel waits at a time and nothing else is waited on:

* rank 1 already arrived: the barrier returns at once, with rank 0's arrival
  stored in rank 1's array;
* rank 1 never arrives: the wait runs out after its short limit, the kernel
  sets ``KVB_STATUS_PEER_WAIT`` and returns, and the context stays usable (a
  prefill launched afterwards is correct);
* a word left over from an earlier epoch does not satisfy a later barrier.
"""

import time

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _gpu():
    if not torch.cuda.is_available() or torch.cuda.get_device_capability()[0] != 10:
        pytest.skip("needs an sm_100 (B200) device")
    from kvboost_b200 import ops
    ops.read_status(torch.device("cuda"))
    yield


def _arrays():
    a = torch.zeros(2, dtype=torch.int32, device="cuda")   # rank 0's words
    b = torch.zeros(2, dtype=torch.int32, device="cuda")   # rank 1's words
    return a, b


def test_barrier_passes_when_the_peer_has_arrived():
    from kvboost_b200 import ops
    from kvboost_b200.context_parallel import peer_barrier
    a, b = _arrays()
    a[1] = 1                                   # rank 1 arrived at epoch 1
    peer_barrier([a.data_ptr(), b.data_ptr()], 0, 1, torch.device("cuda"),
                 timeout_ns=2_000_000_000)
    torch.cuda.synchronize()
    assert ops.read_status(torch.device("cuda")) == 0
    assert a.tolist() == [1, 1] and b.tolist() == [1, 0]


def test_barrier_gives_up_and_reports_a_missing_peer():
    from kvboost_b200 import _lib, ops
    from kvboost_b200.context_parallel import peer_barrier
    from kvboost_b200.ops import prefill_attention
    a, b = _arrays()
    t0 = time.time()
    peer_barrier([a.data_ptr(), b.data_ptr()], 0, 1, torch.device("cuda"), timeout_ns=20_000_000)
    torch.cuda.synchronize()
    assert time.time() - t0 < 10
    assert ops.read_status(torch.device("cuda")) & _lib.KVB_STATUS_PEER_WAIT
    # the context is still usable
    g = torch.Generator().manual_seed(0)
    q, k, v = (torch.randn(1, 4, 128, 64, generator=g).to(torch.bfloat16).cuda() for _ in range(3))
    o, _ = prefill_attention(q, k, v, 0.125, True, return_lse=False)
    ref = torch.nn.functional.scaled_dot_product_attention(q.float(), k.float(), v.float(),
                                                           is_causal=True, scale=0.125)
    assert (o.float() - ref).abs().max().item() <= 2e-2
    assert ops.read_status(torch.device("cuda")) == 0


def test_stale_epoch_does_not_satisfy_a_later_barrier():
    from kvboost_b200 import _lib, ops
    from kvboost_b200.context_parallel import peer_barrier
    a, b = _arrays()
    a[1] = 1                                   # rank 1 arrived at epoch 1, not 2
    peer_barrier([a.data_ptr(), b.data_ptr()], 0, 2, torch.device("cuda"), timeout_ns=20_000_000)
    torch.cuda.synchronize()
    assert ops.read_status(torch.device("cuda")) & _lib.KVB_STATUS_PEER_WAIT
    assert b.tolist() == [2, 0]
