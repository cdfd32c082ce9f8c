"""The bounded device waits run out and report it, on one GPU, with nothing
left hung: a wait that nothing will satisfy, given a short limit, must end
within that limit, set its status, set the library's device error word
(gdn_take_device_error) and leave the context usable.

* gdn_gather_wait_timeout: the stream-ordered wait of the fused NVLink head
  gather (the acquire poll on the per-rank counters), with a counter that no
  rank ever increments and a 20 ms limit.
* gdn_tc05_selftest mode 128: the tensor-core self-test waits on an MMA
  mbarrier to which no MMA commits, with a poll budget of 4096 (the same
  bounded mbarrier wait that every tcgen05 kernel of the library uses).
"""
import ctypes
import time

import pytest
import torch

import gdn_b200 as G

pytestmark = pytest.mark.gpu


def test_gather_wait_runs_out_and_reports():
    L = G.lib()
    assert G.take_device_error() == 0
    flags = torch.zeros(8, dtype=torch.int32, device="cuda")    # one counter per rank, never signalled
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    st = G.stream_ptr(flags.device)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    G.check(L.gdn_gather_wait_timeout(G.ptr(flags), 2, 1, 20, G.ptr(err), st))
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    assert int(err.item()) == 1
    assert dt < 2.0, dt                       # the 20 ms limit, not the 4 s default
    assert G.take_device_error() == 1
    assert G.take_device_error() == 0         # taken and cleared
    # a counter that has been reached: no error, and the context still works
    flags.fill_(3)
    err.zero_()
    G.check(L.gdn_gather_wait_timeout(G.ptr(flags), 2, 3, 20, G.ptr(err), st))
    torch.cuda.synchronize()
    assert int(err.item()) == 0 and G.take_device_error() == 0
    # the limit is checked on the host
    with pytest.raises(G.GdnError) as e:
        G.check(L.gdn_gather_wait_timeout(G.ptr(flags), 2, 3, 0, G.ptr(err), st))
    assert e.value.code == G.GDN_ERR_RANGE


def test_mma_barrier_wait_runs_out_and_reports():
    L = G.lib()
    assert G.take_device_error() == 0
    N = K = 64
    A = torch.randn(128, K, device="cuda")
    B = torch.randn(N, K, device="cuda")
    D = torch.full((128, N), 5.0, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    st = G.stream_ptr(A.device)
    G.check(L.gdn_tc05_selftest(G.ptr(A), G.ptr(B), G.ptr(D), N, K, 128, G.ptr(status), st))
    torch.cuda.synchronize()
    assert int(status.item()) == 1
    assert bool((D == 5.0).all())             # nothing written after the timeout
    assert G.take_device_error() == 1
    # the same kernel with an MMA afterwards: correct, no error (context intact, TMEM freed)
    status.zero_()
    G.check(L.gdn_tc05_selftest(G.ptr(A), G.ptr(B), G.ptr(D), N, K, 1, G.ptr(status), st))
    torch.cuda.synchronize()
    ref = A.bfloat16().float() @ B.bfloat16().float().t()
    assert int(status.item()) == 0
    assert torch.allclose(D, ref, rtol=1e-4, atol=1e-3)
    assert G.take_device_error() == 0
    with pytest.raises(G.GdnError) as e:
        G.check(L.gdn_tc05_selftest(G.ptr(A), G.ptr(B), G.ptr(D), N, K, 128 | 1, G.ptr(status), st))
    assert e.value.code == G.GDN_ERR_FLAGS
