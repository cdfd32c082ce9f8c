"""gdn_chunked_fwd_static -- the chunked prefill on the library's fixed device
scratch, for callers that cannot allocate device memory when they call (an
FFI binding with no device allocator, an engine that handed all free memory
to its pools at start-up) -- through the C ABI, against the caller-workspace
entry point gdn_chunked_fwd_ws on the same inputs.

Both entries run the same kernels on the same inputs, so the results must be
bit-identical (torch.equal).  Two calls in a row with different shapes (a
uniform batch with a start state and fp32 o, then packed sequences with bf16
o and zero start state), so the second call runs on scratch that still holds
the first call's records; the first is also checked against the CPU oracle
directly (2e-3 relative L2, the prefill bound).  A call longer than the 64 MiB
scratch holds runs in windows, again bit-identical to one pass on a caller
workspace; a batch whose smallest window does not fit is rejected with
GDN_ERR_SHAPE and leaves its outputs untouched.

Collected last (file name) so that it also runs after every other test in the
same process; it passes alone too.
"""
import ctypes

import numpy as np
import pytest
import torch

import gdn_b200 as G
import gdn_oracle as O

pytestmark = pytest.mark.gpu
PREFILL_TOL = 2e-3
D = 128


def P(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def make_inputs(seed, lens, Hk, Hv, packed, state):
    """q, k, v bf16 (tokens, heads, 128), gate inputs, optional start state."""
    rng = np.random.default_rng(seed)
    n = sum(lens)
    t = lambda shape: torch.from_numpy(O.bf16_round(rng.standard_normal(shape, dtype=np.float32)))  # noqa: E731
    f = lambda x: torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()  # noqa: E731
    X = dict(q=t((n, Hk, D)).cuda().bfloat16(), k=t((n, Hk, D)).cuda().bfloat16(),
             v=t((n, Hv, D)).cuda().bfloat16(),
             a=f(rng.standard_normal((n, Hv))), b=f(rng.standard_normal((n, Hv))),
             A_log=f(rng.uniform(0.0, np.log(16.0), Hv)), dt_bias=f(rng.uniform(0.0, 1.0, Hv)))
    X["S0"] = f(rng.standard_normal((len(lens), Hv, D, D)) * 0.05) if state else None
    X["cu"] = (torch.from_numpy(np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)).cuda()
               if packed else None)
    X["B"] = len(lens)
    X["T"] = n if packed else lens[0]
    X["Hk"], X["Hv"] = Hk, Hv
    return X


def call(fn, X, o, S, flags, *extra):
    """One chunked call through the C ABI; returns its status code."""
    return fn(P(X["q"]), P(X["k"]), P(X["v"]), Hk_stride(X), Hk_stride(X), X["Hv"] * D,
              P(X["a"]), P(X["b"]), P(X["A_log"]), P(X["dt_bias"]), P(X["S0"]), P(S), P(o), P(X["cu"]),
              X["B"], X["T"], X["Hk"], X["Hv"], D, D, flags, *extra, stream())


def Hk_stride(X):
    return X["Hk"] * D


def outputs(X, o_dtype):
    n = X["q"].shape[0]
    o = torch.full((n, X["Hv"], D), 7.0, dtype=o_dtype, device="cuda")
    S = torch.full((X["B"], X["Hv"], D, D), 7.0, dtype=torch.float32, device="cuda")
    return o, S


def reference(X, flags, o_dtype):
    """The same call through gdn_chunked_fwd_ws on a caller workspace."""
    L = G.lib()
    need = L.gdn_chunked_workspace_bytes(X["B"], X["T"], X["Hv"], 1 if X["cu"] is not None else 0)
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    o, S = outputs(X, o_dtype)
    rc = call(L.gdn_chunked_fwd_ws, X, o, S, flags, P(ws), ctypes.c_size_t(need))
    assert rc == G.GDN_OK, L.gdn_last_error().decode()
    return o, S


def rel_l2(a, b):
    return O.rel_l2(a.float().cpu().numpy(), b.float().cpu().numpy())


def oracle(X):
    """O.chunked_delta per sequence (uniform batch) from the host copies."""
    q = O.l2norm(X["q"].float().cpu().numpy().reshape(X["B"], X["T"], X["Hk"], D)) * np.float32(D ** -0.5)
    k = O.l2norm(X["k"].float().cpu().numpy().reshape(X["B"], X["T"], X["Hk"], D))
    v = X["v"].float().cpu().numpy().reshape(X["B"], X["T"], X["Hv"], D)
    a = X["a"].cpu().numpy().reshape(X["B"], X["T"], X["Hv"])
    b = X["b"].cpu().numpy().reshape(X["B"], X["T"], X["Hv"])
    al, bt = O.gates(a, b, X["A_log"].cpu().numpy(), X["dt_bias"].cpu().numpy())
    S0 = None if X["S0"] is None else X["S0"].cpu().numpy()
    return O.chunked_delta(O.expand_heads(q, X["Hv"]), O.expand_heads(k, X["Hv"]), v, al, bt, S0)


def test_static_scratch_matches_workspace_entry_on_two_calls_in_a_row():
    L = G.lib()
    X1 = make_inputs(70, [200, 200], Hk=2, Hv=6, packed=False, state=True)
    X2 = make_inputs(71, [100, 0, 257, 3], Hk=1, Hv=3, packed=True, state=False)
    f1 = G.F_QK_L2NORM
    f2 = G.F_QK_L2NORM | G.F_O_BF16
    r1 = reference(X1, f1, torch.float32)
    r2 = reference(X2, f2, torch.bfloat16)
    o1, S1 = outputs(X1, torch.float32)
    o2, S2 = outputs(X2, torch.bfloat16)
    rc1 = call(L.gdn_chunked_fwd_static, X1, o1, S1, f1)
    rc2 = call(L.gdn_chunked_fwd_static, X2, o2, S2, f2)
    assert rc1 == G.GDN_OK and rc2 == G.GDN_OK, L.gdn_last_error().decode()
    torch.cuda.synchronize()
    for (o, S), (ro, rS) in (((o1, S1), r1), ((o2, S2), r2)):
        assert torch.equal(o, ro) and torch.equal(S, rS)
    oo, oS = oracle(X1)
    assert rel_l2(o1.view(2, 200, 6, D), torch.from_numpy(oo)) < PREFILL_TOL
    assert rel_l2(S1, torch.from_numpy(oS)) < PREFILL_TOL
    assert G.take_device_error() == 0


def test_static_scratch_runs_a_longer_call_in_windows():
    """1,024 tokens x 48 value heads need 67 MiB of records in one pass; the
    static entry runs them in windows of its 64 MiB, bit-identical to one pass
    on a caller workspace (with and without state_out)."""
    L = G.lib()
    X = make_inputs(73, [1024], Hk=16, Hv=48, packed=False, state=True)
    need = L.gdn_chunked_workspace_bytes(1, 1024, 48, 0)
    assert need > 64 << 20
    ro, rS = reference(X, G.F_QK_L2NORM, torch.float32)
    o, S = outputs(X, torch.float32)
    rc = call(L.gdn_chunked_fwd_static, X, o, S, G.F_QK_L2NORM)
    assert rc == G.GDN_OK, L.gdn_last_error().decode()
    o2, _ = outputs(X, torch.float32)
    rc = call(L.gdn_chunked_fwd_static, X, o2, None, G.F_QK_L2NORM)
    assert rc == G.GDN_OK, L.gdn_last_error().decode()
    torch.cuda.synchronize()
    assert torch.equal(o, ro) and torch.equal(S, rS) and torch.equal(o2, ro)
    assert G.take_device_error() == 0


def test_static_scratch_rejects_a_batch_whose_smallest_window_does_not_fit():
    """16 sequences x 48 value heads: one record each (768 records of 89 KiB)
    already exceed the 64 MiB scratch: GDN_ERR_SHAPE, outputs untouched.  The
    buffers have the call's full size, so nothing could be out of bounds
    either way."""
    L = G.lib()
    X = make_inputs(72, [64] * 16, Hk=16, Hv=48, packed=False, state=False)
    assert G.chunked_workspace_min_bytes(16, 48, True) > 64 << 20
    o, S = outputs(X, torch.float32)
    rc = call(L.gdn_chunked_fwd_static, X, o, S, G.F_QK_L2NORM)
    assert rc == G.GDN_ERR_SHAPE
    assert "static scratch" in L.gdn_last_error().decode()
    torch.cuda.synchronize()
    assert bool((o == 7.0).all()) and bool((S == 7.0).all())
