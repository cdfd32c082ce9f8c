"""Decode / verify kernel (gdn_recurrent_fwd and friends) against the CPU
oracle and the golden vectors of the reference's sequential_delta.

Tolerance: 1e-5 max-relative (max|a-b| / max|b|, cpp/src/tests.cpp:38-45) on
the fp32 output and state, the decode bound of the north star (the reference's
own test bound is 2e-5, cpp/src/tests.cpp:227).  bf16 outputs: 4e-3, i.e. one
bf16 rounding of the fp32 result."""
import numpy as np
import pytest
import torch

import delta_kernel
import gdn_b200 as G
import gdn_oracle as O
from conftest import golden

pytestmark = pytest.mark.gpu
TOL = 1e-5


def dev(x, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(x)).to("cuda", dtype)


def host(t):
    return t.float().cpu().numpy()


def oracle_step(inp, S0, l2norm_qk=False, collect=True):
    Hv = inp["v"].shape[2]
    q, k = inp["q"], inp["k"]
    if l2norm_qk:
        q = O.l2norm(q) * np.float32(128 ** -0.5)
        k = O.l2norm(k)
    al, bt = O.gates(inp["a"], inp["b"], inp["A_log"], inp["dt_bias"])
    return O.delta_reference(O.expand_heads(q, Hv), O.expand_heads(k, Hv), inp["v"], al, bt, S0,
                             collect=collect)


def device_inputs(inp):
    return (dev(inp["q"], torch.bfloat16), dev(inp["k"], torch.bfloat16), dev(inp["v"], torch.bfloat16),
            dev(inp["a"]), dev(inp["b"]), dev(inp["A_log"]), dev(inp["dt_bias"]))


def test_dropin_name_matches_reference_module():
    assert delta_kernel.available()
    assert delta_kernel.gated_delta_metal is delta_kernel.gated_delta_cuda


def test_golden_vectors_through_delta_kernel():
    d = golden("recurrent_d128.npz")
    for i in range(int(d["ncases"])):
        p = f"c{i}_"
        args = [dev(d[p + n]) for n in ("q", "k", "v", "alpha", "beta", "S0")]
        o, S, states = delta_kernel.gated_delta_cuda(*args, collect=True)
        assert O.rel_err(host(o), d[p + "o"]) < TOL, i
        assert O.rel_err(host(S), d[p + "S"]) < TOL, i
        assert len(states) == int(d[p + "shape"][1])
        if p + "states" in d:
            st = np.stack([host(s) for s in states], 2)
            assert O.rel_err(st, d[p + "states"]) < TOL, i
        o2, S2 = delta_kernel.gated_delta_cuda(*args[:5], None)      # S = None -> zeros
        ro, rS = O.delta_reference(*(d[p + n] for n in ("q", "k", "v", "alpha", "beta")))
        assert O.rel_err(host(o2), ro) < TOL and O.rel_err(host(S2), rS) < TOL


@pytest.mark.parametrize("B,T", [(1, 1), (2, 1), (3, 4), (1, 9), (2, 33)])
def test_raw_gates_bf16_gqa_with_checkpoints(B, T):
    rng = np.random.default_rng(100 + 7 * B + T)
    inp = O.synth_decode_inputs(rng, B, T)
    ro, rS, rst = oracle_step(inp, inp["S0"])
    S0 = dev(inp["S0"])
    ckpt = torch.empty((B, 48, T, 128, 128), device="cuda")
    o, S, _ = G.recurrent_fwd(*device_inputs(inp), state_in=S0, ckpt=ckpt,
                              state_out=torch.empty_like(S0))
    torch.cuda.synchronize()
    assert O.rel_err(host(o), ro) < TOL
    assert O.rel_err(host(S), rS) < TOL
    assert O.rel_err(host(ckpt), rst) < TOL
    assert torch.equal(ckpt[:, :, T - 1], S)


def test_in_place_zero_state_and_bf16_output():
    rng = np.random.default_rng(7)
    inp = O.synth_decode_inputs(rng, 2, 2)
    S = dev(inp["S0"])
    o, S_out, _ = G.recurrent_fwd(*device_inputs(inp), state_in=S, state_out=S, o_dtype=torch.bfloat16)
    ro, rS = oracle_step(inp, inp["S0"], collect=False)
    assert S_out.data_ptr() == S.data_ptr() and o.dtype == torch.bfloat16
    assert O.rel_err(host(S), rS) < TOL
    assert O.rel_err(host(o), ro) < 4e-3
    o, S2, _ = G.recurrent_fwd(*device_inputs(inp), state_in=None)
    ro, rS = oracle_step(inp, None, collect=False)
    assert O.rel_err(host(o), ro) < TOL and O.rel_err(host(S2), rS) < TOL


def test_t0_copies_state_and_b0_is_noop():
    rng = np.random.default_rng(8)
    inp = O.synth_decode_inputs(rng, 2, 1)
    S0 = dev(inp["S0"])
    q, k, v, a, b, A_log, dt_bias = device_inputs(inp)
    e = lambda x: x[:, :0].contiguous()  # noqa: E731
    _, S1, _ = G.recurrent_fwd(e(q), e(k), e(v), e(a), e(b), A_log, dt_bias, state_in=S0)
    assert torch.equal(S1, S0)
    z = lambda x: x[:0].contiguous()  # noqa: E731
    o, S2, _ = G.recurrent_fwd(z(q), z(k), z(v), z(a), z(b), A_log, dt_bias, state_in=z(S0))
    assert o.numel() == 0 and S2.numel() == 0


def test_in_kernel_l2norm():
    rng = np.random.default_rng(9)
    inp = O.synth_decode_inputs(rng, 2, 3)
    inp["q"] = O.bf16_round(rng.standard_normal(inp["q"].shape, dtype=np.float32))
    inp["k"] = O.bf16_round(rng.standard_normal(inp["k"].shape, dtype=np.float32))
    o, S, _ = G.recurrent_fwd(*device_inputs(inp), state_in=dev(inp["S0"]), l2norm=True)
    ro, rS = oracle_step(inp, inp["S0"], l2norm_qk=True, collect=False)
    assert O.rel_err(host(o), ro) < TOL and O.rel_err(host(S), rS) < TOL


def test_fp32_inputs_and_direct_gates_match_bf16_raw_path():
    rng = np.random.default_rng(10)
    inp = O.synth_decode_inputs(rng, 2, 2)
    al, bt = O.gates(inp["a"], inp["b"], inp["A_log"], inp["dt_bias"])
    q, k, v = (dev(inp[n]) for n in ("q", "k", "v"))
    o, S, _ = G.recurrent_fwd(q, k, v, dev(al), dev(bt), state_in=dev(inp["S0"]), gates_direct=True)
    ro, rS = oracle_step(inp, inp["S0"], collect=False)
    assert O.rel_err(host(o), ro) < TOL and O.rel_err(host(S), rS) < TOL


def test_verify_then_rollback_by_index():
    """config 2 semantics at small batch: a 4-token verify block writes
    checkpoints; a per-sequence accept count n selects the start state of the
    next decode step (DeltaCache::commit, cpp/src/model.cpp:439-457) with no copy."""
    B, T = 5, 4
    rng = np.random.default_rng(11)
    ver = O.synth_decode_inputs(rng, B, T)
    _, _, rst = oracle_step(ver, ver["S0"])
    S_prev = dev(ver["S0"])
    ckpt = torch.empty((B, 48, T, 128, 128), device="cuda")
    G.recurrent_fwd(*device_inputs(ver), state_in=S_prev, ckpt=ckpt)
    commit = np.array([0, 1, 2, 4, 5], np.int32)          # 5 is out of range
    nxt = O.synth_decode_inputs(rng, B, 1)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    o, S, _ = G.recurrent_fwd_from_ckpt(*device_inputs(nxt), S_prev, ckpt,
                                        torch.from_numpy(commit).cuda(), err_flag=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 1
    for bi, n in enumerate(commit):
        start = ver["S0"][bi:bi + 1] if n == 0 else (
            rst[bi:bi + 1, :, n - 1] if n <= T else np.zeros_like(ver["S0"][bi:bi + 1]))
        one = {kk: (vv[bi:bi + 1] if vv.ndim > 1 else vv) for kk, vv in nxt.items()}
        ro, rS = oracle_step(one, start, collect=False)
        assert O.rel_err(host(o[bi:bi + 1]), ro) < TOL, bi
        assert O.rel_err(host(S[bi:bi + 1]), rS) < TOL, bi


def test_config2_full_size_verify():
    """B=32, T=4, one layer, checkpoints after every position."""
    B, T = 32, 4
    rng = np.random.default_rng(12)
    inp = O.synth_decode_inputs(rng, B, T)
    ckpt = torch.empty((B, 48, T, 128, 128), device="cuda")
    o, _, _ = G.recurrent_fwd(*device_inputs(inp), state_in=dev(inp["S0"]), ckpt=ckpt)
    ro, rS, rst = oracle_step(inp, inp["S0"])
    assert O.rel_err(host(o), ro) < TOL
    assert O.rel_err(host(ckpt), rst) < TOL


def test_large_batch_linearity_and_spot_check():
    """Size-independent property at a config-1 batch: for fixed q, k, gates the
    step is linear in (S, v); plus an oracle spot check of a few heads."""
    B, T = 64, 1
    rng = np.random.default_rng(13)
    inp = O.synth_decode_inputs(rng, B, T)
    al, bt = O.gates(inp["a"], inp["b"], inp["A_log"], inp["dt_bias"])
    q, k = dev(inp["q"]), dev(inp["k"])
    v1, v2 = dev(inp["v"]), torch.randn(B, T, 48, 128, device="cuda")
    S1, S2 = dev(inp["S0"]), 0.05 * torch.randn(B, 48, 128, 128, device="cuda")
    run = lambda v, S: G.recurrent_fwd(q, k, v, dev(al), dev(bt), state_in=S, gates_direct=True)  # noqa: E731
    o1, T1, _ = run(v1, S1)
    o2, T2, _ = run(v2, S2)
    o3, T3, _ = run(v1 + v2, S1 + S2)
    assert O.rel_err(host(o1 + o2), host(o3)) < 1e-5
    assert O.rel_err(host(T1 + T2), host(T3)) < 1e-5
    for bi in (0, 17, 63):
        one = {kk: (vv[bi:bi + 1] if vv.ndim > 1 else vv) for kk, vv in inp.items()}
        ro, rS = oracle_step(one, inp["S0"][bi:bi + 1], collect=False)
        assert O.rel_err(host(o1[bi:bi + 1]), ro) < TOL and O.rel_err(host(T1[bi:bi + 1]), rS) < TOL


def test_rollback_in_place_and_zero_state_b24():
    """B = 24, T = 2 (eight rows per warp): rollback by index with an
    out-of-range entry, then an in-place step, then a zero start state; all
    against the oracle, and no kernel may have set the device error word."""
    B, T = 24, 2
    rng = np.random.default_rng(14)
    ver = O.synth_decode_inputs(rng, B, T)
    _, _, rst = oracle_step(ver, ver["S0"])
    S_prev = dev(ver["S0"])
    ckpt = torch.empty((B, 48, T, 128, 128), device="cuda")
    G.recurrent_fwd(*device_inputs(ver), state_in=S_prev, ckpt=ckpt)
    commit = (np.arange(B) % (T + 2)).astype(np.int32)      # includes T+1: out of range
    nxt = O.synth_decode_inputs(rng, B, 1)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    o, S, _ = G.recurrent_fwd_from_ckpt(*device_inputs(nxt), S_prev, ckpt,
                                        torch.from_numpy(commit).cuda(), err_flag=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 1
    starts = np.stack([ver["S0"][bi] if n == 0 else (rst[bi, :, n - 1] if n <= T else np.zeros_like(ver["S0"][bi]))
                       for bi, n in enumerate(commit)])
    ro, rS = oracle_step(nxt, starts, collect=False)
    assert O.rel_err(host(o), ro) < TOL and O.rel_err(host(S), rS) < TOL
    S_in = dev(starts)
    o2, S2, _ = G.recurrent_fwd(*device_inputs(nxt), state_in=S_in, state_out=S_in)
    assert S2.data_ptr() == S_in.data_ptr()
    assert O.rel_err(host(o2), ro) < TOL and O.rel_err(host(S_in), rS) < TOL
    o3, S3, _ = G.recurrent_fwd(*device_inputs(nxt), state_in=None)
    ro3, rS3 = oracle_step(nxt, None, collect=False)
    assert O.rel_err(host(o3), ro3) < TOL and O.rel_err(host(S3), rS3) < TOL
    assert G.take_device_error() == 0


def test_no_device_errors_recorded():
    assert G.take_device_error() == 0


def test_overlap_prev_flag_gives_the_same_bits_and_is_refused_elsewhere():
    """GDN_F_OVERLAP_PREV (launch as a programmatic dependent of the previous
    kernel) over a chain of three layers with their own states: the same o
    and states as ordinary launches; the from-checkpoint and pool entries,
    whose commit_n / slots may come from the previous kernel, refuse it."""
    rng = np.random.default_rng(44)
    B = 5
    layers = [O.synth_decode_inputs(rng, B, 1) for _ in range(3)]
    res = {}
    for ov in (False, True):
        outs = []
        for inp in layers:
            o, S, _ = G.recurrent_fwd(*device_inputs(inp), state_in=dev(inp["S0"]), overlap_prev=ov)
            outs.append((o, S))
        torch.cuda.synchronize()
        res[ov] = outs
    for (o1, S1), (o2, S2) in zip(res[False], res[True]):
        assert torch.equal(o1, o2) and torch.equal(S1, S2)
    inp = layers[0]
    ck = torch.zeros((B, 48, 1, 128, 128), device="cuda")
    n = torch.zeros(B, dtype=torch.int32, device="cuda")
    with pytest.raises(G.GdnError) as e:
        G.check(G.lib().gdn_recurrent_fwd_from_ckpt(*[G.ptr(t) for t in device_inputs(inp)], G.ptr(dev(inp["S0"])),
                                                    G.ptr(ck), G.ptr(n), 1, G.ptr(dev(inp["S0"])),
                                                    G.ptr(torch.empty((B, 1, 48, 128), device="cuda")), None, None,
                                                    B, 1, 16, 48, 128, 128, G.F_OVERLAP_PREV, None))
    assert e.value.code == G.GDN_ERR_FLAGS


def test_overlap_prev_two_layers_in_turn_from_a_graph_is_bit_identical():
    """Two layers used in turn (A, B, A, B, ... for 20 steps) at B = 1, each
    updating its own state in place, launched with GDN_F_OVERLAP_PREV and
    replayed from a CUDA graph: launch N + 2 reads the state that launch N
    wrote, so the o rows and final states must equal those of ordinary
    launches bit for bit."""
    rng = np.random.default_rng(45)
    steps = 20
    layers = [O.synth_decode_inputs(rng, 1, 1) for _ in range(2)]
    ins = [device_inputs(inp) for inp in layers]

    def run(overlap, graph):
        states = [dev(inp["S0"]) for inp in layers]
        outs = [torch.empty((1, 1, 48, 128), device="cuda") for _ in range(steps)]

        def body():
            for s in range(steps):
                j = s % 2
                G.recurrent_fwd(*ins[j], state_in=states[j], state_out=states[j], o=outs[s], overlap_prev=overlap)
        if graph:
            body()                                  # warm-up (module loading) outside the capture
            torch.cuda.synchronize()
            for j, inp in enumerate(layers):
                states[j].copy_(dev(inp["S0"]))
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                body()
            for j, inp in enumerate(layers):
                states[j].copy_(dev(inp["S0"]))
            torch.cuda.synchronize()
            g.replay()
        else:
            body()
        torch.cuda.synchronize()
        return outs, states

    ref_o, ref_S = run(False, False)
    got_o, got_S = run(True, True)
    for s in range(steps):
        assert torch.equal(ref_o[s], got_o[s]), s
    for j in range(2):
        assert torch.equal(ref_S[j], got_S[j]), j
    assert not torch.equal(ref_S[0], dev(layers[0]["S0"]))    # the chain really moved the states
    assert G.take_device_error() == 0
