"""On-device acceptance of a speculative-verify block (gdn_spec_verify)
against the CPU oracle (oracle/gdn_oracle.py:spec_verify, the rejection test
of python/speculative.py:170-190), the reference selftest's marginal property
through the kernel, and the whole verify -> accept -> rollback -> decode chain
on the device with no host round trip.

Accept lengths and commit indices: exact.  Drawn tokens: exact, except where
the uniform lands within 1e-5 (relative) of a CDF step, where fp32 and fp64
prefix sums may legitimately disagree; those cases must still be a neighbour.
Decode after the rollback: 1e-5 max-relative, the decode bound."""
import numpy as np
import pytest
import torch

import gdn_b200 as G
import gdn_oracle as O

pytestmark = pytest.mark.gpu


def dev(x, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(x)).to("cuda", dtype)


def softmax(x, axis=-1):
    e = np.exp(x - x.max(axis=axis, keepdims=True))
    return (e / e.sum(axis=axis, keepdims=True)).astype(np.float32)


def spec_case(rng, B, k, V, temp=1.0):
    p = softmax(rng.standard_normal((B, k + 1, V)).astype(np.float32) * 3 / temp)
    q = softmax((rng.standard_normal((B, k, V)) * 3 / temp + 0.5 * np.log(p[:, :k] + 1e-9)).astype(np.float32))
    draft = np.stack([[rng.choice(V, p=q[b, i].astype(np.float64) / q[b, i].sum(dtype=np.float64))
                       for i in range(k)] for b in range(B)]).astype(np.int32)
    ua = rng.random((B, k), dtype=np.float32)
    us = rng.random(B, dtype=np.float32)
    return p, q, draft, ua, us


def near_cdf_step(p, q, j, k, u):
    r = np.asarray(p[k], np.float64) if j == k else np.maximum(np.asarray(p[j], np.float64) - q[j], 0)
    if j < k and not r.sum() > 1e-12:
        r = np.asarray(p[j], np.float64)
    cdf = np.cumsum(r)
    t = u * cdf[-1]
    return np.min(np.abs(cdf - t)) <= 1e-5 * cdf[-1]


@pytest.mark.parametrize("B,k,V", [(64, 1, 6), (64, 3, 1000), (32, 4, 151936), (5, 32, 257)])
def test_spec_verify_matches_oracle(B, k, V):
    rng = np.random.default_rng(B * 131 + k * 7 + V)
    p, q, draft, ua, us = spec_case(rng, B, k, V)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    acc, commit, tok = G.spec_verify(dev(p), dev(q), dev(draft, torch.int32), dev(ua), dev(us), err_flag=err)
    acc, commit, tok = acc.cpu().numpy(), commit.cpu().numpy(), tok.cpu().numpy()
    assert int(err.item()) == 0
    for b in range(B):
        j, n, v = O.spec_verify(p[b], q[b], draft[b], ua[b], us[b])
        assert (acc[b], commit[b]) == (j, n), b
        if tok[b] != v:
            assert near_cdf_step(p[b], q[b], j, k, float(us[b])) and abs(int(tok[b]) - v) <= 1, (b, tok[b], v)


@pytest.mark.parametrize("V", [65536 + 333, 151936])
def test_cluster_path_ragged_and_empty_residual(V):
    """Vocabularies of 64K entries and more take the 8-CTA cluster kernel.
    V = 65869 leaves the last CTA of the cluster 2 of 65 blocks.  Half the
    sequences have p = 0.5 q on the rejected row (an empty residual, so the
    cluster re-sums p itself); every draft there is rejected by u > 0.5."""
    B, k = 6, 2
    rng = np.random.default_rng(V)
    p, q, draft, ua, us = spec_case(rng, B, k, V)
    for b in range(0, B, 2):
        p[b, 0] = 0.5 * q[b, 0]
        ua[b, 0] = 0.75
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    acc, commit, tok = G.spec_verify(dev(p), dev(q), dev(draft, torch.int32), dev(ua), dev(us), err_flag=err)
    acc, commit, tok = acc.cpu().numpy(), commit.cpu().numpy(), tok.cpu().numpy()
    assert int(err.item()) == 0
    for b in range(B):
        j, n, v = O.spec_verify(p[b], q[b], draft[b], ua[b], us[b])
        if b % 2 == 0:
            assert j == 0
        assert (acc[b], commit[b]) == (j, n), b
        if tok[b] != v:
            assert near_cdf_step(p[b], q[b], j, k, float(us[b])) and abs(int(tok[b]) - v) <= 1, (b, tok[b], v)


def test_out_of_range_draft_is_rejected_and_flagged():
    rng = np.random.default_rng(3)
    p, q, draft, ua, us = spec_case(rng, 4, 3, 50)
    ua[:] = 0.0                                  # every in-range draft would be accepted
    draft[2, 1] = 50
    draft[3, 0] = -1
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    acc, commit, _ = G.spec_verify(dev(p), dev(q), dev(draft, torch.int32), dev(ua), dev(us), err_flag=err)
    assert acc.cpu().tolist() == [3, 3, 1, 0]
    assert commit.cpu().tolist() == [4, 4, 2, 1]
    assert int(err.item()) == 1


def test_marginal_of_accept_or_resample_is_the_target():
    """python/speculative.py:256-283 through the kernel: for a 6-way (p, q),
    every draft d weighted by q[d], and a midpoint grid of the acceptance and
    sampling uniforms, the distribution of the emitted token is p."""
    rng = np.random.default_rng(7)
    V, N = 6, 64
    grid = (np.arange(N, dtype=np.float32) + 0.5) / N
    for _ in range(3):
        p1 = softmax(rng.standard_normal(V).astype(np.float32) * 2)
        q1 = softmax(rng.standard_normal(V).astype(np.float32) * 2)
        d = np.repeat(np.arange(V), N * N).astype(np.int32)
        ua = np.tile(np.repeat(grid, N), V)
        us = np.tile(grid, V * N)
        B = d.size
        P = np.broadcast_to(np.stack([p1, p1]), (B, 2, V)).copy()      # p_1 (all accepted) = p too
        Q = np.broadcast_to(q1[None, None], (B, 1, V)).copy()
        acc, _, tok = G.spec_verify(dev(P), dev(Q), dev(d[:, None], torch.int32), dev(ua[:, None]), dev(us))
        tok = tok.cpu().numpy()
        acc = acc.cpu().numpy()
        # emitted first token: the draft when accepted, else the resampled token
        first = np.where(acc == 1, d, tok)
        w = q1[d].astype(np.float64) / (N * N)
        marg = np.bincount(first, weights=w, minlength=V)
        assert np.max(np.abs(marg - p1)) < 2.0 / N


def test_verify_accept_rollback_chain_on_device():
    """config 2 shape: a 4-token verify block with checkpoints, the acceptance
    test on the device, then the next decode step started from checkpoint
    commit_n - 1 (or the previous state) and the conv window rolled back --
    all stream-ordered, no host read in between -- against the oracle's
    DeltaCache.commit (cpp/src/model.cpp:439-457)."""
    B, T, V = 8, 4, 4096
    k = T - 1
    rng = np.random.default_rng(21)
    ver = O.synth_decode_inputs(rng, B, T)
    p, q, draft, ua, us = spec_case(rng, B, k, V, temp=0.7)
    S_prev = dev(ver["S0"])
    ckpt = torch.empty((B, 48, T, 128, 128), device="cuda")
    qv, kv_, vv, a, b, A_log, dtb = (dev(ver["q"], torch.bfloat16), dev(ver["k"], torch.bfloat16),
                                     dev(ver["v"], torch.bfloat16), dev(ver["a"]), dev(ver["b"]),
                                     dev(ver["A_log"]), dev(ver["dt_bias"]))
    G.recurrent_fwd(qv, kv_, vv, a, b, A_log, dtb, state_in=S_prev, ckpt=ckpt)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    acc, commit, tok = G.spec_verify(dev(p), dev(q), dev(draft, torch.int32), dev(ua), dev(us), err_flag=err)
    # conv window: a (B, T, C) block after a (B, 3, C) window, rolled back by commit_n
    C = 256
    xw = O.bf16_round(rng.standard_normal((B, 3, C), dtype=np.float32))
    xb = O.bf16_round(rng.standard_normal((B, T, C), dtype=np.float32))
    conv_out = G.conv_commit(dev(xw, torch.bfloat16), dev(xb, torch.bfloat16), commit, err_flag=err)
    nxt = O.synth_decode_inputs(rng, B, 1)
    o, S, _ = G.recurrent_fwd_from_ckpt(dev(nxt["q"], torch.bfloat16), dev(nxt["k"], torch.bfloat16),
                                        dev(nxt["v"], torch.bfloat16), dev(nxt["a"]), dev(nxt["b"]),
                                        dev(nxt["A_log"]), dev(nxt["dt_bias"]), S_prev, ckpt, commit, err_flag=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    al, bt = O.gates(ver["a"], ver["b"], ver["A_log"], ver["dt_bias"])
    _, _, rst = O.delta_reference(O.expand_heads(ver["q"], 48), O.expand_heads(ver["k"], 48), ver["v"], al, bt,
                                  ver["S0"], collect=True)
    commit_h = commit.cpu().numpy()
    conv_h = conv_out.float().cpu().numpy()
    for bi in range(B):
        j, n, _ = O.spec_verify(p[bi], q[bi], draft[bi], ua[bi], us[bi])
        assert commit_h[bi] == n
        start = ver["S0"][bi:bi + 1] if n == 0 else rst[bi:bi + 1, :, n - 1]
        one = {kk: (vv_[bi:bi + 1] if vv_.ndim > 1 else vv_) for kk, vv_ in nxt.items()}
        ga, gb = O.gates(one["a"], one["b"], one["A_log"], one["dt_bias"])
        ro, rS = O.delta_reference(O.expand_heads(one["q"], 48), O.expand_heads(one["k"], 48), one["v"], ga, gb,
                                   start, collect=False)
        assert O.rel_err(o[bi:bi + 1].float().cpu().numpy(), ro) < 1e-5, bi
        assert O.rel_err(S[bi:bi + 1].float().cpu().numpy(), rS) < 1e-5, bi
        window = np.concatenate([xw[bi], xb[bi]])[n:n + 3]
        assert np.array_equal(conv_h[bi], window), bi
