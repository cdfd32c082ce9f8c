"""Generate the golden vectors in this folder by running the REFERENCE's own
Python GDN code (python/qwen35.py from ggluo/Qwen3.8-27B-MLX) over a numpy
stand-in for MLX (``mlx_stub/``; MLX itself is not installable here).

Run once, in a container where the reference checkout exists:

    python tests/golden/gen_golden.py --ref /path/to/reference/python

The reference path can come from the GDN_REFERENCE_PY environment variable
instead; one of the two is required.  Outputs (``*.npz``) are committed; tests only read them and never
touch the reference tree.

What is pinned (all functions are the reference's own, unmodified):

* ``recurrent_*.npz``   ``sequential_delta`` (python/qwen35.py:450-475) with
  ``collect=True``, on the seeded cases and distributions of
  cpp/src/tests.cpp:206-218 (q = l2norm(N)*Dk^-1/2, k = l2norm(N), v = N,
  alpha ~ U(0.85,1), beta ~ U(0,1), S0 = 0.1*N).
* ``chunked_*.npz``     ``chunked_delta`` (python/qwen35.py:365-431) next to
  ``sequential_delta`` over the length sweep L in {1,5,16,63,64,65,130,200}
  that BUILD_LOG.md:314 reports, with test-style gates and with model-style
  gates (alpha = exp(-exp(A_log)*softplus(a+dt_bias)), A_log ~ U(0, ln 16),
  which underflows below the 1e-6 clip).
* ``spec_residual.npz`` ``residual`` (python/speculative.py:100-106) of the
  speculative acceptance step on seeded softmax pairs.
* ``block_*.npz``       ``GatedDeltaNet.__call__`` (python/qwen35.py:572-639)
  with the input/output projections replaced by fixed tensors, driving a
  ``DeltaCache`` (python/qwen35.py:291-328) through prefill (chunked path),
  a decode step, a recorded 4-token verify block, ``commit(2)`` and another
  decode step, in float32 and in bf16 activations.
"""
from __future__ import annotations

import argparse
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def load_reference(ref_py: str):
    sys.path.insert(0, os.path.join(HERE, "mlx_stub"))
    vision = types.ModuleType("vision")       # vision tower is not on the GDN path
    vision.VisionConfig = object
    sys.modules["vision"] = vision
    sys.path.insert(0, ref_py)
    import mlx.core as mx  # noqa: E402  (the stand-in)
    import qwen35  # noqa: E402  (the reference)
    return mx, qwen35


def l2n(x):
    return x / np.sqrt(np.sum(x * x, axis=-1, keepdims=True) + np.float32(1e-6))


def test_inputs(rng, B, L, H, D):
    """cpp/src/tests.cpp:209-218 distributions, generated with numpy's PCG64."""
    q = (l2n(rng.standard_normal((B, L, H, D), dtype=np.float32)) * np.float32(D ** -0.5)).astype(np.float32)
    k = l2n(rng.standard_normal((B, L, H, D), dtype=np.float32)).astype(np.float32)
    v = rng.standard_normal((B, L, H, D), dtype=np.float32)
    al = rng.uniform(0.85, 1.0, (B, L, H)).astype(np.float32)
    bt = rng.uniform(0.0, 1.0, (B, L, H)).astype(np.float32)
    S0 = (rng.standard_normal((B, H, D, D), dtype=np.float32) * np.float32(0.1)).astype(np.float32)
    return q, k, v, al, bt, S0


def model_gates(rng, B, L, H):
    """BASELINE config distributions: a,b ~ N(0,1); A_log ~ U(0, ln 16);
    dt_bias ~ U(0,1); gates as python/qwen35.py:597-600 computes them."""
    a = rng.standard_normal((B, L, H), dtype=np.float32)
    b = rng.standard_normal((B, L, H), dtype=np.float32)
    A_log = rng.uniform(0.0, np.log(16.0), (H,)).astype(np.float32)
    dt_bias = rng.uniform(0.0, 1.0, (H,)).astype(np.float32)
    return a, b, A_log, dt_bias


def gen_recurrent(mx, qwen35, D, cases, seed, name):
    rng = np.random.default_rng(seed)
    out = {}
    for i, (B, L, H) in enumerate(cases):
        q, k, v, al, bt, S0 = test_inputs(rng, B, L, H, D)
        o, S, states = qwen35.sequential_delta(mx.array(q), mx.array(k), mx.array(v),
                                               mx.array(al), mx.array(bt), mx.array(S0),
                                               collect=True)
        p = f"c{i}_"
        out.update({p + "shape": np.array([B, L, H, D]), p + "q": q, p + "k": k, p + "v": v,
                    p + "alpha": al, p + "beta": bt, p + "S0": S0,
                    p + "o": np.asarray(o, np.float32), p + "S": np.asarray(S, np.float32)})
        if L <= 9:
            out[p + "states"] = np.stack([np.asarray(s, np.float32) for s in states], 2)
    out["ncases"] = np.array(len(cases))
    np.savez_compressed(os.path.join(HERE, name), **out)


def gen_chunked(mx, qwen35, D, H, lengths, seed, name, model_style):
    rng = np.random.default_rng(seed)
    out = {}
    for i, L in enumerate(lengths):
        q, k, v, al, bt, S0 = test_inputs(rng, 1, L, H, D)
        if model_style:
            a, b, A_log, dt_bias = model_gates(rng, 1, L, H)
            A = mx.exp(mx.array(A_log))
            al = np.asarray(mx.exp(-A * qwen35.nn.softplus(mx.array(a) + mx.array(dt_bias))), np.float32)
            bt = np.asarray(mx.sigmoid(mx.array(b)), np.float32)
            out.update({f"c{i}_a": a, f"c{i}_b": b, f"c{i}_A_log": A_log, f"c{i}_dt_bias": dt_bias})
        args = [mx.array(x) for x in (q, k, v, al, bt)]
        # from a nonzero state; chunked_delta takes S as (B,H,Dv,Dk)
        yc2, Sc2 = qwen35.chunked_delta(*args, mx.array(S0))
        ys2, Ss2 = qwen35.sequential_delta(*args, mx.array(S0))
        p = f"c{i}_"
        out.update({p + "shape": np.array([1, L, H, D]), p + "q": q, p + "k": k, p + "v": v,
                    p + "alpha": al, p + "beta": bt, p + "S0": S0,
                    p + "o_chunk_s0": np.asarray(yc2, np.float32), p + "S_chunk_s0": np.asarray(Sc2, np.float32),
                    p + "o_seq_s0": np.asarray(ys2, np.float32), p + "S_seq_s0": np.asarray(Ss2, np.float32)})
    out["ncases"] = np.array(len(lengths))
    np.savez_compressed(os.path.join(HERE, name), **out)


def gen_block(mx, qwen35, dtype_name, seed, name):
    """GatedDeltaNet.__call__ + DeltaCache on nk=1, nv=3, dk=dv=128, K=4."""
    rng = np.random.default_rng(seed)
    act = mx.bfloat16 if dtype_name == "bf16" else mx.float32
    cfg = qwen35.TextConfig(hidden_size=8, linear_num_key_heads=1, linear_num_value_heads=3,
                            linear_key_head_dim=128, linear_value_head_dim=128,
                            linear_conv_kernel_dim=4)
    net = qwen35.GatedDeltaNet(cfg)
    C = net.qkv_dim
    conv_w = (rng.standard_normal((C, 1, 4), dtype=np.float32) * np.float32(0.5))
    A_log = rng.uniform(0.0, np.log(16.0), (net.nv,)).astype(np.float32)
    dt_bias = rng.uniform(0.0, 1.0, (net.nv,)).astype(np.float32)
    gamma = (1.0 + 0.1 * rng.standard_normal((net.dv,))).astype(np.float32)
    if act == mx.bfloat16:      # checkpoint tensors are bf16 in the model
        conv_w = np.asarray(mx.array(conv_w).astype(act).astype(mx.float32))
        A_log = np.asarray(mx.array(A_log).astype(act).astype(mx.float32))
        dt_bias = np.asarray(mx.array(dt_bias).astype(act).astype(mx.float32))
        gamma = np.asarray(mx.array(gamma).astype(act).astype(mx.float32))
    net.conv1d.weight = mx.array(conv_w).astype(act)
    net.A_log = mx.array(A_log)
    net.dt_bias = mx.array(dt_bias)
    net.norm.weight = mx.array(gamma)
    net.out_proj = lambda y: y          # the block output before out_proj

    def run(cache, L, tag, out):
        qkv = rng.standard_normal((1, L, C), dtype=np.float32)
        z = rng.standard_normal((1, L, net.z_dim), dtype=np.float32)
        a = rng.standard_normal((1, L, net.nv), dtype=np.float32)
        b = rng.standard_normal((1, L, net.nv), dtype=np.float32)
        qkv_m, z_m = mx.array(qkv).astype(act), mx.array(z).astype(act)
        a_m, b_m = mx.array(a).astype(act), mx.array(b).astype(act)
        net.in_proj_qkv = lambda x: qkv_m
        net.in_proj_z = lambda x: z_m
        net.in_proj_a = lambda x: a_m
        net.in_proj_b = lambda x: b_m
        x = mx.zeros((1, L, 8), act)
        y = net(x, cache)
        out[tag + "qkv"] = np.asarray(qkv_m.astype(mx.float32))
        out[tag + "z"] = np.asarray(z_m.astype(mx.float32))
        out[tag + "a"] = np.asarray(a_m.astype(mx.float32))
        out[tag + "b"] = np.asarray(b_m.astype(mx.float32))
        out[tag + "y"] = np.asarray(y.astype(mx.float32))
        return y

    out = {"conv_w": conv_w[:, 0, :], "A_log": A_log, "dt_bias": dt_bias, "gamma": gamma,
           "dims": np.array([net.nk, net.nv, net.dk, net.dv, net.K])}
    cache = qwen35.DeltaCache()
    run(cache, 20, "p_", out)                       # prefill: L >= 16 -> chunked_delta
    out["p_state"] = np.asarray(cache.state, np.float32)
    out["p_conv"] = np.asarray(cache.conv.astype(mx.float32))
    run(cache, 1, "d1_", out)                       # decode step
    out["d1_conv"] = np.asarray(cache.conv.astype(mx.float32))
    cache.record = True
    run(cache, 4, "v_", out)                        # speculative verify block
    cache.commit(2)                                 # accept the first 2 of 4
    out["v_state"] = np.asarray(cache.state, np.float32)
    out["v_conv"] = np.asarray(cache.conv.astype(mx.float32))
    out["v_offset"] = np.array(cache.offset)
    run(cache, 1, "d2_", out)                       # decode after rollback
    out["d2_conv"] = np.asarray(cache.conv.astype(mx.float32))
    short = qwen35.DeltaCache()
    run(short, 5, "s_", out)                        # short prefill: sequential path
    out["s_state"] = np.asarray(short.state, np.float32)
    out["s_conv"] = np.asarray(short.conv.astype(mx.float32))
    np.savez_compressed(os.path.join(HERE, name), **out)


def gen_spec(mx, seed, name):
    """``residual`` of the speculative acceptance step (python/speculative.py:
    100-106), the reference's own function, on seeded softmax pairs (V = 6 as
    its selftest, and V = 50), plus p == q (empty residual -> p) and a
    one-hot p (greedy)."""
    import speculative  # noqa: E402  (the reference; imports qwen35, generate, tokenizer)
    rng = np.random.default_rng(seed)
    ps, qs, rs = [], [], []

    def softmax(x):
        e = np.exp(x - x.max())
        return (e / e.sum()).astype(np.float32)

    for V in (6, 50):
        for _ in range(8):
            p = softmax(rng.standard_normal(V).astype(np.float32) * 2)
            q = softmax(rng.standard_normal(V).astype(np.float32) * 2)
            ps.append(p), qs.append(q)
    p = softmax(rng.standard_normal(50).astype(np.float32))
    ps.append(p), qs.append(p.copy())
    oh = np.zeros(50, np.float32)
    oh[7] = 1
    ps.append(oh), qs.append(softmax(rng.standard_normal(50).astype(np.float32)))
    for p, q in zip(ps, qs):
        rs.append(np.asarray(speculative.residual(mx.array(p), mx.array(q)), np.float32))
    out = {}
    for i, (p, q, r) in enumerate(zip(ps, qs, rs)):
        out[f"p{i}"], out[f"q{i}"], out[f"r{i}"] = p, q, r
    np.savez_compressed(os.path.join(HERE, name), **out)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("GDN_REFERENCE_PY"),
                    help="the reference checkout's python/ folder (or set GDN_REFERENCE_PY)")
    ap.add_argument("--only", choices=["spec"], default=None, help="regenerate one file set only")
    args = ap.parse_args()
    if not args.ref:
        ap.error("give --ref /path/to/reference/python or set GDN_REFERENCE_PY")
    mx, qwen35 = load_reference(args.ref)
    if args.only == "spec":
        gen_spec(mx, 1008, "spec_residual.npz")
        return
    gen_recurrent(mx, qwen35, 32, [(1, 1, 4), (1, 4, 4), (1, 9, 4), (2, 3, 2), (1, 64, 2)],
                  1001, "recurrent_d32.npz")
    gen_recurrent(mx, qwen35, 128, [(1, 1, 3), (1, 4, 1), (2, 3, 1), (1, 9, 1)],
                  1002, "recurrent_d128.npz")
    lengths = [1, 5, 16, 63, 64, 65, 130, 200]
    gen_chunked(mx, qwen35, 32, 2, lengths, 1003, "chunked_d32.npz", model_style=False)
    gen_chunked(mx, qwen35, 32, 1, lengths, 1004, "chunked_d32_model_gates.npz", model_style=True)
    gen_chunked(mx, qwen35, 128, 1, [130], 1005, "chunked_d128.npz", model_style=True)
    gen_block(mx, qwen35, "f32", 1006, "block_f32.npz")
    gen_block(mx, qwen35, "bf16", 1007, "block_bf16.npz")
    gen_spec(mx, 1008, "spec_residual.npz")
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    main()
