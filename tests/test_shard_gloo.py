"""Multi-rank host logic on CPU: world-size-2 (and 4) gloo process groups run
one GDN layer head-sharded (each rank: its conv channels, gates, state and
gated norm, computed by the CPU oracle), all-gather the normed head outputs,
and must reproduce the unsharded layer exactly -- the sharding needs no
communication inside the recurrence.  Also: the shard map itself."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import gdn_oracle as O
import gdn_shard as S


def test_head_shard_map():
    shards = [S.head_shard(r, 8) for r in range(8)]
    assert [(s.k0, s.k1, s.v0, s.v1) for s in shards[:2]] == [(0, 2, 0, 6), (2, 4, 6, 12)]
    assert sum(s.hv for s in shards) == 48 and sum(s.hk for s in shards) == 16
    # every channel of the 10240-wide conv input belongs to exactly one rank
    owned = sorted(c for s in shards for c in S.channel_index(s))
    assert owned == list(range(10240))
    with pytest.raises(ValueError):
        S.head_shard(0, 3)
    with pytest.raises(ValueError):
        S.head_shard(2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _layer(rng, L, Hk, Hv):
    C = 2 * Hk * 128 + Hv * 128
    return dict(
        qkv=O.bf16_round(rng.standard_normal((1, L, C), dtype=np.float32)),
        z=O.bf16_round(rng.standard_normal((1, L, Hv * 128), dtype=np.float32)),
        a=rng.standard_normal((1, L, Hv), dtype=np.float32),
        b=rng.standard_normal((1, L, Hv), dtype=np.float32),
        conv_w=O.bf16_round(rng.standard_normal((C, 4), dtype=np.float32) * np.float32(0.5)),
        A_log=rng.uniform(0.0, np.log(16.0), (Hv,)).astype(np.float32),
        dt_bias=rng.uniform(0.0, 1.0, (Hv,)).astype(np.float32),
        gamma=(1 + 0.1 * rng.standard_normal(128)).astype(np.float32),
    )


def _rank_main(rank, world, port, L, Hk, Hv, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        x = _layer(np.random.default_rng(7), L, Hk, Hv)
        sh = S.head_shard(rank, world, Hk, Hv)
        ch = S.channel_index(sh, Hk)
        w = O.BlockWeights(conv_w=x["conv_w"][ch], A_log=x["A_log"][sh.v0:sh.v1],
                           dt_bias=x["dt_bias"][sh.v0:sh.v1], gamma=x["gamma"], nk=sh.hk, nv=sh.hv)
        zz = x["z"].reshape(1, L, Hv, 128)[:, :, sh.v0:sh.v1].reshape(1, L, sh.hv * 128)
        cache = O.DeltaCache()
        out = O.gdn_block(x["qkv"][..., ch], zz, x["a"][..., sh.v0:sh.v1], x["b"][..., sh.v0:sh.v1], w, cache)
        part = torch.from_numpy(out.reshape(L, sh.hv, 128).copy())
        gathered = [torch.empty_like(part) for _ in range(world)]
        dist.all_gather(gathered, part)
        st = torch.from_numpy(cache.state.copy())
        states = [torch.empty_like(st) for _ in range(world)]
        dist.all_gather(states, st)
        t = torch.tensor([float(rank + 1)])
        dist.all_reduce(t, op=dist.ReduceOp.MAX)        # the bench's max-over-ranks timing
        if rank == 0:
            q.put((S.assemble([g.numpy() for g in gathered]), S.assemble([s.numpy() for s in states], 1),
                   float(t.item())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_layer_equals_unsharded(world):
    L, Hk, Hv = 20, 4, 12            # chunked path (L >= 16), GQA 3:1
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, L, Hk, Hv, q)) for r in range(world)]
    for p in procs:
        p.start()
    out, states, tmax = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    x = _layer(np.random.default_rng(7), L, Hk, Hv)
    w = O.BlockWeights(conv_w=x["conv_w"], A_log=x["A_log"], dt_bias=x["dt_bias"], gamma=x["gamma"],
                       nk=Hk, nv=Hv)
    cache = O.DeltaCache()
    ref = O.gdn_block(x["qkv"], x["z"], x["a"], x["b"], w, cache).reshape(L, Hv, 128)
    assert np.array_equal(out, ref)
    assert np.array_equal(states, cache.state)
    assert tmax == float(world)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_layer_weight_shards_and_token_slices(world):
    """gdn_layer's host logic on CPU tensors: the ranks' weight rows put back
    together are the full weights (conv channels in [q | k | v] order, value
    heads in order), W_out and gamma are whole on every rank, and the token
    slices of out_proj cover every token exactly once."""
    import gdn_layer
    Hk, Hv, hidden = 16, 48, 64
    w = gdn_layer.random_weights(hidden, Hk, Hv, torch.device("cpu"), seed=3)
    parts = [gdn_layer.shard_weights(w, r, world, Hk, Hv) for r in range(world)]
    idx = [S.channel_index(S.head_shard(r, world, Hk, Hv), Hk) for r in range(world)]
    qkv = torch.empty_like(w["W_qkv"])
    conv = torch.empty_like(w["conv_w"])
    for p, ix in zip(parts, idx):
        qkv[ix] = p["W_qkv"]
        conv[ix] = p["conv_w"]
    assert torch.equal(qkv, w["W_qkv"]) and torch.equal(conv, w["conv_w"])
    for name in ("W_z", "W_a", "W_b", "A_log", "dt_bias"):
        assert torch.equal(torch.cat([p[name] for p in parts]), w[name]), name
    assert all(torch.equal(p["W_out"], w["W_out"]) and torch.equal(p["gamma"], w["gamma"]) for p in parts)
    for tokens in (0, 1, 7, 4096, 427463):
        layers = [gdn_layer.GDNLayer(p["W_qkv"], p["W_z"], p["W_a"], p["W_b"], p["conv_w"], p["A_log"], p["dt_bias"],
                                     p["gamma"], p["W_out"], Hk, Hv, r, world) for r, p in enumerate(parts)]
        cover = []
        for L in layers:
            lo, hi = L.token_slice(tokens)
            cover.extend(range(lo, hi))
        assert cover == list(range(tokens)), tokens
