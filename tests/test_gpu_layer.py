"""A whole Gated DeltaNet layer (gdn_layer.GDNLayer: in_proj GEMMs -> conv ->
chunked recurrence with the gated norm -> out_proj) against the oracle's
GatedDeltaNet between its projections (gdn_oracle.gdn_block) with numpy
projections.

The projections round to bf16 as the reference's bf16 GEMMs do; the conv
output feeding the recurrence is bf16 on the GPU and fp32 in the oracle's
"f32" mode, so the normed output is compared at 5e-3 relative L2 and the
layer output (one more bf16 GEMM) at 1e-2 -- a wiring error (a wrong
channel, head, stride or token slice) is off by O(1)."""
import numpy as np
import pytest
import torch

import gdn_layer
import gdn_oracle as O

pytestmark = pytest.mark.gpu


def bf(x):
    return O.bf16_round(np.asarray(x, np.float32))


def reference(x, w, Hk, Hv, lens):
    """numpy: projections (fp32 of bf16 values, rounded to bf16), the oracle
    block per sequence, bf16 cast, out_proj.  Returns (normed, y)."""
    h = lambda t: t.float().cpu().numpy()  # noqa: E731
    xq = h(x)
    qkv = bf(xq @ h(w["W_qkv"]).T)
    z = bf(xq @ h(w["W_z"]).T)
    a = bf(xq @ h(w["W_a"]).T)
    b = bf(xq @ h(w["W_b"]).T)
    wts = O.BlockWeights(conv_w=h(w["conv_w"]), A_log=h(w["A_log"]), dt_bias=h(w["dt_bias"]),
                         gamma=h(w["gamma"]), nk=Hk, nv=Hv)
    outs, s = [], 0
    for L in lens:
        sl = slice(s, s + L)
        if L:
            outs.append(O.gdn_block(qkv[None, sl], z[None, sl], a[None, sl], b[None, sl], wts)[0])
        s += L
    normed = np.concatenate(outs)
    y = bf(normed) @ h(w["W_out"]).T
    return normed, y


@pytest.mark.parametrize("lens,packed", [([80, 80], False), ([50, 0, 130, 7], True)])
@pytest.mark.parametrize("Hk,Hv", [(4, 12), (2, 6)])
def test_layer_prefill_matches_oracle_block(lens, packed, Hk, Hv):
    """(2, 6) is an 8-GPU rank's shard: z | a | b is 780 columns, padded to 784."""
    hidden = 512
    dev = torch.device("cuda")
    w = gdn_layer.random_weights(hidden, Hk, Hv, dev, seed=7)
    tokens = sum(lens)
    g = torch.Generator(device=dev)
    g.manual_seed(8)
    x = torch.randn((tokens, hidden), generator=g, device=dev).bfloat16()
    layer = gdn_layer.layer_from(w, Hk, Hv)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]).astype(np.int32), device=dev) if packed else None
    normed = layer.core(layer.conv_projection(x, cu, len(lens)), *layer.projections_zab(x), cu_seqlens=cu,
                        B=len(lens))
    y, (lo, hi) = layer.forward_prefill(x, cu_seqlens=cu, B=len(lens))
    torch.cuda.synchronize()
    assert (lo, hi) == (0, tokens)
    rn, ry = reference(x, w, Hk, Hv, lens)
    assert O.rel_l2(normed.float().cpu().numpy().reshape(tokens, -1), rn) < 5e-3
    assert O.rel_l2(y.float().cpu().numpy(), ry) < 1e-2


def test_layer_decode_over_pool_matches_oracle_cache():
    """Three decode steps of 3 sequences in slots of a 6-slot pool (states
    and conv rings), against the oracle block with a per-sequence DeltaCache
    (per-token recurrence): the layer output every step, and the states and
    conv windows left in the slots."""
    Hk, Hv, hidden, n_slots = 4, 12, 512, 6
    dev = torch.device("cuda")
    w = gdn_layer.random_weights(hidden, Hk, Hv, dev, seed=9)
    layer = gdn_layer.layer_from(w, Hk, Hv)
    C = layer.C
    g = torch.Generator(device=dev)
    g.manual_seed(10)
    pool = torch.randn((n_slots, Hv, 128, 128), generator=g, device=dev) * 0.05
    ring = torch.randn((n_slots, 3, C), generator=g, device=dev).bfloat16()
    pos = torch.tensor([0, 1, 2, 0, 1, 2], dtype=torch.int32, device=dev)
    slots = torch.tensor([4, 0, 2], dtype=torch.int32, device=dev)
    B = 3
    h = lambda t: t.float().cpu().numpy()  # noqa: E731
    sl = slots.tolist()
    cache = O.DeltaCache(conv=np.stack([np.stack([h(ring[s, (int(pos[s]) + j) % 3]) for j in range(3)]) for s in sl]),
                         state=h(pool[slots.long()]))
    wts = O.BlockWeights(conv_w=h(w["conv_w"]), A_log=h(w["A_log"]), dt_bias=h(w["dt_bias"]),
                         gamma=h(w["gamma"]), nk=Hk, nv=Hv)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    for step in range(3):
        x = torch.randn((B, hidden), generator=g, device=dev).bfloat16()
        y, (lo, hi) = layer.forward_decode(x, pool, slots, ring, pos, err_flag=err)
        torch.cuda.synchronize()
        xq = h(x)
        qkv = bf(xq @ h(w["W_qkv"]).T)[:, None]
        z = bf(xq @ h(w["W_z"]).T)[:, None]
        a = bf(xq @ h(w["W_a"]).T)[:, None]
        b = bf(xq @ h(w["W_b"]).T)[:, None]
        out = O.gdn_block(qkv, z, a, b, wts, cache=cache)[:, 0]
        ry = bf(out) @ h(w["W_out"]).T
        assert (lo, hi) == (0, B)
        assert O.rel_l2(h(y), ry) < 1e-2, step
    assert int(err.item()) == 0
    assert O.rel_l2(h(pool[slots.long()]), cache.state) < 5e-3
    win = np.stack([np.stack([h(ring[s, (int(pos[s]) + j) % 3]) for j in range(3)]) for s in sl])
    assert O.rel_l2(win, cache.conv) < 1e-2
