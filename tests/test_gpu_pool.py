"""Serving-batch state pool: gdn_recurrent_fwd_pool (states in slots of a
pool, selected by a device index array) and the conv window as a ring per
slot (gdn_conv1d_fwd_pool + gdn_conv_ring_append).

The pooled calls run the same arithmetic as the dense entry points on the
same inputs, so they are compared bit for bit (torch.equal) with the dense
calls on gathered copies of the slots; one case also checks the oracle
(1e-5 max-relative, the decode bound).  Slots the call does not name must
stay untouched."""
import numpy as np
import pytest
import torch

import gdn_b200 as G
import gdn_oracle as O

pytestmark = pytest.mark.gpu
TOL = 1e-5


def dev(x, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(x)).to("cuda", dtype)


def inputs(rng, B, T):
    inp = O.synth_decode_inputs(rng, B, T)
    t = (dev(inp["q"], torch.bfloat16), dev(inp["k"], torch.bfloat16), dev(inp["v"], torch.bfloat16),
         dev(inp["a"]), dev(inp["b"]), dev(inp["A_log"]), dev(inp["dt_bias"]))
    return inp, t


def pool_of(rng, n_slots, Hv=48):
    return dev(rng.standard_normal((n_slots, Hv, 128, 128), dtype=np.float32) * np.float32(0.05))


@pytest.mark.parametrize("T", [1, 4])
def test_pool_final_matches_dense_and_leaves_other_slots(T):
    rng = np.random.default_rng(100 + T)
    B, n_slots = 3, 7
    inp, x = inputs(rng, B, T)
    pool = pool_of(rng, n_slots)
    before = pool.clone()
    slots = torch.tensor([5, 0, 3], dtype=torch.int32, device="cuda")
    dense_in = pool[slots.long()].contiguous()
    o_ref, S_ref, _ = G.recurrent_fwd(*x, state_in=dense_in)
    o, _ = G.recurrent_fwd_pool(*x, pool, slots, G.POOL_FINAL)
    torch.cuda.synchronize()
    assert torch.equal(o, o_ref)
    assert torch.equal(pool[slots.long()], S_ref)
    others = [s for s in range(n_slots) if s not in (5, 0, 3)]
    assert torch.equal(pool[others], before[others])
    if T == 1:   # and the dense path's oracle pin carries over
        ro, rS = O.delta_reference(O.expand_heads(inp["q"], 48), O.expand_heads(inp["k"], 48), inp["v"],
                                   *O.gates(inp["a"], inp["b"], inp["A_log"], inp["dt_bias"]),
                                   dense_in.cpu().numpy(), collect=False)
        assert O.rel_err(o.cpu().numpy(), ro) < TOL
        assert O.rel_err(pool[slots.long()].cpu().numpy(), rS) < TOL


def test_pool_keep_records_checkpoints_without_writing_the_pool():
    rng = np.random.default_rng(7)
    B, T, n_slots = 4, 4, 6
    _, x = inputs(rng, B, T)
    pool = pool_of(rng, n_slots)
    before = pool.clone()
    slots = torch.tensor([2, 4, 1, 5], dtype=torch.int32, device="cuda")
    ck_ref = torch.empty((B, 48, T, 128, 128), device="cuda")
    o_ref, _, _ = G.recurrent_fwd(*x, state_in=pool[slots.long()].contiguous(), ckpt=ck_ref)
    ck = torch.empty_like(ck_ref)
    o, _ = G.recurrent_fwd_pool(*x, pool, slots, G.POOL_KEEP, ckpt=ck)
    torch.cuda.synchronize()
    assert torch.equal(o, o_ref) and torch.equal(ck, ck_ref)
    assert torch.equal(pool, before)


def test_pool_verify_commit_chain_matches_dense_rollback():
    """Record block -> accept counts -> next step from the committed
    checkpoints, with the pool holding S_prev: the pooled chain equals the
    dense gdn_recurrent_fwd_from_ckpt chain, and POOL_START with T = 0
    materialises the commit (DeltaCache::commit) in the slots."""
    rng = np.random.default_rng(21)
    B, T, n_slots = 4, 4, 9
    _, ver = inputs(rng, B, T)
    pool = pool_of(rng, n_slots)
    slots = torch.tensor([8, 1, 6, 3], dtype=torch.int32, device="cuda")
    S_prev = pool[slots.long()].contiguous()
    ck = torch.empty((B, 48, T, 128, 128), device="cuda")
    G.recurrent_fwd_pool(*ver, pool, slots, G.POOL_KEEP, ckpt=ck)
    commit = torch.tensor([0, 1, 3, 4], dtype=torch.int32, device="cuda")
    _, nxt = inputs(rng, B, 1)
    o_ref, S_ref, _ = G.recurrent_fwd_from_ckpt(*nxt, S_prev, ck, commit)
    p2 = pool.clone()
    o, _ = G.recurrent_fwd_pool(*nxt, p2, slots, G.POOL_FINAL, ckpt_src=ck, commit_n=commit)
    torch.cuda.synchronize()
    assert torch.equal(o, o_ref)
    assert torch.equal(p2[slots.long()], S_ref)
    # T = 0 with POOL_START: the committed state itself lands in the slot
    p3 = pool.clone()
    empty = tuple(t[:, :0].contiguous() for t in nxt[:5]) + nxt[5:]
    G.recurrent_fwd_pool(*empty, p3, slots, G.POOL_START, ckpt_src=ck, commit_n=commit)
    torch.cuda.synchronize()
    for bi, n in enumerate(commit.tolist()):
        want = S_prev[bi] if n == 0 else ck[bi, :, n - 1]
        assert torch.equal(p3[int(slots[bi])], want), bi
    # POOL_START with a step: the slot holds the start state, o is the step's
    p4 = pool.clone()
    o4, _ = G.recurrent_fwd_pool(*nxt, p4, slots, G.POOL_START, ckpt_src=ck, commit_n=commit)
    torch.cuda.synchronize()
    assert torch.equal(o4, o_ref) and torch.equal(p4, p3)


def test_pool_bad_slot_sets_flag_and_writes_no_slot():
    rng = np.random.default_rng(3)
    B, n_slots = 3, 4
    _, x = inputs(rng, B, 1)
    pool = pool_of(rng, n_slots)
    before = pool.clone()
    slots = torch.tensor([1, 4, 2], dtype=torch.int32, device="cuda")     # 4 is out of range
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    dense_in = pool[[1, 2]].contiguous()
    o_ref, S_ref, _ = G.recurrent_fwd(*(t[[0, 2]].contiguous() if t.dim() > 1 else t for t in x), state_in=dense_in)
    o, _ = G.recurrent_fwd_pool(*x, pool, slots, G.POOL_FINAL, err_flag=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 1
    assert torch.equal(o[[0, 2]], o_ref)
    assert torch.equal(pool[[1, 2]], S_ref)
    assert torch.equal(pool[[0, 3]], before[[0, 3]])


def test_pool_argument_checks():
    rng = np.random.default_rng(4)
    _, x = inputs(rng, 2, 1)
    pool = pool_of(rng, 2)
    slots = torch.tensor([0, 1], dtype=torch.int32, device="cuda")
    with pytest.raises(G.GdnError) as e:
        G.recurrent_fwd_pool(*x, pool, slots, 7)
    assert e.value.code == G.GDN_ERR_FLAGS
    ck = torch.empty((2, 48, 1, 128, 128), device="cuda")
    with pytest.raises(G.GdnError) as e:
        G.recurrent_fwd_pool(*x, pool, slots, G.POOL_FINAL, ckpt_src=ck)       # commit_n missing
    assert e.value.code == G.GDN_ERR_NULL
    with pytest.raises(G.GdnError) as e:
        G.recurrent_fwd_pool(*x, pool, slots, G.POOL_FINAL, ckpt=pool.view(2, 48, 1, 128, 128))
    assert e.value.code == G.GDN_ERR_ALIAS


# ---- conv ring ---------------------------------------------------------------

C = 10240


def conv_weights(rng):
    return dev(rng.standard_normal((C, 4), dtype=np.float32) * np.float32(0.5), torch.bfloat16)


def test_ring_decode_steps_match_the_dense_conv_over_the_whole_sequence():
    """Prefill of a few tokens, then single-token steps with a one-row ring
    append each: every y equals the dense conv over the concatenated sequence."""
    rng = np.random.default_rng(30)
    n_slots, B = 5, 2
    slots = torch.tensor([3, 1], dtype=torch.int32, device="cuda")
    w = conv_weights(rng)
    ring = torch.zeros((n_slots, 3, C), dtype=torch.bfloat16, device="cuda")
    pos = torch.zeros(n_slots, dtype=torch.int32, device="cuda")
    lens = [5, 2]
    steps = 6
    full = [dev(rng.standard_normal((lens[i] + steps, C), dtype=np.float32), torch.bfloat16) for i in range(B)]
    ref = [G.conv1d_fwd(f[None].contiguous(), w)[0][0] for f in full]
    # prefill: packed sequences of lengths 5 and 2
    xp = torch.cat([full[0][:lens[0]], full[1][:lens[1]]]).contiguous()
    cu = torch.tensor([0, lens[0], lens[0] + lens[1]], dtype=torch.int32, device="cuda")
    y = G.conv1d_fwd_pool(xp, w, ring, pos, slots, cu_seqlens=cu)
    G.conv_ring_append(xp, ring, pos, slots, cu_seqlens=cu)
    torch.cuda.synchronize()
    assert torch.equal(y[:lens[0]], ref[0][:lens[0]]) and torch.equal(y[lens[0]:], ref[1][:lens[1]])
    for s in range(steps):
        xs = torch.stack([full[0][lens[0] + s], full[1][lens[1] + s]])[:, None].contiguous()   # (B, 1, C)
        ys = G.conv1d_fwd_pool(xs, w, ring, pos, slots)
        G.conv_ring_append(xs, ring, pos, slots)
        torch.cuda.synchronize()
        assert torch.equal(ys[0, 0], ref[0][lens[0] + s]), s
        assert torch.equal(ys[1, 0], ref[1][lens[1] + s]), s
    # the ring holds the last 3 rows, oldest at ring_pos
    for i, sl in enumerate(slots.tolist()):
        hd = int(pos[sl])
        got = torch.stack([ring[sl, (hd + j) % 3] for j in range(3)])
        assert torch.equal(got, full[i][-3:])
    assert torch.equal(ring[[0, 2, 4]], torch.zeros_like(ring[[0, 2, 4]]))


def test_ring_commit_after_a_verify_block_matches_conv_commit():
    rng = np.random.default_rng(31)
    n_slots, B, T = 6, 5, 4
    slots = torch.tensor([5, 0, 2, 4, 1], dtype=torch.int32, device="cuda")
    w = conv_weights(rng)
    ring = dev(rng.standard_normal((n_slots, 3, C), dtype=np.float32), torch.bfloat16)
    pos = torch.tensor([0, 1, 2, 0, 1, 2], dtype=torch.int32, device="cuda")
    # dense view of the windows, oldest first
    dense = torch.stack([torch.stack([ring[s, (int(pos[s]) + j) % 3] for j in range(3)]) for s in slots.tolist()])
    x = dev(rng.standard_normal((B, T, C), dtype=np.float32), torch.bfloat16)
    y_ref, _ = G.conv1d_fwd(x, w, state_in=dense.contiguous())
    y = G.conv1d_fwd_pool(x, w, ring, pos, slots)
    torch.cuda.synchronize()
    assert torch.equal(y, y_ref)
    commit = torch.tensor([0, 1, 2, 3, 4], dtype=torch.int32, device="cuda")
    win_ref = G.conv_commit(dense.contiguous(), x, commit)
    G.conv_ring_append(x, ring, pos, slots, counts=commit)
    torch.cuda.synchronize()
    for i, sl in enumerate(slots.tolist()):
        hd = int(pos[sl])
        got = torch.stack([ring[sl, (hd + j) % 3] for j in range(3)])
        assert torch.equal(got, win_ref[i]), i


def test_ring_bad_slot_or_count_sets_flag():
    rng = np.random.default_rng(32)
    w = conv_weights(rng)
    ring = torch.zeros((2, 3, C), dtype=torch.bfloat16, device="cuda")
    pos = torch.zeros(2, dtype=torch.int32, device="cuda")
    x = dev(rng.standard_normal((2, 1, C), dtype=np.float32), torch.bfloat16)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    G.conv1d_fwd_pool(x, w, ring, pos, torch.tensor([0, 2], dtype=torch.int32, device="cuda"), err_flag=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 1
    err.zero_()
    G.conv_ring_append(x, ring, pos, torch.tensor([0, 1], dtype=torch.int32, device="cuda"),
                       counts=torch.tensor([1, 2], dtype=torch.int32, device="cuda"), err_flag=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 1
    assert torch.equal(ring[0, 0], x[0, 0]) and torch.equal(ring[1], torch.zeros_like(ring[1]))
    assert pos.tolist() == [1, 0]
