"""Multi-GPU check of gdn_layer.GDNLayer, run as one process per GPU:

    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \\
        --master-port P tests/mgpu/layer_check.py

Every rank holds the same seeded full weights and input, runs the layer on
its head shard (in_proj rows of its channels, the fused NVLink gather, out_proj
on its token slice) and compares with the whole layer run on this GPU alone
(prefill, then two decode steps over state pools and conv rings):
the gathered normed output and its token slice of the layer output, within
1e-3 relative L2 (the sharded projections are GEMMs of other shapes, whose
sums may run in another order).  Exits non-zero on a mismatch or a device error.
"""
import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path[:0] = [os.path.join(ROOT, "qwen3.8-27b-mlx_b200", "python"), os.path.join(ROOT, "oracle")]
import gdn_b200 as G  # noqa: E402
import gdn_layer  # noqa: E402


def rel(a, b):
    a, b = a.float(), b.float()
    return float(torch.linalg.vector_norm(a - b) / torch.linalg.vector_norm(b))


def main():
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    Hk, Hv, hidden = 8, 24, 1024
    w = gdn_layer.random_weights(hidden, Hk, Hv, dev, seed=11)
    ok = True
    for rnd, lens in enumerate([[256, 256], [100, 3, 300, 61]]):
        packed = len(set(lens)) > 1
        tokens = sum(lens)
        g = torch.Generator(device=dev)
        g.manual_seed(100 + rnd)
        x = torch.randn((tokens, hidden), generator=g, device=dev).bfloat16()
        cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]).astype(np.int32), device=dev) if packed else None
        full = gdn_layer.layer_from(w, Hk, Hv)
        normed_full = full.core(full.conv_projection(x, cu, len(lens)), *full.projections_zab(x), cu_seqlens=cu,
                                B=len(lens))
        y_full, _ = full.forward_prefill(x, cu_seqlens=cu, B=len(lens))
        part = gdn_layer.layer_from(w, Hk, Hv, rank, world)
        y, (lo, hi) = part.forward_prefill(x, cu_seqlens=cu, B=len(lens))
        normed = part._gathers[part._g_i ^ 1].out
        torch.cuda.synchronize(dev)
        e_n, e_y = rel(normed, normed_full), rel(y, y_full[lo:hi])
        err = part.gather_errors() + G.take_device_error(dev)
        print(f"rank {rank} round {rnd}: normed rel {e_n:.2e}, out_proj slice [{lo},{hi}) rel {e_y:.2e}, "
              f"device errors {err}", flush=True)
        ok &= e_n < 1e-3 and e_y < 1e-3 and err == 0
        part.close()
    # decode: two steps of 6 sequences in slots of pools, sharded against one GPU
    full = gdn_layer.layer_from(w, Hk, Hv)
    part = gdn_layer.layer_from(w, Hk, Hv, rank, world)
    sh = part.shard
    n_slots, Bd = 10, 6
    g = torch.Generator(device=dev)
    g.manual_seed(200)
    pool_f = torch.randn((n_slots, Hv, 128, 128), generator=g, device=dev) * 0.05
    ring_f = torch.randn((n_slots, 3, full.C), generator=g, device=dev).bfloat16()
    pos_f = torch.zeros(n_slots, dtype=torch.int32, device=dev)
    slots = torch.tensor([7, 2, 9, 0, 4, 5], dtype=torch.int32, device=dev)
    idx = torch.tensor(gdn_layer.gdn_shard.channel_index(sh, Hk), device=dev)
    pool_p = pool_f[:, sh.v0:sh.v1].contiguous()
    ring_p = ring_f[:, :, idx].contiguous()
    pos_p = pos_f.clone()
    for step in range(2):
        x = torch.randn((Bd, hidden), generator=g, device=dev).bfloat16()
        y_full, _ = full.forward_decode(x, pool_f, slots, ring_f, pos_f)
        y, (lo, hi) = part.forward_decode(x, pool_p, slots, ring_p, pos_p)
        torch.cuda.synchronize(dev)
        e_y = rel(y, y_full[lo:hi]) if hi > lo else 0.0
        e_s = rel(pool_p, pool_f[:, sh.v0:sh.v1])
        print(f"rank {rank} decode step {step}: out_proj slice [{lo},{hi}) rel {e_y:.2e}, state rel {e_s:.2e}",
              flush=True)
        # bf16 in_proj outputs of GEMMs of other shapes may round one ulp apart; the state carries that
        ok &= e_y < 1e-2 and e_s < 1e-2
    dist.barrier()
    dist.destroy_process_group()
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()
