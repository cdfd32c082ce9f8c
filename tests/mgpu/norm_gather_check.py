"""Multi-GPU check of gdn_chunked_norm_gather_ws, run as one process per GPU:

    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \\
        --master-port P tests/mgpu/norm_gather_check.py

Every rank builds the same seeded layer (all heads), runs its head shard
with the gathered norm writing into every rank's output over NVLink, waits
for all ranks, and compares the whole gathered output with the single-GPU
fused path over all heads (gdn_chunked_norm_fwd_ws): bit-identical, since
each head is computed by the same kernels.  Two rounds (uniform batch, then
packed sequences) exercise the per-round counters.  Exits non-zero on a
mismatch or a device error.
"""
import ctypes
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
import gdn_shard  # noqa: E402


def main():
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    lib = G.lib()
    Hk, Hv = 8, 24                       # divisible at world 2, 4, 8
    shard = gdn_shard.head_shard(rank, world, Hk, Hv)
    ok = True
    for rnd, lens in enumerate([[192, 192], [100, 0, 257, 64, 3]]):
        packed = len(set(lens)) > 1
        total = sum(lens)
        g = torch.Generator(device=dev)
        g.manual_seed(1000 + rnd)
        x = torch.randn((total, 2 * Hk * 128 + Hv * 128), generator=g, device=dev).bfloat16()
        z = torch.randn((total, Hv, 128), generator=g, device=dev).bfloat16()
        a = torch.randn((total, Hv), generator=g, device=dev)
        b = torch.randn((total, Hv), generator=g, device=dev)
        A_log = torch.rand((Hv,), generator=g, device=dev) * float(np.log(16.0))
        dtb = torch.rand((Hv,), generator=g, device=dev)
        gamma = 1 + 0.1 * torch.randn((128,), generator=g, device=dev)
        S0 = torch.randn((len(lens), Hv, 128, 128), generator=g, device=dev) * 0.05
        cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]).astype(np.int32), device=dev) if packed else None
        B, T = (len(lens), total) if packed else (len(lens), lens[0])
        C = x.shape[1]
        q_all = x[:, :Hk * 128].view(total, Hk, 128)
        k_all = x[:, Hk * 128:2 * Hk * 128].view(total, Hk, 128)
        v_all = x[:, 2 * Hk * 128:].view(total, Hv, 128)
        lead = (total,) if packed else (B, T)
        shp = lambda t: t if packed else t.reshape(lead + t.shape[1:])  # noqa: E731
        # reference: all heads on this GPU
        ref, _ = G.chunked_norm_fwd(shp(q_all), shp(k_all), shp(v_all), shp(a), shp(b), A_log, dtb, shp(z), gamma,
                                    state_in=S0, cu_seqlens=cu)
        # this rank's shard, gathered into every rank's buffer
        pg = gdn_shard.PeerGather(total, Hv, dev)
        P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
        q = x[:, shard.k0 * 128:shard.k1 * 128]
        k = x[:, Hk * 128 + shard.k0 * 128:Hk * 128 + shard.k1 * 128]
        v = x[:, 2 * Hk * 128 + shard.v0 * 128:2 * Hk * 128 + shard.v1 * 128]
        zs = z[:, shard.v0:shard.v1].contiguous()
        a_s, b_s = a[:, shard.v0:shard.v1].contiguous(), b[:, shard.v0:shard.v1].contiguous()
        A_s, dt_s = A_log[shard.v0:shard.v1].contiguous(), dtb[shard.v0:shard.v1].contiguous()
        S_s = S0[:, shard.v0:shard.v1].contiguous()
        S_out = torch.empty_like(S_s)
        need = G.chunked_workspace_bytes(B, T, shard.hv, packed)
        ws = torch.empty(need, dtype=torch.uint8, device=dev)
        st = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
        for _ in range(2):
            pg.run(lib, P(q), P(k), P(v), C, C, C, P(a_s), P(b_s), P(A_s), P(dt_s), P(S_s), P(S_out), P(zs),
                   shard.hv * 128, P(gamma), 1e-6, shard.v0, P(cu) if packed else None, B, T, shard.hk, shard.hv,
                   G.F_QK_L2NORM, P(ws), need, st)
            pg.wait(lib, st)
        torch.cuda.synchronize(dev)
        got = pg.out.view(lead + (Hv, 128))
        same = torch.equal(got, ref)
        err = int(pg.err.item()) + G.take_device_error(dev)
        print(f"rank {rank} round {rnd}: gathered == single-GPU {same}, device errors {err}", flush=True)
        ok &= same and err == 0
        pg.close()
        del pg
    dist.barrier()
    dist.destroy_process_group()
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()
