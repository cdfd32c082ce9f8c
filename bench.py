#!/usr/bin/env python
"""Benchmark of the B200 Gated DeltaNet hot path.  Prints ONE JSON line (rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline workload: all 48 GDN layers of Qwen3.5/3.8-27B
decode one token for a batch of B = 256 sequences; per layer and sequence the
fp32 state (48 value heads x 128 x 128) is read and written once, in place.
A step is the 48 per-layer launches of ``gdn_recurrent_fwd`` (sequential, as
the layers of a real model are), replayed from a CUDA graph.  The metric is
state bytes moved (read + write) per second of device time.

N > 1 GPUs (torchrun, one process per GPU): the K-head groups are sharded
(rank r owns 16/N key heads and their 48/N value heads) over a global batch
of B*N sequences, so per-GPU work is fixed ("weak" scaling), and after every
layer the bf16 head outputs are all-gathered over NCCL (the layer-boundary
collective), overlapped with the next layer on a side stream.

``--impl reference`` times the reference's CPU path (the C oracle's
restatement of delta::run_reference, all host threads) on a bounded sample of
the same workload and prints the same line with "impl": "reference".
"""
from __future__ import annotations

import argparse
import ctypes
import datetime
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "qwen3.8-27b-mlx_b200")
for _p in (os.path.join(PKG, "python"), os.path.join(ROOT, "oracle")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "GDN decode state HBM GB/s vs ~8 TB/s; chunked prefill tokens/s at 1/2/4/8 GPU"
D = 128
HK, HV = 16, 48
# ncu dram__bytes_read.sum + dram__bytes_write.sum of one recurrent_kernel launch
# at B = 256, 48 value heads (810,676,992 + 748,824,832 bytes)
DECODE_TRAFFIC_B256 = 810676992 + 748824832
STATE_BYTES = D * D * 4                   # one (Dv, Dk) fp32 head state


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------

class ClockSampler:
    FIELDS = ("index,uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.uuid = None
        try:
            self.uuid = str(torch.cuda.get_device_properties(device).uuid)
        except Exception:
            pass
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                out = ""
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self):
        rows = []
        for ln in getattr(self, "lines", []):
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            if self.uuid and self.uuid.replace("GPU-", "") not in f[1]:
                continue
            rows.append(f)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        sm = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(rows[0][3]) if rows[0][3].replace(".", "").isdigit() else None,
                "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------

def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def barrier(world):
    if world > 1:
        torch.distributed.barrier()


def max_over_ranks(x, world, device):
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=device)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------------------
# the decode workload
# ---------------------------------------------------------------------------

class DecodeLayers:
    """Device buffers of L stacked GDN layers for one rank's head shard."""

    def __init__(self, L, B, hk, hv, device, seed):
        self.L, self.B, self.hk, self.hv = L, B, hk, hv
        g = torch.Generator(device=device)
        self.q, self.k, self.v, self.a, self.b = [], [], [], [], []
        self.A_log, self.dt_bias, self.S, self.o = [], [], [], []
        for layer in range(L):
            g.manual_seed(seed * 1000 + layer)
            qf = torch.randn((B, 1, hk, D), generator=g, device=device).bfloat16().float()
            kf = torch.randn((B, 1, hk, D), generator=g, device=device).bfloat16().float()
            qf = qf * torch.rsqrt((qf * qf).sum(-1, keepdim=True) + 1e-6) * D ** -0.5
            kf = kf * torch.rsqrt((kf * kf).sum(-1, keepdim=True) + 1e-6)
            self.q.append(qf.bfloat16().contiguous())
            self.k.append(kf.bfloat16().contiguous())
            self.v.append(torch.randn((B, 1, hv, D), generator=g, device=device).bfloat16())
            self.a.append(torch.randn((B, 1, hv), generator=g, device=device))
            self.b.append(torch.randn((B, 1, hv), generator=g, device=device))
            self.A_log.append(torch.rand((hv,), generator=g, device=device) * float(np.log(16.0)))
            self.dt_bias.append(torch.rand((hv,), generator=g, device=device))
            self.S.append(torch.randn((B, hv, D, D), generator=g, device=device) * 0.05)
            self.o.append(torch.empty((B, 1, hv, D), dtype=torch.bfloat16, device=device))

    def state_bytes(self, B=None):
        return 2 * (B or self.B) * self.hv * STATE_BYTES * self.L


def launch_layer(lib, X, layer, B, stream_handle, q=None, k=None, v=None, a=None, b=None, o=None, overlap=False):
    """One gdn_recurrent_fwd launch over the first B sequences of one layer
    (in-place state update, bf16 output); overlap: GDN_F_OVERLAP_PREV -- the
    previous kernel in the stream is another layer's, so this launch may
    overlap its tail."""
    import gdn_b200 as G
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    S = X.S[layer]
    rc = lib.gdn_recurrent_fwd(P(q if q is not None else X.q[layer]), P(k if k is not None else X.k[layer]),
                               P(v if v is not None else X.v[layer]), P(a if a is not None else X.a[layer]),
                               P(b if b is not None else X.b[layer]), P(X.A_log[layer]), P(X.dt_bias[layer]),
                               P(S), P(S), P(o if o is not None else X.o[layer]), None,
                               B, 1, X.hk, X.hv, D, D, G.F_O_BF16 | (G.F_OVERLAP_PREV if overlap else 0),
                               stream_handle)
    if rc != 0:
        raise RuntimeError(f"gdn_recurrent_fwd failed: {rc} {lib.gdn_last_error().decode()}")


def time_graph(fn, steps, warmup, device, world):
    """Capture fn() (one step) in a CUDA graph, warm up, then time `steps`
    replays with CUDA events; returns max-over-ranks milliseconds."""
    s = torch.cuda.Stream(device)
    s.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(s):
        fn()                                 # load modules outside the capture
    torch.cuda.current_stream(device).wait_stream(s)
    torch.cuda.synchronize(device)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    for _ in range(warmup):
        g.replay()
    torch.cuda.synchronize(device)
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        g.replay()
    e1.record()
    torch.cuda.synchronize(device)
    barrier(world)
    ms = e0.elapsed_time(e1)
    del g
    return max_over_ranks(ms, world, device)


def run_pool_decode(args, lib, X, Bg, device, Lp=8):
    """Decode over a state pool (gdn_recurrent_fwd_pool): Bg sequences in
    seeded random slots of a pool of 2*Bg, Lp layers, against the dense
    in-place launch on the same inputs (both CUDA-graph replays, states far
    above L2); and one layer's conv step through the ring (gdn_conv1d_fwd_pool
    + gdn_conv_ring_append, one row written per sequence) against the dense
    conv with a carried (B, 3, C) window."""
    import gdn_b200 as G
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    Lp = min(Lp, X.L)
    n_slots = 2 * Bg
    g = torch.Generator(device=device)
    g.manual_seed(4242)
    pools = [torch.randn((n_slots, X.hv, D, D), generator=g, device=device) * 0.05 for _ in range(Lp)]
    slots = torch.randperm(n_slots, generator=g, device=device)[:Bg].to(torch.int32)
    err = torch.zeros(1, dtype=torch.int32, device=device)

    def step_pool():
        h = ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)
        for layer in range(Lp):
            rc = lib.gdn_recurrent_fwd_pool(P(X.q[layer]), P(X.k[layer]), P(X.v[layer]), P(X.a[layer]),
                                            P(X.b[layer]), P(X.A_log[layer]), P(X.dt_bias[layer]), P(pools[layer]),
                                            P(slots), n_slots, None, None, 0, G.POOL_FINAL, P(X.o[layer]), None,
                                            P(err), Bg, 1, X.hk, X.hv, D, D, G.F_O_BF16, h)
            if rc:
                raise RuntimeError(lib.gdn_last_error().decode())

    def step_dense():
        h = ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)
        for layer in range(Lp):
            launch_layer(lib, X, layer, Bg, h)

    steps = max(args.steps, 10)
    ms_pool = time_graph(step_pool, steps, args.warmup, device, 1) / steps
    ms_dense = time_graph(step_dense, steps, args.warmup, device, 1) / steps
    per_step = 2 * Bg * X.hv * STATE_BYTES * Lp
    Cc = 2 * X.hk * D + X.hv * D
    x = torch.randn((Bg, 1, Cc), generator=g, device=device).bfloat16()
    w = (torch.randn((Cc, 4), generator=g, device=device) * 0.5).bfloat16()
    y = torch.empty_like(x)
    ring = torch.zeros((n_slots, 3, Cc), dtype=torch.bfloat16, device=device)
    pos = torch.zeros(n_slots, dtype=torch.int32, device=device)
    win = [torch.zeros((Bg, 3, Cc), dtype=torch.bfloat16, device=device) for _ in range(2)]

    def conv_ring():
        h = ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)
        rc = lib.gdn_conv1d_fwd_pool(P(x), P(w), P(ring), P(pos), P(slots), n_slots, P(y), None, Bg, 1, Cc, 4, 0,
                                     P(err), h)
        rc = rc or lib.gdn_conv_ring_append(P(x), P(ring), P(pos), P(slots), n_slots, None, None, Bg, 1, Cc, 4,
                                            P(err), h)
        if rc:
            raise RuntimeError(lib.gdn_last_error().decode())

    def conv_dense():
        h = ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)
        rc = lib.gdn_conv1d_fwd(P(x), P(w), P(win[0]), P(win[1]), P(y), None, Bg, 1, Cc, 4, 0, h)
        if rc:
            raise RuntimeError(lib.gdn_last_error().decode())

    csteps = 200
    us_ring = time_graph(conv_ring, csteps, args.warmup, device, 1) / csteps * 1e3
    us_dense = time_graph(conv_dense, csteps, args.warmup, device, 1) / csteps * 1e3
    torch.cuda.synchronize(device)
    if int(err.item()):
        raise RuntimeError("pool decode recorded a slot error")
    out = {"workload": f"{Lp} layers x B={Bg} decode, states in random slots of a {n_slots}-slot pool "
                       f"({n_slots * X.hv * STATE_BYTES * Lp / 1e9:.1f} GB)",
           "recurrent_pool_gbs": round(per_step / (ms_pool * 1e-3) / 1e9, 1),
           "recurrent_dense_gbs": round(per_step / (ms_dense * 1e-3) / 1e9, 1),
           "conv_ring_us": round(us_ring, 2), "conv_dense_us": round(us_dense, 2),
           "conv_note": f"one layer's conv step, B={Bg}, C={Cc}: ring (conv + one-row append) vs dense "
                        "(conv + 3-row window copy)"}
    del pools, ring, win
    torch.cuda.empty_cache()
    return out


def run_ours(args, world, rank, local):
    import gdn_b200 as G
    import gdn_shard
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    lib = G.lib()
    shard = gdn_shard.head_shard(rank, world, HK, HV)
    hk, hv = shard.hk, shard.hv
    B = args.batch
    Bg = B * world                                  # global batch; every rank holds all of it for its heads
    L = args.layers
    X = DecodeLayers(L, Bg, hk, hv, device, seed=17 + rank)
    torch.cuda.synchronize(device)
    hbm_peak, _, peak_kind = peaks()

    gathered = None
    comm = None
    if world > 1:
        gathered = [torch.empty((world,) + tuple(X.o[i].shape), dtype=torch.bfloat16, device=device)
                    for i in range(L)]
        comm = torch.cuda.Stream(device)

    def step(Bsub=Bg):
        st = torch.cuda.current_stream(device)
        h = ctypes.c_void_p(st.cuda_stream)
        for layer in range(L):
            launch_layer(lib, X, layer, Bsub, h, overlap=True)   # consecutive launches are different layers
            if world > 1:
                comm.wait_stream(st)
                with torch.cuda.stream(comm):
                    torch.distributed.all_gather_into_tensor(gathered[layer], X.o[layer])
        if world > 1:
            st.wait_stream(comm)

    # --- headline: graph-replayed steps (N == 1) or eager steps with the gathers (N > 1)
    with ClockSampler(device) as clk:
        if world == 1:
            ms = time_graph(step, args.steps, args.warmup, device, world)
        else:
            for _ in range(args.warmup):
                step()
            torch.cuda.synchronize(device)
            barrier(world)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(args.steps):
                step()
            e1.record()
            torch.cuda.synchronize(device)
            barrier(world)
            ms = max_over_ranks(e0.elapsed_time(e1), world, device)
    clocks = clk.summary()
    ms_step = ms / args.steps
    bytes_step_rank = X.state_bytes()
    value = world * bytes_step_rank / (ms_step * 1e-3) / 1e9

    # --- roofline: the dominant kernel's average launch duration (CUDA events per launch)
    st = torch.cuda.current_stream(device)
    h = ctypes.c_void_p(st.cuda_stream)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(L)]
    durs = []
    for _ in range(max(1, min(args.steps, 20))):
        for layer in range(L):
            evs[layer][0].record(st)
            launch_layer(lib, X, layer, Bg, h)
            evs[layer][1].record(st)
        torch.cuda.synchronize(device)
        durs += [a.elapsed_time(b) for a, b in evs]
    launch_ms = statistics.mean(durs)
    per_launch = 2 * Bg * hv * STATE_BYTES
    achieved = per_launch / (launch_ms * 1e-3) / 1e9
    # dram bytes of one launch from an ncu capture (--traffic overrides): the
    # value for 256 sequences x 48 heads of state per launch was measured on
    # this kernel at that shape; other shapes report null
    traffic, traffic_src = args.traffic, "--traffic" if args.traffic is not None else None
    if traffic is None and per_launch == 2 * 256 * HV * STATE_BYTES:   # same bytes at every shard split
        traffic, traffic_src = DECODE_TRAFFIC_B256, "ncu dram__bytes_read.sum + dram__bytes_write.sum, B=256 launch"
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                "frac": round(achieved / hbm_peak, 4), "peak_kind": peak_kind,
                "frac_of_8TBps": round(achieved / 8000.0, 4),
                "kernel": "recurrent_kernel", "bytes_per_launch": per_launch,
                "launch_ms": round(launch_ms, 5), "traffic": traffic, "traffic_source": traffic_src}

    # --- batch sweep (B in {1, 16, 64, 256})
    sweep = {}
    if world == 1 and args.sweep:
        for Bs in [int(x) for x in args.sweep.split(",") if x]:
            if Bs > Bg:
                continue
            msb = time_graph(lambda: step(Bs), max(args.steps, 20), args.warmup, device, world)
            sweep[str(Bs)] = round(X.state_bytes(Bs) / (msb / max(args.steps, 20) * 1e-3) / 1e9, 1)

    # --- the same decode over a serving-batch state pool (scattered slots) and the conv ring
    def guarded(name, fn):
        """An optional section: its exception becomes an "error" entry of the
        line (and a traceback on stderr) instead of costing the headline.  Its
        failures are the same on every rank (the collective checks raise on all
        ranks together), so the ranks stay in step."""
        try:
            return fn()
        except Exception as e:  # noqa: BLE001
            import traceback
            traceback.print_exc(file=sys.stderr)
            torch.cuda.empty_cache()
            return {"error": f"{name}: {type(e).__name__}: {e}"}

    pool = None
    if world == 1 and not args.no_pool:
        pool = guarded("pool_decode", lambda: run_pool_decode(args, lib, X, Bg, device))

    # --- end to end through the C ABI with host buffers (pipelined per layer)
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(args, lib, X, Bg, device, world)

    cpu = None
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        cpu = cpu_baseline(seconds=args.cpu_seconds, B=Bg, L=args.ref_layers)

    verify = None
    if not args.no_verify:
        verify = guarded("verify_chain", lambda: run_verify_chain(args, lib, device, world, hk, hv, hbm_peak))

    prefill = None
    if not args.no_prefill:
        del X
        torch.cuda.empty_cache()
        prefill = guarded("prefill", lambda: run_prefill(args, lib, device, world))
        if world == 1 and rank == 0 and not args.no_cpu_baseline and "config3" in prefill:
            prefill["config3"]["cpu_baseline"] = cpu_prefill_baseline(T=args.prefill_T, seconds=args.cpu_seconds)
    layer = None
    if not args.no_layer:
        layer = {"decode": guarded("layer.decode", lambda: run_layer_decode(args, device, world))}
        if not args.no_prefill:
            layer.update(guarded("layer", lambda: run_layer(args, device, world)))

    # compact copies of the secondary results where a reader of the line looks
    # first: the decode sweep next to the headline's roofline, and the prefill
    # configs' throughput and tensor-roofline fractions (details in *_detail)
    roofline["by_batch_gbs"] = sweep
    roofline["by_batch_frac"] = {b: round(v / hbm_peak, 4) for b, v in sweep.items()}
    prefill_summary = None
    if isinstance(prefill, dict):
        prefill_summary = {}
        for name, r in prefill.items():
            if not isinstance(r, dict) or "roofline" not in r:
                prefill_summary[name] = r
                continue
            keep = {k: r[k] for k in ("schedule", "tokens_per_s", "tokens_per_s_per_layer", "ms_per_layer",
                                      "tokens_per_s_without_gather") if k in r}
            if "stack_48_layers" in r:
                keep["tokens_per_s_48_layers"] = r["stack_48_layers"]["tokens_per_s"]
                keep["ms_48_layers"] = r["stack_48_layers"]["ms"]
            keep["chunked_ms"] = r["kernel_ms"].get("chunked")
            keep["tensor_frac"] = r["roofline"]["frac"]
            if "cpu_baseline" in r:
                keep["cpu_tokens_per_s"] = r["cpu_baseline"]["value"]
            prefill_summary[name] = keep
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded; BASELINE config-0 distributions, independent seed per layer)",
        "config": {"workload": f"config1: {L} GDN layers, decode T=1, B={Bg} per GPU shard, "
                               f"Hk={HK} Hv={HV} Dk=Dv=128, fp32 state in place, bf16 q/k/v/o",
                   "global_batch": Bg, "seq_len": 1, "layers": L,
                   "parallelism": "single" if world == 1 else f"kheads{world}+allgather",
                   "heads_per_gpu": {"k": hk, "v": hv},
                   "l2": f"inputs larger than L2 (state {bytes_step_rank / 2 / 1e9:.1f} GB per GPU)",
                   "timing": ("CUDA graph replay of the 48 launches, each a programmatic dependent of the previous "
                              "layer's (GDN_F_OVERLAP_PREV)") if world == 1 else
                             "eager + NCCL all-gather, launches with GDN_F_OVERLAP_PREV"},
        "roofline": roofline, "clocks": clocks, "gpu_launches": args.steps * L,
        "sweep_gbs_by_batch": sweep, "e2e": e2e, "cpu_baseline": cpu, "prefill": prefill_summary,
        "pool_decode": pool, "verify_chain": verify, "prefill_detail": prefill, "layer": layer,
    }
    return line


VOCAB = 248320          # Qwen3.5/3.8 vocabulary (the verify pass's distributions are over it)


def run_verify_chain(args, lib, device, world, hk, hv, hbm_peak, B=32, k=3):
    """BASELINE config 2 as a device-resident chain per step: the (k+1)-token
    verify block with checkpoints (gdn_recurrent_fwd), the acceptance test on
    seeded target/draft distributions over the vocabulary (gdn_spec_verify),
    the conv-window rollback (gdn_conv_commit) and the next decode step from
    the accepted checkpoint (gdn_recurrent_fwd_from_ckpt) -- no host read.
    Reports ms per step (max over ranks), the checkpoint-write bandwidth of
    the verify kernel and the acceptance kernel's read rate."""
    import gdn_b200 as G
    g = torch.Generator(device=device)
    g.manual_seed(31)
    T = k + 1
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    def bf(*shape):
        return torch.randn(shape, generator=g, device=device).bfloat16()
    q, kk, v = bf(B, T, hk, D), bf(B, T, hk, D), bf(B, T, hv, D)
    q1, k1, v1 = bf(B, 1, hk, D), bf(B, 1, hk, D), bf(B, 1, hv, D)
    a = torch.randn((B, T, hv), generator=g, device=device)
    b = torch.randn((B, T, hv), generator=g, device=device)
    a1, b1 = torch.randn((B, 1, hv), generator=g, device=device), torch.randn((B, 1, hv), generator=g, device=device)
    A_log = torch.rand((hv,), generator=g, device=device) * float(np.log(16.0))
    dtb = torch.rand((hv,), generator=g, device=device)
    S = torch.randn((B, hv, D, D), generator=g, device=device) * 0.05
    S_next = torch.empty_like(S)
    ckpt = torch.empty((B, hv, T, D, D), device=device)
    o = torch.empty((B, T, hv, D), dtype=torch.bfloat16, device=device)
    o1 = torch.empty((B, 1, hv, D), dtype=torch.bfloat16, device=device)
    C = 2 * hk * D + hv * D
    xw, xb = bf(B, 3, C), bf(B, T, C)
    conv_next = torch.empty_like(xw)
    # target and draft distributions that overlap like a real MTP head's (the
    # draft's logits are the target's plus noise): a few drafts get accepted
    logits = torch.randn((B, T, VOCAB), generator=g, device=device) * 4
    pr = torch.softmax(logits, -1)
    qr = torch.softmax(logits[:, :k] + torch.randn((B, k, VOCAB), generator=g, device=device) * 0.5, -1)
    draft = torch.multinomial(qr.reshape(-1, VOCAB), 1, generator=g).reshape(B, k).int()
    ua = torch.rand((B, k), generator=g, device=device)
    us = torch.rand((B,), generator=g, device=device)
    acc, commit, tok = (torch.empty(B, dtype=torch.int32, device=device) for _ in range(3))
    err = torch.zeros(1, dtype=torch.int32, device=device)
    st = torch.cuda.current_stream(device)
    h = ctypes.c_void_p(st.cuda_stream)
    flags = G.F_O_BF16

    def chk(rc):
        if rc:
            raise RuntimeError(lib.gdn_last_error().decode())

    def verify():
        chk(lib.gdn_recurrent_fwd(P(q), P(kk), P(v), P(a), P(b), P(A_log), P(dtb), P(S), None, P(o), P(ckpt),
                                  B, T, hk, hv, D, D, flags, h))

    def accept():
        chk(lib.gdn_spec_verify(P(pr), P(qr), P(draft), P(ua), P(us), B, k, VOCAB, P(acc), P(commit), P(tok),
                                P(err), h))

    def rollback_and_decode():
        chk(lib.gdn_conv_commit(P(xw), P(xb), P(commit), P(conv_next), P(err), B, T, C, 4, h))
        chk(lib.gdn_recurrent_fwd_from_ckpt(P(q1), P(k1), P(v1), P(a1), P(b1),
                                            P(A_log), P(dtb), P(S), P(ckpt), P(commit), T, P(S_next), P(o1), None,
                                            P(err), B, 1, hk, hv, D, D, flags, h))

    def chain():
        verify()
        accept()
        rollback_and_decode()

    steps = max(5, args.steps // 10)
    for _ in range(max(args.warmup, 3)):
        chain()
    torch.cuda.synchronize(device)
    barrier(world)
    e = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    e[0].record(st)
    for _ in range(steps):
        chain()
    e[1].record(st)
    torch.cuda.synchronize(device)
    barrier(world)
    ms = max_over_ranks(e[0].elapsed_time(e[1]) / steps, world, device)
    # per-kernel times: 10 back-to-back launches each (both are idempotent: verify
    # writes only the checkpoints, accept only its outputs), so the figure is a
    # launch in steady state rather than one launch after a synchronize
    reps = 10
    e[0].record(st)
    for _ in range(reps):
        verify()
    e[1].record(st)
    for _ in range(reps):
        accept()
    e[2].record(st)
    torch.cuda.synchronize(device)
    tv, ta = e[0].elapsed_time(e[1]) / reps, e[1].elapsed_time(e[2]) / reps
    state = B * hv * D * D * 4
    verify_bytes = state * (1 + T)                         # read S, write T checkpoints (S_out aliases the last)
    j = acc.cpu().numpy()
    accept_bytes = int(sum((2 if jj < k else 1) * VOCAB * 4 for jj in j))   # residual row pair or p_k row
    if int(err.item()):
        raise RuntimeError("verify chain raised the device error flag")
    return {"workload": f"config2: B={B}, k+1={T} verify with checkpoints -> on-device accept over V={VOCAB} "
                        f"-> conv rollback -> decode from the accepted checkpoint (Hk={hk} Hv={hv} per GPU)",
            "ms_per_step": round(ms, 4), "verify_ms": round(tv, 4),
            "verify_gbs": round(verify_bytes / (tv * 1e-3) / 1e9, 1),
            "verify_frac": round(verify_bytes / (tv * 1e-3) / 1e9 / hbm_peak, 4),
            "accept_ms": round(ta, 4), "accept_gbs": round(accept_bytes / (ta * 1e-3) / 1e9, 1),
            "mean_accepted": round(float(j.mean()), 3), "gpu_launches_per_step": 4}


def run_e2e(args, lib, X, Bg, device, world):
    """Same metric through the C ABI with the per-step inputs copied from
    pinned host memory and the outputs read back, all inside the timed region.
    Copies of layer l+1 overlap the kernel of layer l (two slots per buffer)."""
    L = X.L
    names = ("q", "k", "v", "a", "b")
    host = [{n: getattr(X, n)[i].cpu().pin_memory() for n in names} for i in range(L)]
    o_host = [torch.empty(X.o[i].shape, dtype=X.o[i].dtype).pin_memory() for i in range(L)]
    slots = [{n: torch.empty_like(getattr(X, n)[0]) for n in names} for _ in range(2)]
    o_slots = [torch.empty_like(X.o[0]) for _ in range(2)]
    h2d_b = sum(t.numel() * t.element_size() for t in host[0].values()) * L
    d2h_b = sum(t.numel() * t.element_size() for t in o_host)
    comp = torch.cuda.current_stream(device)
    cin, cout = torch.cuda.Stream(device), torch.cuda.Stream(device)
    ev = lambda: torch.cuda.Event()  # noqa: E731
    in_ready = [ev(), ev()]
    slot_free = [ev(), ev()]
    out_done = [ev(), ev()]
    kdone = [ev(), ev()]
    hcomp = ctypes.c_void_p(comp.cuda_stream)

    def step():
        for layer in range(L):
            s = layer % 2
            cin.wait_event(slot_free[s])
            with torch.cuda.stream(cin):
                for n in names:
                    slots[s][n].copy_(host[layer][n], non_blocking=True)
            in_ready[s].record(cin)
            comp.wait_event(in_ready[s])
            comp.wait_event(out_done[s])
            launch_layer(lib, X, layer, Bg, hcomp, o=o_slots[s], **slots[s])
            kdone[s].record(comp)
            slot_free[s].record(comp)
            cout.wait_event(kdone[s])
            with torch.cuda.stream(cout):
                o_host[layer].copy_(o_slots[s], non_blocking=True)
            out_done[s].record(cout)
        comp.wait_stream(cout)

    for e in slot_free + out_done:
        e.record(comp)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(device)
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    steps = max(1, args.steps // 2)
    e0.record(comp)
    cin.wait_stream(comp)
    for _ in range(steps):
        step()
    e1.record(comp)
    torch.cuda.synchronize(device)
    barrier(world)
    ms = max_over_ranks(e0.elapsed_time(e1), world, device) / steps
    value = world * X.state_bytes() / (ms * 1e-3) / 1e9
    return {"value": round(value, 1), "unit": "GB/s", "h2d_bytes_per_step": h2d_b,
            "d2h_bytes_per_step": d2h_b, "ms_per_step": round(ms, 4), "steps": steps,
            "api": "gdn_recurrent_fwd (C ABI via ctypes), pinned host inputs/outputs"}


# ---------------------------------------------------------------------------
# prefill: BASELINE config 3 (conv -> chunked recurrence -> gated norm)
# ---------------------------------------------------------------------------

FLOP_PER_TOKEN_HEAD = 12 * 64 * 128 + 6 * 128 * 128      # chunked WY form, C = 64, D = 128


class PrefillLayer:
    """One GDN layer's prefill inputs on the device (BASELINE config 3/4
    distributions) for a shard of hk key / hv value heads: x (tokens, C)
    bf16 projection output (C = 2*hk*128 + hv*128), conv weights, z, gamma,
    gate inputs.  `lens` packs sequences of those lengths (cu_seqlens)."""

    def __init__(self, lens, device, seed, hk=HK, hv=HV, split=False, head0=0, hv_total=None):
        g = torch.Generator(device=device)
        g.manual_seed(seed)
        C = 2 * hk * D + hv * D
        self.lens = list(lens)
        self.B, self.N = len(self.lens), int(sum(self.lens))
        self.hk, self.hv, self.C = hk, hv, C
        cu = np.concatenate([[0], np.cumsum(self.lens)]).astype(np.int32)
        self.cu = torch.from_numpy(cu).to(device)
        self.uniform = len(set(self.lens)) == 1
        self.T = self.lens[0] if self.uniform else self.N
        self.x = torch.randn((self.N, C), generator=g, device=device).bfloat16()
        self.w = (torch.randn((C, 4), generator=g, device=device) * 0.5).bfloat16()
        self.z = torch.randn((self.N, hv, D), generator=g, device=device).bfloat16()
        self.gamma = 1 + 0.1 * torch.randn((D,), generator=g, device=device)
        self.a = torch.randn((self.N, hv), generator=g, device=device)
        self.b = torch.randn((self.N, hv), generator=g, device=device)
        self.A_log = torch.rand((hv,), generator=g, device=device) * float(np.log(16.0))
        self.dt_bias = torch.rand((hv,), generator=g, device=device)
        self.y = torch.empty_like(self.x)
        self.o = torch.empty((self.N, hv, D), dtype=torch.float32, device=device)
        self.S = torch.empty((self.B, hv, D, D), dtype=torch.float32, device=device)
        self.out = torch.empty((self.N, hv, D), dtype=torch.bfloat16, device=device)
        self.schedule = self.base = "fused"
        self.ws = None
        self.ws_cap = 0
        self.head0, self.hv_total = head0, hv_total if hv_total is not None else hv
        self.pgs, self.pg_i, self.pg_last = None, 0, None
        if split:
            self.use_schedule("split")

    def use_schedule(self, schedule):
        """fused: gdn_chunked_fwd then the gated norm; split: gdn_chunked_fwd_ws
        (prep + scan on a workspace allocated here, outside any timed region)
        then the norm; split_norm: gdn_chunked_norm_fwd_ws, the norm fused
        into the scan (no separate norm launch); split_gather (head-sharded
        ranks): gdn_chunked_norm_gather_ws, the scan also storing every
        chunk's rows into all ranks' (tokens, Hv_total, 128) outputs over
        NVLink, then gdn_gather_wait -- no separate all-gather.  Two
        PeerGather buffers alternate across layers."""
        import gdn_b200 as G
        self.schedule = self.base = schedule
        if schedule == "split_gather" and self.pgs is None:
            import gdn_shard
            self.pgs = [gdn_shard.PeerGather(self.N, self.hv_total, self.x.device) for _ in range(2)]
        if schedule != "fused" and self.ws is None:
            need = G.chunked_workspace_bytes(self.B, self.T, self.hv, not self.uniform)
            if self.ws_cap:            # bounded workspace: the library runs the call in windows
                need = max(min(need, self.ws_cap), G.chunked_workspace_min_bytes(self.B, self.hv, True))
            self.ws = torch.empty(need, dtype=torch.uint8, device=self.x.device)

    def use_split(self, on):
        self.use_schedule("split" if on else "fused")

    def _cu(self):
        return None if self.uniform else ctypes.c_void_p(self.cu.data_ptr())

    def conv(self, lib, h):
        import gdn_b200 as G
        P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
        rc = lib.gdn_conv1d_fwd(P(self.x), P(self.w), None, None, P(self.y), self._cu(), self.B, self.T, self.C, 4, 0, h)
        if rc:
            raise RuntimeError(lib.gdn_last_error().decode())
        del G

    def chunked(self, lib, h):
        import gdn_b200 as G
        P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
        hk, C = self.hk, self.C
        base = self.y.data_ptr()
        q = ctypes.c_void_p(base)
        k = ctypes.c_void_p(base + hk * D * 2)
        v = ctypes.c_void_p(base + 2 * hk * D * 2)
        if self.base == "split_gather":
            pg = self.pgs[self.pg_i]
            self.pg_i ^= 1
            pg.run(lib, q, k, v, C, C, C, P(self.a), P(self.b), P(self.A_log), P(self.dt_bias), None, P(self.S),
                   P(self.z), self.hv * D, P(self.gamma), 1e-6, self.head0, self._cu(), self.B, self.T, hk,
                   self.hv, G.F_QK_L2NORM, P(self.ws), self.ws.numel(), h)
            self.pg_last = pg
            return
        if self.base == "split_norm":
            rc = lib.gdn_chunked_norm_fwd_ws(q, k, v, C, C, C, P(self.a), P(self.b), P(self.A_log),
                                             P(self.dt_bias), None, P(self.S), P(self.z), self.hv * D,
                                             P(self.gamma), ctypes.c_float(1e-6), P(self.out), self.hv * D, 0,
                                             self._cu(), self.B, self.T, hk, self.hv, D, D,
                                             G.F_QK_L2NORM, P(self.ws), self.ws.numel(), h)
        elif self.base == "split":
            rc = lib.gdn_chunked_fwd_ws(q, k, v, C, C, C, P(self.a), P(self.b), P(self.A_log), P(self.dt_bias),
                                        None, P(self.S), P(self.o), self._cu(), self.B, self.T, hk, self.hv, D, D,
                                        G.F_QK_L2NORM, P(self.ws), self.ws.numel(), h)
        else:
            rc = lib.gdn_chunked_fwd(q, k, v, C, C, C, P(self.a), P(self.b), P(self.A_log), P(self.dt_bias),
                                     None, P(self.S), P(self.o), self._cu(), self.B, self.T, hk, self.hv, D, D,
                                     G.F_QK_L2NORM, h)
        if rc:
            raise RuntimeError(lib.gdn_last_error().decode())

    def norm(self, lib, h):
        if self.base == "split_gather":
            self.pg_last.wait(lib, h)      # norm and gather fused into the scan; wait for every rank
            return
        if self.base == "split_norm":
            return                         # fused into the scan
        P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
        rc = lib.gdn_gated_rmsnorm_fwd(P(self.o), P(self.z), P(self.gamma), P(self.out),
                                       self.N * self.hv, D, ctypes.c_float(1e-6), 0, h)
        if rc:
            raise RuntimeError(lib.gdn_last_error().decode())

    def step(self, lib, h):
        self.conv(lib, h)
        self.chunked(lib, h)
        self.norm(lib, h)

    def flops(self):
        return FLOP_PER_TOKEN_HEAD * self.N * self.hv

    def gather_errors(self):
        """Timeouts recorded by gdn_gather_wait (0 when every wait completed)."""
        return sum(int(pg.err.item()) for pg in self.pgs) if self.pgs else 0

    def close(self):
        """Unmap the PeerGather buffers (collective)."""
        if self.pgs:
            for pg in self.pgs:
                pg.close()
            self.pgs = None


def config4_lengths(seed=4, B=8, lo=16384, hi=65536):
    """B=8 sequences of seeded lengths uniform in [16384, 65536]."""
    rng = np.random.default_rng(seed)
    return [int(x) for x in rng.integers(lo, hi + 1, size=B)]


def time_prefill_layer(X, lib, device, world, steps, warmup, gathered=None):
    """Max-over-ranks ms of one layer (conv -> chunked -> norm, and for N > 1
    the all-gather of the bf16 head outputs) and per-kernel ms (CUDA events)."""
    st = torch.cuda.current_stream(device)
    h = ctypes.c_void_p(st.cuda_stream)

    fused_gather = X.base == "split_gather"

    def layer():
        X.step(lib, h)
        if gathered is not None and not fused_gather:
            torch.distributed.all_gather_into_tensor(gathered, X.out)

    for _ in range(warmup):
        layer()
    torch.cuda.synchronize(device)
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(steps):
        layer()
    e1.record(st)
    torch.cuda.synchronize(device)
    barrier(world)
    ms = max_over_ranks(e0.elapsed_time(e1) / steps, world, device)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    durs = {"conv": [], "chunked": [], "norm": []}
    for _ in range(max(1, min(steps, 3))):
        ev[0].record(st); X.conv(lib, h); ev[1].record(st)
        X.chunked(lib, h); ev[2].record(st)
        X.norm(lib, h); ev[3].record(st)
        torch.cuda.synchronize(device)
        durs["conv"].append(ev[0].elapsed_time(ev[1]))
        durs["chunked"].append(ev[1].elapsed_time(ev[2]))
        durs["norm"].append(ev[2].elapsed_time(ev[3]))
    kms = {k: statistics.mean(v) for k, v in durs.items()}
    if fused_gather:
        torch.cuda.synchronize(device)
        if max_over_ranks(float(X.gather_errors()), world, device):   # every rank raises together
            raise RuntimeError("gdn_gather_wait timed out on a rank: peer gather incomplete")
    if gathered is not None and not fused_gather:
        # the same layer without the all-gather (recurrence throughput alone), max over ranks
        barrier(world)
        e0.record(st)
        for _ in range(steps):
            X.step(lib, h)
        e1.record(st)
        torch.cuda.synchronize(device)
        barrier(world)
        kms["layer_without_gather"] = max_over_ranks(e0.elapsed_time(e1) / steps, world, device)
    return ms, kms


def time_stack(X, lib, device, world, n_layers, gathered=None):
    """Max-over-ranks ms of n_layers layer steps back to back (one pass, after
    the schedule's own warm-up): BASELINE config 4 is a stack of 48 GDN layers
    (the same shapes in every layer, so one set of buffers serves them all)."""
    st = torch.cuda.current_stream(device)
    h = ctypes.c_void_p(st.cuda_stream)
    fused_gather = X.base == "split_gather"
    torch.cuda.synchronize(device)
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(n_layers):
        X.step(lib, h)
        if gathered is not None and not fused_gather:
            torch.distributed.all_gather_into_tensor(gathered, X.out)
    e1.record(st)
    torch.cuda.synchronize(device)
    barrier(world)
    if fused_gather and max_over_ranks(float(X.gather_errors()), world, device):
        raise RuntimeError("gdn_gather_wait timed out on a rank: peer gather incomplete")
    return max_over_ranks(e0.elapsed_time(e1), world, device)


def run_prefill(args, lib, device, world):
    """Configs 3 and 4 on this rank's K-head shard (16/N key, 48/N value heads);
    for N > 1 each layer ends with the NCCL all-gather of the bf16 outputs, or
    (split_gather) the scan itself stores them into every rank's output.
    tokens/s counts the layer's tokens once (all heads) per max-over-ranks second."""
    import gdn_shard
    _, tf_peak, peak_kind = peaks()
    rank = torch.distributed.get_rank() if world > 1 else 0
    shard = gdn_shard.head_shard(rank, world, HK, HV)
    hk, hv = shard.hk, shard.hv
    res = {}
    cases = [("config3", [args.prefill_T])]
    if not args.no_config4:
        cases.append(("config4", config4_lengths()))
    # auto: the two split schedules (the one-kernel fused schedule is 3-4x slower
    # and is timed only when asked for by name)
    schedules = ["split", "split_norm"] if args.prefill_schedule == "auto" else [args.prefill_schedule]
    if world > 1 and args.prefill_schedule == "auto" and not args.no_peer_gather:
        schedules.append("split_gather")
    for name, lens in cases:
        X = PrefillLayer(lens, device, seed=99 + rank, hk=hk, hv=hv, head0=shard.v0, hv_total=HV)
        X.ws_cap = int(args.prefill_ws_gb * 1e9)
        gathered = None
        if world > 1:
            gathered = torch.empty((world,) + tuple(X.out.shape), dtype=torch.bfloat16, device=device)
        steps = max(2, args.steps // 10) if name == "config4" else max(3, args.steps // 5)
        timed = {}
        for sched in schedules:          # every rank times every schedule, in the same order
            X.use_schedule(sched)
            timed[sched] = time_prefill_layer(X, lib, device, world, steps, max(args.warmup, 1)
                                              if name == "config4" else max(args.warmup, 3), gathered)
        best = min(timed, key=lambda k: timed[k][0])
        ms, kms = timed[best]
        stack = None
        if name == "config4" and args.stack_layers > 0:
            X.use_schedule(best)
            ms_stack = time_stack(X, lib, device, world, args.stack_layers, gathered)
            stack = {"layers": args.stack_layers, "ms": round(ms_stack, 3),
                     "tokens_per_s": round(X.N / (ms_stack * 1e-3), 1)}
        X.close()
        achieved = X.flops() / (kms["chunked"] * 1e-3) / 1e12
        kernel = {"fused": "chunked_kernel", "split": "chunk_prep_kernel + chunk_scan_kernel",
                  "split_norm": "chunk_prep_kernel + chunk_scan_kernel<norm>",
                  "split_gather": "chunk_prep_kernel + chunk_scan_kernel<norm, peer stores>"}[best]
        res[name] = {
            "schedule": best,
            "ms_per_layer_by_schedule": {k: round(v[0], 4) for k, v in timed.items()},
            "workspace_bytes": int(X.ws.numel()) if X.ws is not None else 0,
            "workload": (f"{name}: {X.B} seq, {X.N} tokens, conv(C={X.C}, K=4)+SiLU -> chunked C=64 "
                         f"(Hk={hk} Hv={hv} per GPU, S0=0, in-kernel l2norm) -> gated RMSNorm"
                         + ((" -> all-gather fused into the scan (NVLink peer stores)"
                             if best.startswith("split_gather")
                             else " -> NCCL all-gather") if world > 1 else "")),
            ("tokens_per_s" if name == "config3" else "tokens_per_s_per_layer"): round(X.N / (ms * 1e-3), 1),
            "ms_per_layer": round(ms, 4),
            **({"stack_48_layers": stack} if stack else {}),
            **({"tokens_per_s_without_gather": round(X.N / (kms["layer_without_gather"] * 1e-3), 1)}
               if "layer_without_gather" in kms else {}),
            "kernel_ms": {k: round(v, 4) for k, v in kms.items()},
            "roofline": {"bound": "tensor", "kernel": kernel, "achieved": round(achieved, 2),
                         "peak": tf_peak, "unit": "TFLOP/s", "frac": round(achieved / tf_peak, 4),
                         "peak_kind": peak_kind + " bf16 dense (the kernels' MMAs are kind::f16, bf16 and fp16 operands)",
                         "flop_per_launch": X.flops(), "flop_per_token_head": FLOP_PER_TOKEN_HEAD}}
        del X, gathered
        torch.cuda.empty_cache()
    return res


HIDDEN = 5120                      # hidden_size (python/qwen35.py:75)
LAYER_FLOP_PER_TOKEN = 2 * HIDDEN * (2 * HK * D + 2 * HV * D + 2 * HV) + 2 * HV * D * HIDDEN   # in_proj + out_proj


def run_layer(args, device, world):
    """A whole GDN layer (gdn_layer.GDNLayer) on configs 3 and 4: in_proj_qkv
    with the conv in its epilogue and in_proj_z|a|b (this library's tcgen05
    GEMMs) -> chunked recurrence with the norm (and, for N > 1, the head
    all-gather fused into it) -> out_proj on this rank's token slice (tcgen05
    GEMM).  tokens/s counts every token once per max-over-ranks second;
    per-part ms and the GEMMs' TFLOP/s come from CUDA events on each rank."""
    import gdn_layer
    rank = torch.distributed.get_rank() if world > 1 else 0
    w = gdn_layer.random_weights(HIDDEN, HK, HV, device, seed=31)
    layer = gdn_layer.layer_from(w, HK, HV, rank, world)
    res = {}
    cases = [("config3", [args.prefill_T])]
    if not args.no_config4:
        cases.append(("config4", config4_lengths()))
    st = torch.cuda.current_stream(device)
    for name, lens in cases:
        tokens = sum(lens)
        packed = len(set(lens)) > 1
        cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]).astype(np.int32), device=device) if packed else None
        g = torch.Generator(device=device)
        g.manual_seed(77)
        x = torch.randn((tokens, HIDDEN), generator=g, device=device).bfloat16()
        B = len(lens)
        steps = max(2, args.steps // 10) if name == "config4" else max(3, args.steps // 5)
        for _ in range(max(args.warmup, 1)):
            layer.forward_prefill(x, cu_seqlens=cu, B=B)
        torch.cuda.synchronize(device)
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(device) as clk:
            e0.record(st)
            for _ in range(steps):
                y, (lo, hi) = layer.forward_prefill(x, cu_seqlens=cu, B=B)
            e1.record(st)
            torch.cuda.synchronize(device)
        barrier(world)
        ms = max_over_ranks(e0.elapsed_time(e1) / steps, world, device)
        if max_over_ranks(float(layer.gather_errors()), world, device):
            raise RuntimeError("layer gather wait timed out")
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
        ev[0].record(st)
        yc = layer.conv_projection(x, cu_seqlens=cu, B=B)
        ev[1].record(st)
        z, a, b = layer.projections_zab(x)
        ev[2].record(st)
        out = layer.core(yc, z, a, b, cu_seqlens=cu, B=B)
        ev[3].record(st)
        y = layer.out_projection(out[lo:hi].reshape(hi - lo, HV * D))
        ev[4].record(st)
        torch.cuda.synchronize(device)
        parts = {"in_proj_qkv_conv": ev[0].elapsed_time(ev[1]), "in_proj_zab": ev[1].elapsed_time(ev[2]),
                 "gdn_core": ev[2].elapsed_time(ev[3]), "out_proj": ev[3].elapsed_time(ev[4])}
        # the fused kernel computes 128 rows per 125 tokens (the conv halo); counted here as useful work only
        qkv_flop = 2 * tokens * HIDDEN * layer.C
        zab_flop = 2 * tokens * HIDDEN * (layer.hv * D + 2 * layer.hv)
        out_flop = 2 * (hi - lo) * HV * D * HIDDEN
        res[name] = {
            "workload": (f"{name}: {B} seq, {tokens} tokens, hidden {HIDDEN}: in_proj_qkv with the conv + SiLU in "
                         f"its epilogue (gdn_in_proj_conv) and in_proj_z|a|b (gdn_gemm_bf16), both tcgen05 -> "
                         f"chunked + gated norm" + (" + NVLink head gather" if world > 1 else "")
                         + " -> out_proj on the rank's token slice (gdn_gemm_bf16)"),
            "tokens_per_s": round(tokens / (ms * 1e-3), 1), "ms_per_layer": round(ms, 4),
            "part_ms": {k: round(v, 4) for k, v in parts.items()},
            "gemm_tflops": {"in_proj_qkv_conv": round(qkv_flop / (parts["in_proj_qkv_conv"] * 1e-3) / 1e12, 1),
                            "in_proj_zab": round(zab_flop / (parts["in_proj_zab"] * 1e-3) / 1e12, 1),
                            "out_proj": round(out_flop / (parts["out_proj"] * 1e-3) / 1e12, 1)},
            "flop_per_token_projections": LAYER_FLOP_PER_TOKEN, "clocks": clk.summary(),
            "note": "the GEMMs hold the GPU at its power cap, so the latency-bound recurrence kernels run at the "
                    "capped SM clock here (compare prefill.kernel_ms)"}
        del x, yc, z, a, b, out, y
        torch.cuda.empty_cache()
    layer.close()
    del layer, w
    torch.cuda.empty_cache()
    return res


def run_gemm(args, device):
    """The layer's projection GEMMs on their own (rows = tokens, the three
    weight shapes of the 27B GDN layer): this library's tcgen05 kernels
    (gdn_gemm_bf16, gdn_in_proj_conv with the conv + SiLU in its epilogue)
    against cuBLAS through torch.matmul, CUDA events over `steps` calls each
    after `warmup` calls.  For --gemm-only and ncu captures of the GEMM."""
    import gdn_b200 as G
    M, steps, warmup = args.gemm_m, max(args.steps, 1), max(args.warmup, 1)
    g = torch.Generator(device=device).manual_seed(7)

    def timed(fn):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / steps

    res = {"workload": f"M={M} token rows, bf16 in / fp32 accumulate / bf16 out", "shapes": {}}
    for name, N, K in (("in_proj_qkv", 10240, 5120), ("in_proj_zab", 6240, 5120), ("out_proj", 5120, 6144)):
        A = torch.randn((M, K), generator=g, device=device).bfloat16()
        B = (torch.randn((N, K), generator=g, device=device) * K ** -0.5).bfloat16()
        C = torch.empty((M, N), device=device, dtype=torch.bfloat16)
        fl = 2.0 * M * N * K
        ms = timed(lambda: G.gemm_bf16(A, B, C))
        ms_cublas = timed(lambda: torch.matmul(A, B.t(), out=C))
        r = {"ms": round(ms, 4), "tflops": round(fl / ms / 1e9, 1), "cublas_ms": round(ms_cublas, 4),
             "cublas_tflops": round(fl / ms_cublas / 1e9, 1), "vs_cublas": round(ms_cublas / ms, 3)}
        if name == "in_proj_qkv":
            w = (torch.randn((N, 4), generator=g, device=device) * 0.5).bfloat16()
            y = torch.empty_like(C)
            r["with_conv_ms"] = round(timed(lambda: G.in_proj_conv(A.view(1, M, K), B, w, y=y.view(1, M, N))), 4)
        res["shapes"][name] = r
        del A, B, C
    res["device_error"] = G.take_device_error()
    return res


def run_layer_decode(args, device, world, Lp=8):
    """Decode steps through whole layers (gdn_layer.GDNLayer.forward_decode):
    B = args.batch x N sequences per step in seeded random slots of per-layer
    state pools (2B slots) and conv rings, Lp layers sharing one weight set
    (232 MB per layer of projection weights, re-read every layer), replayed
    from a CUDA graph at N = 1 (eager with the NCCL head all-gather at N > 1).
    tokens/s are for a 48-layer stack: B / (48 x the per-layer time)."""
    import gdn_layer
    rank = torch.distributed.get_rank() if world > 1 else 0
    w = gdn_layer.random_weights(HIDDEN, HK, HV, device, seed=41)
    layer = gdn_layer.layer_from(w, HK, HV, rank, world)
    B = args.batch * world                  # per-GPU work fixed: each rank runs every sequence on 1/N of the heads
    n_slots = 2 * B
    g = torch.Generator(device=device)
    g.manual_seed(43)
    pools = [torch.randn((n_slots, layer.hv, D, D), generator=g, device=device) * 0.05 for _ in range(Lp)]
    rings = [torch.zeros((n_slots, 3, layer.C), dtype=torch.bfloat16, device=device) for _ in range(Lp)]
    poss = [torch.zeros(n_slots, dtype=torch.int32, device=device) for _ in range(Lp)]
    slots = torch.randperm(n_slots, generator=g, device=device)[:B].to(torch.int32)
    xs = [torch.randn((B, HIDDEN), generator=g, device=device).bfloat16() for _ in range(Lp)]
    err = torch.zeros(1, dtype=torch.int32, device=device)

    def step():
        for i in range(Lp):
            layer.forward_decode(xs[i], pools[i], slots, rings[i], poss[i], err_flag=err)

    steps = max(args.steps, 10)
    if world == 1:
        ms = time_graph(step, steps, max(args.warmup, 3), device, world) / steps
    else:
        for _ in range(max(args.warmup, 3)):
            step()
        torch.cuda.synchronize(device)
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            step()
        e1.record()
        torch.cuda.synchronize(device)
        barrier(world)
        ms = max_over_ranks(e0.elapsed_time(e1) / steps, world, device)
    torch.cuda.synchronize(device)
    if int(err.item()):
        raise RuntimeError("decode layer recorded a slot error")
    per_layer = ms / Lp
    out = {"workload": f"{Lp} whole layers x B={B} decode (hidden {HIDDEN}; in_proj / out_proj tcgen05 GEMMs, conv ring, "
                       f"state pool in random slots of {n_slots}, gated norm"
                       + (", NCCL head all-gather, token-sliced out_proj" if world > 1 else "") + ")",
           "ms_per_layer": round(per_layer, 4), "tokens_per_s_48_layers": round(B / (48 * per_layer * 1e-3), 1),
           "timing": "CUDA graph replay" if world == 1 else "eager"}
    layer.close()
    del layer, w, pools, rings, xs
    torch.cuda.empty_cache()
    return out


def cpu_prefill_baseline(T=4096, seconds=10.0):
    """The reference's prefill CPU path (chunked_delta, numpy oracle with BLAS
    threads) plus conv and gated norm, whole config-3 layers (at least one)
    for about `seconds`; tokens/s."""
    import gdn_oracle as O
    rng = np.random.default_rng(7)
    C = 2 * HK * D + HV * D
    x = O.bf16_round(rng.standard_normal((1, T, C), dtype=np.float32))
    w = O.bf16_round(rng.standard_normal((C, 4), dtype=np.float32) * np.float32(0.5))
    z = O.bf16_round(rng.standard_normal((1, T, HV, D), dtype=np.float32))
    gamma = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    a = rng.standard_normal((1, T, HV), dtype=np.float32)
    b = rng.standard_normal((1, T, HV), dtype=np.float32)
    A_log = rng.uniform(0.0, np.log(16.0), (HV,)).astype(np.float32)
    dt = rng.uniform(0.0, 1.0, (HV,)).astype(np.float32)
    wts = O.BlockWeights(conv_w=w, A_log=A_log, dt_bias=dt, gamma=gamma)
    n, t0 = 0, time.perf_counter()
    while True:
        O.gdn_block(x, z.reshape(1, T, HV * D), a, b, wts)
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    return {"value": round(n * T / el, 1), "unit": "tokens/s", "cores": os.cpu_count() or 1, "kind": "port",
            "sample": f"{n} x config-3 layer at T={T} (numpy restatement of the reference's CPU prefill: "
                      f"conv, chunked_delta, gated norm; BLAS threads = all cores), {el:.1f} s"}


# ---------------------------------------------------------------------------
# CPU: the reference's per-token recurrence (C oracle, all host threads)
# ---------------------------------------------------------------------------

def cpu_sample(B=1, L=48, seed=5):
    import gdn_oracle as O
    rng = np.random.default_rng(seed)
    layers = []
    for _ in range(L):
        inp = O.synth_decode_inputs(rng, B, 1)
        inp["S"] = inp.pop("S0")
        layers.append(inp)
    return layers


def cpu_step(layers, threads):
    import gdn_oracle as O
    for x in layers:
        O.recurrent_c(x["q"], x["k"], x["v"], x["a"], x["b"], x["A_log"], x["dt_bias"], x["S"],
                      S_out=x["S"], nthreads=threads)


def cpu_baseline(seconds=10.0, B=256, L=4):
    """The C oracle on the headline decode workload's batch (B sequences, all
    48 heads), L layers per step (a bounded sample of the 48), ~`seconds`."""
    threads = os.cpu_count() or 1
    layers = cpu_sample(B, L)
    cpu_step(layers, threads)
    n, t0 = 0, time.perf_counter()
    while True:
        cpu_step(layers, threads)
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    gbs = n * 2 * B * HV * STATE_BYTES * len(layers) / el / 1e9
    return {"value": round(gbs, 2), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{n} steps of {L} of the 48 layers x B={B} decode, C restatement of "
                      f"delta::run_reference (oracle/gdn_oracle.c, OpenMP over heads), {el:.1f} s"}


def run_reference(args, world, rank):
    """The reference arm: the C restatement of delta::run_reference on the
    host cores, at the headline workload's batch (args.batch x N sequences,
    all 48 heads), each step args.ref_layers of the 48 layers."""
    if rank != 0:
        return None
    threads = os.cpu_count() or 1
    B = args.batch * world
    Ls = args.ref_layers
    layers = cpu_sample(B, Ls)
    for _ in range(args.warmup):
        cpu_step(layers, threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_step(layers, threads)
    el = time.perf_counter() - t0
    ms = el * 1e3 / args.steps
    gbs = 2 * B * HV * STATE_BYTES * len(layers) / (ms * 1e-3) / 1e9
    sample = (f"each step: {Ls} of the 48 layers x B={B} of the config-1 decode (the layers are alike, so "
              f"GB/s is that of the 48-layer step), C restatement of delta::run_reference "
              f"(oracle/gdn_oracle.c), {threads} threads")
    return {"metric": METRIC, "impl": "reference", "value": round(gbs, 3), "unit": "GB/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded; BASELINE config-0 distributions)",
            "config": {"workload": f"config1: 48 GDN layers, decode T=1, B={B} (CPU sample: {Ls} layers per step)",
                       "global_batch": B, "seq_len": 1, "layers": 48, "layers_per_step_sampled": Ls,
                       "parallelism": "cpu"},
            "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--batch", type=int, default=256, help="sequences per GPU shard")
    ap.add_argument("--layers", type=int, default=48)
    ap.add_argument("--sweep", default="1,16,64")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--ref-layers", type=int, default=4,
                    help="CPU baseline / reference arm: layers of the 48 run per step (bounded sample)")
    ap.add_argument("--traffic", type=float, default=None,
                    help="dram bytes per launch from an ncu capture, reported as roofline.traffic")
    ap.add_argument("--small", action="store_true", help="ncu-sized case: B=64 (201 MB of state per layer, above L2), 2 layers, no extras")
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--no-verify", action="store_true", help="skip the config-2 verify/accept/rollback chain")
    ap.add_argument("--no-pool", action="store_true", help="skip the state-pool / conv-ring decode comparison")
    ap.add_argument("--no-layer", action="store_true", help="skip the whole-layer prefill (projections included)")
    ap.add_argument("--prefill-T", type=int, default=4096)
    ap.add_argument("--no-config4", action="store_true", help="skip the config-4 layer (B=8 varlen 16K-64K)")
    ap.add_argument("--prefill-schedule", choices=["auto", "fused", "split", "split_norm", "split_gather"],
                    default="auto", help="chunked schedule for configs 3/4; auto times split, split_norm (and "
                    "split_gather at N > 1) and reports the fastest; fused only when named")
    ap.add_argument("--no-peer-gather", action="store_true",
                    help="N > 1: leave out the schedule whose scan stores into every rank's output over NVLink")
    ap.add_argument("--prefill-only", action="store_true", help="only the config-3 prefill (for profiling)")
    ap.add_argument("--stack-layers", type=int, default=48,
                    help="config 4: also time this many layer steps back to back (BASELINE's 48-layer stack; 0 = skip)")
    ap.add_argument("--gemm-only", action="store_true", help="only the projection GEMMs against cuBLAS (--gemm-m rows)")
    ap.add_argument("--gemm-m", type=int, default=65536)
    ap.add_argument("--prefill-ws-gb", type=float, default=0.0,
                    help="cap the split schedule's workspace (GB); smaller than one pass runs in windows")
    args = ap.parse_args()
    if args.small:
        args.batch, args.layers, args.sweep = 64, 2, ""
        args.no_e2e = args.no_cpu_baseline = args.no_prefill = args.no_verify = args.no_pool = args.no_layer = True
    args.warmup = max(args.warmup, 0)

    world, rank, local = dist_env()
    if args.impl == "reference":
        line = run_reference(args, world, rank)
        if line is not None:
            print(json.dumps(line), flush=True)
        return 0
    if world > 1:
        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                             device_id=torch.device("cuda", local))
    try:
        if args.gemm_only:
            device = torch.device("cuda", local)
            torch.cuda.set_device(device)
            line = {"gemm": run_gemm(args, device)}
            if rank == 0:
                print(json.dumps(line), flush=True)
            return 0
        if args.prefill_only:
            import gdn_b200 as G
            device = torch.device("cuda", local)
            torch.cuda.set_device(device)
            line = {"prefill": run_prefill(args, G.lib(), device, world)}
            if not args.no_layer:
                line["layer"] = run_layer(args, device, world)
            if rank == 0:
                print(json.dumps(line), flush=True)
            return 0
        line = run_ours(args, world, rank, local)
        if rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
