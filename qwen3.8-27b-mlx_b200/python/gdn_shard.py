"""Head-parallel sharding of a Gated DeltaNet layer across the GPUs of one box.

Key head i serves value heads i*r .. i*r+r-1 (r = Hv / Hk, repeat_interleave
in python/qwen35.py:592-594), so splitting the 16 key heads into N contiguous
groups splits the 48 value heads into N contiguous groups with no head
shared between ranks.  Everything of the layer between its projections is
per head -- the conv channels of those heads, the gates, the state, the
recurrence and the gated norm -- so a rank runs its shard with no
communication, and the only collective is one all-gather of the normed head
outputs at the layer boundary (before out_proj).

Channel layout of the conv input (cpp/src/model.cpp:592-596): contiguous
[q (Hk*Dk) | k (Hk*Dk) | v (Hv*Dv)].
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List


@dataclass(frozen=True)
class HeadShard:
    rank: int
    world: int
    k0: int          # first key head
    k1: int          # one past the last key head
    v0: int          # first value head
    v1: int

    @property
    def hk(self) -> int:
        return self.k1 - self.k0

    @property
    def hv(self) -> int:
        return self.v1 - self.v0


def head_shard(rank: int, world: int, Hk: int = 16, Hv: int = 48) -> HeadShard:
    """Key heads [Hk*rank/world, Hk*(rank+1)/world) and their value heads."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    if Hk % world or Hv % Hk:
        raise ValueError(f"Hk={Hk} must divide by world={world} and Hv={Hv} by Hk")
    r = Hv // Hk
    k0, k1 = Hk * rank // world, Hk * (rank + 1) // world
    return HeadShard(rank, world, k0, k1, k0 * r, k1 * r)


def conv_channels(sh: HeadShard, Hk: int = 16, Dk: int = 128, Dv: int = 128) -> List[range]:
    """The conv-input channel ranges of this shard, in [q | k | v] order."""
    q = range(sh.k0 * Dk, sh.k1 * Dk)
    k = range(Hk * Dk + sh.k0 * Dk, Hk * Dk + sh.k1 * Dk)
    v = range(2 * Hk * Dk + sh.v0 * Dv, 2 * Hk * Dk + sh.v1 * Dv)
    return [q, k, v]


def channel_index(sh: HeadShard, Hk: int = 16, Dk: int = 128, Dv: int = 128) -> List[int]:
    """Flat list of this shard's conv channels, in the shard's own [q|k|v] order."""
    out: List[int] = []
    for r in conv_channels(sh, Hk, Dk, Dv):
        out.extend(r)
    return out


def assemble(parts, axis_heads: int = -2):
    """Per-rank head blocks (rank order) -> the full head axis.  Works for
    numpy arrays and torch tensors whose head axis is `axis_heads`."""
    first = parts[0]
    if hasattr(first, "cpu") and hasattr(first, "dim"):        # torch
        import torch
        return torch.cat(list(parts), dim=axis_heads)
    import numpy as np
    return np.concatenate(list(parts), axis=axis_heads)


class PeerGather:
    """The all-heads output of a head-sharded layer in every rank's memory,
    filled by the layer's own scan kernels over NVLink
    (gdn_chunked_norm_gather_ws) instead of a separate all-gather.

    ``out`` (tokens, Hv_total, 128) bf16 and a counter array are ordinary
    device tensors of each rank, shared with the other ranks through CUDA IPC
    (gdn_ipc_export / gdn_ipc_open, opened with the local device current so
    peer access from it is enabled), so each rank holds device pointers to
    every rank's copies -- plain peer mappings, no multicast object.  ``run``
    launches this rank's shard writing its heads into all of them; ``wait``
    orders this rank's stream after every rank's call of the same round.
    Two instances alternated across layers keep a consumer from reading a
    buffer that the next layer's call writes."""

    def __init__(self, tokens: int, hv_total: int, device, group=None):
        import ctypes

        import torch
        import torch.distributed as dist

        import gdn_b200 as G

        lib = G.lib()
        grp = group if group is not None else dist.group.WORLD
        self.world = dist.get_world_size(grp)
        self.rank = dist.get_rank(grp)
        if self.world > 8:
            raise ValueError("at most 8 ranks")
        self.out = torch.zeros((tokens, hv_total, 128), dtype=torch.bfloat16, device=device)
        self.flags = torch.zeros(64, dtype=torch.int32, device=device)
        torch.cuda.synchronize(device)

        def export(t):
            h = (ctypes.c_ubyte * 64)()
            off = ctypes.c_size_t(0)
            G.check(lib.gdn_ipc_export(ctypes.c_void_p(t.data_ptr()), h, ctypes.byref(off)))
            return bytes(h), off.value

        mine = (export(self.out), export(self.flags))
        every = [None] * self.world
        dist.all_gather_object(every, mine, group=grp)
        self._bases = []                     # peer mappings opened here, closed by close()
        outs, flags = [], []
        for r, pair in enumerate(every):
            if r == self.rank:
                outs.append(self.out.data_ptr())
                flags.append(self.flags.data_ptr())
                continue
            got = []
            for handle, off in pair:
                base, ptr = ctypes.c_void_p(), ctypes.c_void_p()
                h = (ctypes.c_ubyte * 64).from_buffer_copy(handle)
                G.check(lib.gdn_ipc_open(h, off, ctypes.byref(base), ctypes.byref(ptr)))
                self._bases.append(base.value)
                got.append(ptr.value)
            outs.append(got[0])
            flags.append(got[1])
        self._lib, self._grp = lib, grp
        self.out_ptrs = (ctypes.c_void_p * self.world)(*outs)
        self.flag_ptrs = (ctypes.c_void_p * self.world)(*flags)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        self.round = 0
        torch.cuda.synchronize(device)
        dist.barrier(grp)

    def close(self):
        """Unmap the peers' buffers (collective: every rank calls it after its last wait)."""
        import ctypes

        import torch
        import torch.distributed as dist
        torch.cuda.synchronize(self.out.device)
        dist.barrier(self._grp)
        for base in self._bases:
            self._lib.gdn_ipc_close(ctypes.c_void_p(base))
        self._bases = []
        dist.barrier(self._grp)

    def run(self, lib, q, k, v, q_stride, k_stride, v_stride, a, b, A_log, dt_bias, state_in, state_out, z,
            z_stride, gamma, eps, out_head0, cu_seqlens, B, T, Hk, Hv, flags, workspace, ws_size, stream):
        """gdn_chunked_norm_gather_ws for this rank's heads (pointer arguments as ctypes values)."""
        import ctypes
        rc = lib.gdn_chunked_norm_gather_ws(q, k, v, q_stride, k_stride, v_stride, a, b, A_log, dt_bias, state_in,
                                            state_out, z, z_stride, gamma, ctypes.c_float(eps),
                                            ctypes.cast(self.out_ptrs, ctypes.c_void_p),
                                            ctypes.cast(self.flag_ptrs, ctypes.c_void_p), self.world, self.rank,
                                            self.out.numel(), self.out.stride(0), out_head0, cu_seqlens, B, T, Hk, Hv,
                                            128, 128, flags, workspace, ctypes.c_size_t(ws_size), stream)
        if rc:
            raise RuntimeError(lib.gdn_last_error().decode())
        self.round += 1

    def wait(self, lib, stream):
        """Stream-ordered wait for every rank's call of this round."""
        import ctypes
        rc = lib.gdn_gather_wait(ctypes.c_void_p(self.flags.data_ptr()), self.world, self.round,
                                 ctypes.c_void_p(self.err.data_ptr()), stream)
        if rc:
            raise RuntimeError(lib.gdn_last_error().decode())
