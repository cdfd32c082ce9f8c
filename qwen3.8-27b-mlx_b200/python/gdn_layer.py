"""One Gated DeltaNet layer around the GDN kernels: the host-side mirror of
GatedDeltaNet::operator() (cpp/src/model.cpp:582-641; python/qwen35.py:
575-640) for prefill and for a decode step over a serving batch's state pool,
on this GPU's K-head shard.  Prefill, every step this library's own kernel:

    y   = silu(conv1d(in_proj_qkv(x)))   gdn_in_proj_conv: the tcgen05 GEMM
                                         with the causal conv + SiLU in its
                                         epilogue (the projection stays on chip)
    z | a | b = in_proj_z/a/b(x)         gdn_gemm_bf16, one GEMM over the
                                         stacked weights; a, b as fp32
    out = norm(chunked(q, k, v, a, b), z)
                                         gdn_chunked_norm_fwd_ws, or on several
                                         ranks gdn_chunked_norm_gather_ws +
                                         gdn_gather_wait (every rank ends with
                                         all heads)
    y   = out_proj(out)                  gdn_gemm_bf16 on this rank's token slice

With the heads sharded, in_proj needs no exchange (x is replicated and each
rank produces its own channels); after the fused gather every rank holds all
heads of every token, so each computes out_proj for 1/N of the tokens -- the
result of a row-parallel out_proj followed by a reduce-scatter, with no
further communication.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

import gdn_b200 as G
import gdn_shard

D = 128


class GDNLayer:
    """Weights of one layer for one rank: W_qkv (C_shard, hidden) rows of the
    shard's conv channels [q | k | v], W_z (hv*128, hidden), W_a, W_b (hv,
    hidden), conv_w (C_shard, 4), A_log / dt_bias (hv,), gamma (128,) fp32 and
    the full W_out (hidden, Hv*128).  All bf16 unless noted, on one device."""

    def __init__(self, W_qkv, W_z, W_a, W_b, conv_w, A_log, dt_bias, gamma, W_out, Hk: int, Hv: int,
                 rank: int = 0, world: int = 1, eps: float = 1e-6):
        self.shard = gdn_shard.head_shard(rank, world, Hk, Hv)
        self.rank, self.world = rank, world
        self.Hk, self.Hv = Hk, Hv
        self.W_qkv, self.W_z, self.W_a, self.W_b = W_qkv, W_z, W_a, W_b
        self.conv_w, self.A_log, self.dt_bias, self.gamma, self.W_out = conv_w, A_log, dt_bias, gamma, W_out
        self.eps = eps
        self.hk, self.hv = self.shard.hk, self.shard.hv
        self.C = 2 * self.hk * D + self.hv * D
        if W_qkv.shape[0] != self.C or W_z.shape[0] != self.hv * D or conv_w.shape[0] != self.C:
            raise ValueError("weights do not match the head shard")
        self._ws: Optional[torch.Tensor] = None
        self._gathers = None
        self._g_i = 0
        # in_proj_z / in_proj_a / in_proj_b stacked: one GEMM, a and b as fp32;
        # zero rows pad the stack to a multiple of 8 columns (the GEMM's
        # output granule), e.g. 6 value heads per rank: 768 + 6 + 6 -> 784
        pad = (-(self.hv * D + 2 * self.hv)) % 8
        parts = [W_z, W_a, W_b] + ([W_z.new_zeros((pad, W_z.shape[1]))] if pad else [])
        self.W_zab = torch.cat(parts, 0).contiguous()

    def token_slice(self, tokens: int):
        """The rows of the layer output this rank computes."""
        per = (tokens + self.world - 1) // self.world
        lo = min(self.rank * per, tokens)
        return lo, min(lo + per, tokens)

    def _workspace(self, B, T, packed, device):
        need = G.chunked_workspace_bytes(B, T, self.hv, packed)
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(need, dtype=torch.uint8, device=device)
        return self._ws

    def projections_zab(self, x):
        """in_proj_z, in_proj_a, in_proj_b of x (tokens, hidden) bf16: z
        (tokens, hv*128) bf16, a and b (tokens, hv) fp32 (one GEMM)."""
        z, ab = G.gemm_bf16(x, self.W_zab, n_f32=self.hv * D, f32_width=self.hv)
        return z, ab[0], ab[1]

    def projections(self, x):
        """in_proj_qkv (without the conv), in_proj_z, in_proj_a, in_proj_b of
        x (tokens, hidden) bf16."""
        qkv = G.gemm_bf16(x, self.W_qkv)
        z, a, b = self.projections_zab(x)
        return qkv, z, a, b

    def conv_projection(self, x, cu_seqlens=None, B: int = 1):
        """silu(conv1d(in_proj_qkv(x))) in one kernel: (tokens, C) bf16."""
        if cu_seqlens is not None:
            y, _ = G.in_proj_conv(x, self.W_qkv, self.conv_w, cu_seqlens=cu_seqlens)
            return y
        y, _ = G.in_proj_conv(x.view(B, x.shape[0] // B, x.shape[1]), self.W_qkv, self.conv_w)
        return y.view(x.shape[0], self.C)

    def core(self, y, z, a, b, cu_seqlens=None, B: int = 1, state_out=None):
        """The chunked recurrence with the gated norm (and, on several ranks,
        the head all-gather fused into it) on the conv output y (tokens, C).
        Returns (tokens, Hv, 128) bf16."""
        tokens = y.shape[0]
        dev = y.device
        packed = cu_seqlens is not None
        T = tokens if packed else tokens // B
        hk, hv, C = self.hk, self.hv, self.C
        P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
        base = y.data_ptr()
        q = ctypes.c_void_p(base)
        k = ctypes.c_void_p(base + hk * D * 2)
        v = ctypes.c_void_p(base + 2 * hk * D * 2)
        ws = self._workspace(B, T, packed, dev)
        st = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
        lib = G.lib()
        zc = z.contiguous()
        cu = P(cu_seqlens) if packed else None
        if self.world == 1:
            out = torch.empty((tokens, self.Hv, D), dtype=torch.bfloat16, device=dev)
            G.check(lib.gdn_chunked_norm_fwd_ws(q, k, v, C, C, C, P(a), P(b), P(self.A_log), P(self.dt_bias), None,
                                                P(state_out) if state_out is not None else None, P(zc), hv * D,
                                                P(self.gamma), ctypes.c_float(self.eps), P(out), self.Hv * D, 0,
                                                cu, B, T, hk, hv, D, D, G.F_QK_L2NORM, P(ws), ws.numel(), st))
            return out
        if self._gathers is None or self._gathers[0].out.shape[0] != tokens:
            self._gathers = [gdn_shard.PeerGather(tokens, self.Hv, dev) for _ in range(2)]
        pg = self._gathers[self._g_i]
        self._g_i ^= 1
        pg.run(lib, q, k, v, C, C, C, P(a), P(b), P(self.A_log), P(self.dt_bias), None,
               P(state_out) if state_out is not None else None, P(zc), hv * D, P(self.gamma), self.eps,
               self.shard.v0, cu, B, T, hk, hv, G.F_QK_L2NORM, P(ws), ws.numel(), st)
        pg.wait(lib, st)
        return pg.out

    def forward_prefill(self, x, cu_seqlens=None, B: int = 1, state_out=None):
        """The layer on x (tokens, hidden) bf16: returns (y rows of this
        rank's token slice (rows, hidden) bf16, (lo, hi))."""
        y = self.conv_projection(x, cu_seqlens, B)
        z, a, b = self.projections_zab(x)
        out = self.core(y, z, a, b, cu_seqlens, B, state_out)
        lo, hi = self.token_slice(x.shape[0])
        return self.out_projection(out[lo:hi].reshape(hi - lo, self.Hv * D)), (lo, hi)

    def out_projection(self, o):
        """out_proj of (rows, Hv*128) bf16 normed head outputs."""
        if o.shape[0] == 0:
            return torch.empty((0, self.W_out.shape[0]), dtype=torch.bfloat16, device=o.device)
        return G.gemm_bf16(o, self.W_out)

    def forward_decode(self, x, pool, slots, ring, ring_pos, err_flag=None):
        """One decode step of B sequences (x (B, hidden) bf16, one token each)
        whose states live in slots of a pool (pool (n_slots, hv, 128, 128)
        fp32, slots (B,) int32) and whose conv windows are rings (ring
        (n_slots, 3, C_shard) bf16, ring_pos (n_slots,) int32): in_proj ->
        conv over the ring (+ its one-row append) -> the recurrence on the
        pool, written back -> gated norm -> out_proj.  On several ranks the
        normed heads (6144 x 2 bytes per token) are all-gathered by NCCL and
        each rank projects its token slice.  Returns (y rows, (lo, hi))."""
        B = x.shape[0]
        hk, hv = self.hk, self.hv
        qkv, z, a, b = self.projections(x)
        qkv3 = qkv.view(B, 1, self.C)
        y = G.conv1d_fwd_pool(qkv3, self.conv_w, ring, ring_pos, slots, err_flag=err_flag)
        G.conv_ring_append(qkv3, ring, ring_pos, slots, err_flag=err_flag)
        # the decode kernel reads (B, T, heads, 128) rows: contiguous copies of the conv output's q | k | v
        q = y[..., :hk * D].reshape(B, 1, hk, D).contiguous()
        k = y[..., hk * D:2 * hk * D].reshape(B, 1, hk, D).contiguous()
        v = y[..., 2 * hk * D:].reshape(B, 1, hv, D).contiguous()
        o, _ = G.recurrent_fwd_pool(q, k, v, a.view(B, 1, hv), b.view(B, 1, hv), self.A_log, self.dt_bias, pool,
                                    slots, G.POOL_FINAL, err_flag=err_flag, l2norm=True)
        normed = G.gated_rmsnorm_fwd(o.view(B * hv, D), z.view(B * hv, D), self.gamma, eps=self.eps).view(B, hv * D)
        if self.world > 1:
            import torch.distributed as dist
            parts = torch.empty((self.world, B, hv * D), dtype=normed.dtype, device=normed.device)
            dist.all_gather_into_tensor(parts, normed)
            normed = parts.permute(1, 0, 2).reshape(B, self.Hv * D)
        lo, hi = self.token_slice(B)
        return self.out_projection(normed[lo:hi].contiguous()), (lo, hi)

    def gather_errors(self) -> int:
        return sum(int(pg.err.item()) for pg in self._gathers) if self._gathers else 0

    def close(self):
        """Release the peer mappings (collective on several ranks)."""
        if self._gathers:
            for pg in self._gathers:
                pg.close()
            self._gathers = None


def shard_weights(full: dict, rank: int, world: int, Hk: int, Hv: int) -> dict:
    """This rank's rows of a layer's full weights (dict with W_qkv, W_z, W_a,
    W_b, conv_w, A_log, dt_bias, gamma, W_out): its conv channels, its value
    heads; gamma and W_out whole."""
    sh = gdn_shard.head_shard(rank, world, Hk, Hv)
    idx = torch.tensor(gdn_shard.channel_index(sh, Hk), device=full["W_qkv"].device)
    vrows = slice(sh.v0 * D, sh.v1 * D)
    return {"W_qkv": full["W_qkv"][idx].contiguous(), "W_z": full["W_z"][vrows].contiguous(),
            "W_a": full["W_a"][sh.v0:sh.v1].contiguous(), "W_b": full["W_b"][sh.v0:sh.v1].contiguous(),
            "conv_w": full["conv_w"][idx].contiguous(), "A_log": full["A_log"][sh.v0:sh.v1].contiguous(),
            "dt_bias": full["dt_bias"][sh.v0:sh.v1].contiguous(), "gamma": full["gamma"], "W_out": full["W_out"]}


def random_weights(hidden: int, Hk: int, Hv: int, device, seed: int = 0) -> dict:
    """Seeded full weights of one layer with the reference's shapes
    (cpp/src/model.cpp:157-177): bf16 projections scaled 1/sqrt(fan-in),
    conv N(0, 0.5), A_log U(0, ln 16), dt_bias U(0, 1), gamma N(1, 0.1)."""
    import math
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    C = 2 * Hk * D + Hv * D

    def lin(o, i):
        return (torch.randn((o, i), generator=g, device=device) / math.sqrt(i)).bfloat16()
    return {"W_qkv": lin(C, hidden), "W_z": lin(Hv * D, hidden), "W_a": lin(Hv, hidden), "W_b": lin(Hv, hidden),
            "conv_w": (torch.randn((C, 4), generator=g, device=device) * 0.5).bfloat16(),
            "A_log": torch.rand((Hv,), generator=g, device=device) * math.log(16.0),
            "dt_bias": torch.rand((Hv,), generator=g, device=device),
            "gamma": 1 + 0.1 * torch.randn((D,), generator=g, device=device),
            "W_out": lin(hidden, Hv * D)}


def layer_from(weights: dict, Hk: int, Hv: int, rank: int = 0, world: int = 1) -> GDNLayer:
    w = shard_weights(weights, rank, world, Hk, Hv) if world > 1 else weights
    return GDNLayer(w["W_qkv"], w["W_z"], w["W_a"], w["W_b"], w["conv_w"], w["A_log"], w["dt_bias"], w["gamma"],
                    w["W_out"], Hk, Hv, rank, world)
