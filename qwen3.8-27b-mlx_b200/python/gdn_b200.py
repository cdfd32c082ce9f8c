"""ctypes binding of the GDN C ABI (include/gdn_b200.h) for torch tensors.

This is the host layer a Python caller uses: it checks dtypes, shapes,
devices and contiguity of torch tensors, then passes raw device pointers and
the current CUDA stream to ``libgdn_b200.so``.  Errors come back as
``GdnError`` carrying the library's status code and message.  There is no
fallback: if the library is missing or the tensors are not on a CUDA device,
the call raises.
"""
from __future__ import annotations

import ctypes
import os
from typing import Optional

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
LIB_PATH = os.environ.get("GDN_B200_LIB", os.path.join(PKG, "libgdn_b200.so"))

GDN_OK = 0
GDN_ERR_NULL = -1
GDN_ERR_SHAPE = -2
GDN_ERR_ALIGN = -3
GDN_ERR_FLAGS = -4
GDN_ERR_ALIAS = -5
GDN_ERR_CUDA = -6
GDN_ERR_RANGE = -7

F_QKV_F32 = 0x1
F_O_BF16 = 0x2
F_GATES_DIRECT = 0x4
F_QK_L2NORM = 0x8
F_OVERLAP_PREV = 0x10
F_CONV_BF16_OPS = 0x100
F_CONV_NO_SILU = 0x200
F_NORM_IN_BF16 = 0x400
F_NORM_OUT_F32 = 0x800

D = 128

_vp = ctypes.c_void_p
_i = ctypes.c_int
_u = ctypes.c_uint

# name -> argtypes; every symbol include/gdn_b200.h declares
SIGNATURES = {
    "gdn_last_error": [],
    "gdn_version": [],
    "gdn_take_device_error": [_vp, _vp],
    "gdn_recurrent_fwd": [_vp] * 11 + [_i] * 6 + [_u, _vp],
    "gdn_recurrent_fwd_from_ckpt": [_vp] * 10 + [_i] + [_vp] * 4 + [_i] * 6 + [_u, _vp],
    "gdn_recurrent_fwd_pool": [_vp] * 9 + [_i] + [_vp] * 2 + [_i, _i] + [_vp] * 3 + [_i] * 6 + [_u, _vp],
    "gdn_delta_run": [_vp] * 9 + [_i] * 5 + [_vp],
    "gdn_tc05_selftest": [_vp] * 3 + [_i] * 3 + [_vp, _vp],
    "gdn_tc05_pair_selftest": [_vp] * 3 + [_i] * 2 + [_vp, _vp],
    "gdn_conv1d_fwd": [_vp] * 6 + [_i] * 4 + [_u, _vp],
    "gdn_chunked_fwd": [_vp] * 3 + [ctypes.c_longlong] * 3 + [_vp] * 8 + [_i] * 6 + [_u, _vp],
    "gdn_chunked_workspace_bytes": [_i] * 4,
    "gdn_chunked_workspace_min_bytes": [_i] * 3,
    "gdn_chunked_fwd_static": [_vp] * 3 + [ctypes.c_longlong] * 3 + [_vp] * 8 + [_i] * 6 + [_u, _vp],
    "gdn_chunked_norm_gather_ws": [_vp] * 3 + [ctypes.c_longlong] * 3 + [_vp] * 7 + [ctypes.c_longlong, _vp,
                                  ctypes.c_float, _vp, _vp, _i, _i, ctypes.c_longlong, ctypes.c_longlong, _i, _vp]
                                  + [_i] * 6 + [_u, _vp, ctypes.c_size_t, _vp],
    "gdn_gather_wait": [_vp, _i, _u, _vp, _vp],
    "gdn_gather_wait_timeout": [_vp, _i, _u, _u, _vp, _vp],
    "gdn_ipc_export": [_vp, _vp, _vp],
    "gdn_ipc_open": [_vp, ctypes.c_size_t, _vp, _vp],
    "gdn_ipc_close": [_vp],
    "gdn_spec_verify": [_vp] * 5 + [_i, _i, ctypes.c_longlong] + [_vp] * 5,
    "gdn_chunked_norm_fwd_ws": [_vp] * 3 + [ctypes.c_longlong] * 3 + [_vp] * 7 + [ctypes.c_longlong, _vp,
                               ctypes.c_float, _vp, ctypes.c_longlong, _i, _vp] + [_i] * 6
                               + [_u, _vp, ctypes.c_size_t, _vp],
    "gdn_chunked_fwd_ws": [_vp] * 3 + [ctypes.c_longlong] * 3 + [_vp] * 8 + [_i] * 6
                          + [_u, _vp, ctypes.c_size_t, _vp],
    "gdn_conv_commit": [_vp] * 5 + [_i] * 4 + [_vp],
    "gdn_conv1d_fwd_pool": [_vp] * 5 + [_i] + [_vp] * 2 + [_i] * 4 + [_u, _vp, _vp],
    "gdn_conv_ring_append": [_vp] * 4 + [_i] + [_vp] * 2 + [_i] * 4 + [_vp, _vp],
    "gdn_gated_rmsnorm_fwd": [_vp] * 4 + [ctypes.c_longlong, _i, ctypes.c_float, _u, _vp],
    "gdn_gemm_bf16": [_vp] * 4 + [_i] * 3 + [ctypes.c_longlong] * 4 + [_i, _vp],
    "gdn_in_proj_conv": [_vp] * 7 + [_i] * 4 + [ctypes.c_longlong] * 3 + [_vp],
}

# return types other than int
RESTYPES = {"gdn_last_error": ctypes.c_char_p, "gdn_chunked_workspace_bytes": ctypes.c_size_t,
            "gdn_chunked_workspace_min_bytes": ctypes.c_size_t}

_lib = None


class GdnError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"gdn error {code}: {msg}")
        self.code = code


def lib():
    """Load libgdn_b200.so (once).  Raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is not built; run __graft_entry__.build()")
        L = ctypes.CDLL(LIB_PATH)
        for name, args in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = RESTYPES.get(name, ctypes.c_int)
        _lib = L
    return _lib


def check(rc: int):
    if rc != GDN_OK:
        raise GdnError(rc, lib().gdn_last_error().decode())


def take_device_error(device=None) -> int:
    """Synchronise the current stream and return (and clear) the device's
    kernel error word (0 = no bounded wait timed out)."""
    dev = device or torch.device("cuda", torch.cuda.current_device())
    out = ctypes.c_int(0)
    check(lib().gdn_take_device_error(stream_ptr(dev), ctypes.byref(out)))
    return out.value


def ptr(t: Optional[torch.Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_ptr(device: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _dev(*ts):
    dev = None
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError("GDN tensors must live on a CUDA device")
        if not t.is_contiguous():
            raise ValueError("GDN tensors must be contiguous")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError("GDN tensors must share one device")
    return dev


def recurrent_fwd(q, k, v, a, b, A_log=None, dt_bias=None, state_in=None, state_out=None,
                  o=None, ckpt=None, *, gates_direct=False, l2norm=False,
                  o_dtype=torch.float32, overlap_prev=False):
    """One decode / verify step through ``gdn_recurrent_fwd``.

    q, k (B,T,Hk,128) and v (B,T,Hv,128), all bf16 or all fp32; a, b (B,T,Hv)
    fp32; A_log, dt_bias (Hv,) fp32; state_in (B,Hv,128,128) fp32 or None.
    Missing outputs are allocated.  Returns (o, state_out, ckpt).
    """
    B, T, Hk, Dk = q.shape
    Hv = v.shape[2]
    flags = 0
    if q.dtype == torch.float32:
        flags |= F_QKV_F32
    elif q.dtype != torch.bfloat16:
        raise ValueError("q, k, v must be bf16 or fp32")
    if not (k.dtype == v.dtype == q.dtype):
        raise ValueError("q, k, v must share a dtype")
    if gates_direct:
        flags |= F_GATES_DIRECT
    if l2norm:
        flags |= F_QK_L2NORM
    if o_dtype == torch.bfloat16:
        flags |= F_O_BF16
    if overlap_prev:
        flags |= F_OVERLAP_PREV
    dev = _dev(q, k, v, a, b, A_log, dt_bias, state_in, state_out, o, ckpt)
    if o is None:
        o = torch.empty((B, T, Hv, v.shape[-1]), dtype=o_dtype, device=dev)
    if state_out is None and ckpt is None:
        state_out = torch.empty((B, Hv, v.shape[-1], Dk), dtype=torch.float32, device=dev)
    check(lib().gdn_recurrent_fwd(ptr(q), ptr(k), ptr(v), ptr(a), ptr(b), ptr(A_log), ptr(dt_bias),
                                  ptr(state_in), ptr(state_out), ptr(o), ptr(ckpt),
                                  B, T, Hk, Hv, Dk, v.shape[-1], flags, stream_ptr(dev)))
    return o, state_out, ckpt


def recurrent_fwd_from_ckpt(q, k, v, a, b, A_log, dt_bias, state_prev, ckpt_src, commit_n,
                            state_out=None, o=None, ckpt=None, err_flag=None, *,
                            l2norm=False, o_dtype=torch.float32):
    """Decode / verify step whose start state is the committed checkpoint
    ``commit_n[b]`` of the previous verify block (``gdn_recurrent_fwd_from_ckpt``)."""
    B, T, Hk, Dk = q.shape
    Hv = v.shape[2]
    flags = (F_QKV_F32 if q.dtype == torch.float32 else 0) | (F_QK_L2NORM if l2norm else 0)
    if o_dtype == torch.bfloat16:
        flags |= F_O_BF16
    if commit_n.dtype != torch.int32:
        raise ValueError("commit_n must be int32")
    dev = _dev(q, k, v, a, b, A_log, dt_bias, state_prev, ckpt_src, commit_n, state_out, o, ckpt, err_flag)
    if o is None:
        o = torch.empty((B, T, Hv, D), dtype=o_dtype, device=dev)
    if state_out is None and ckpt is None:
        state_out = torch.empty((B, Hv, D, D), dtype=torch.float32, device=dev)
    Tsrc = ckpt_src.shape[2]
    check(lib().gdn_recurrent_fwd_from_ckpt(ptr(q), ptr(k), ptr(v), ptr(a), ptr(b), ptr(A_log), ptr(dt_bias),
                                            ptr(state_prev), ptr(ckpt_src), ptr(commit_n), Tsrc,
                                            ptr(state_out), ptr(o), ptr(ckpt), ptr(err_flag),
                                            B, T, Hk, Hv, Dk, D, flags, stream_ptr(dev)))
    return o, state_out, ckpt


POOL_KEEP, POOL_FINAL, POOL_START = 0, 1, 2


def recurrent_fwd_pool(q, k, v, a, b, A_log, dt_bias, pool, slots, pool_write=POOL_FINAL, ckpt_src=None,
                       commit_n=None, o=None, ckpt=None, err_flag=None, *, l2norm=False, o_dtype=torch.float32):
    """Decode / verify step over a state pool (``gdn_recurrent_fwd_pool``):
    sequence b uses slot ``slots[b]`` of ``pool`` (n_slots, Hv, 128, 128)
    fp32; start from the slot or (with ckpt_src, commit_n) a committed
    checkpoint; ``pool_write`` POOL_FINAL / POOL_START / POOL_KEEP.
    Returns (o, ckpt)."""
    B, T, Hk, Dk = q.shape
    Hv = v.shape[2]
    flags = (F_QKV_F32 if q.dtype == torch.float32 else 0) | (F_QK_L2NORM if l2norm else 0)
    if o_dtype == torch.bfloat16:
        flags |= F_O_BF16
    if slots.dtype != torch.int32 or (commit_n is not None and commit_n.dtype != torch.int32):
        raise ValueError("slots and commit_n must be int32")
    dev = _dev(q, k, v, a, b, A_log, dt_bias, pool, slots, ckpt_src, commit_n, o, ckpt, err_flag)
    if o is None:
        o = torch.empty((B, T, Hv, D), dtype=o_dtype, device=dev)
    Tsrc = ckpt_src.shape[2] if ckpt_src is not None else 0
    check(lib().gdn_recurrent_fwd_pool(ptr(q), ptr(k), ptr(v), ptr(a), ptr(b), ptr(A_log), ptr(dt_bias),
                                       ptr(pool), ptr(slots), pool.shape[0], ptr(ckpt_src), ptr(commit_n), Tsrc,
                                       pool_write, ptr(o), ptr(ckpt), ptr(err_flag),
                                       B, T, Hk, Hv, Dk, D, flags, stream_ptr(dev)))
    return o, ckpt


def conv1d_fwd_pool(x, w, ring, ring_pos, slots, y=None, cu_seqlens=None, err_flag=None, *, bf16_ops=False,
                    silu=True):
    """gdn_conv1d_fwd with each sequence's window read from its slot of a
    ring pool (ring (n_slots, 3, C) bf16, ring_pos (n_slots,) int32).  Returns y."""
    if cu_seqlens is not None:
        T, C = x.shape
        B = cu_seqlens.numel() - 1
    else:
        B, T, C = x.shape
    dev = _dev(x, w, ring, ring_pos, slots, y, cu_seqlens, err_flag)
    if y is None:
        y = torch.empty_like(x)
    flags = (F_CONV_BF16_OPS if bf16_ops else 0) | (0 if silu else F_CONV_NO_SILU)
    check(lib().gdn_conv1d_fwd_pool(ptr(x), ptr(w), ptr(ring), ptr(ring_pos), ptr(slots), ring.shape[0], ptr(y),
                                    ptr(cu_seqlens), B, T, C, w.shape[1], flags, ptr(err_flag), stream_ptr(dev)))
    return y


def conv_ring_append(x, ring, ring_pos, slots, counts=None, cu_seqlens=None, err_flag=None):
    """Move the first counts[b] (default: all) tokens of each sequence into its ring slot."""
    if cu_seqlens is not None:
        T, C = x.shape
        B = cu_seqlens.numel() - 1
    else:
        B, T, C = x.shape
    dev = _dev(x, ring, ring_pos, slots, counts, cu_seqlens, err_flag)
    check(lib().gdn_conv_ring_append(ptr(x), ptr(ring), ptr(ring_pos), ptr(slots), ring.shape[0], ptr(counts),
                                     ptr(cu_seqlens), B, T, C, 4, ptr(err_flag), stream_ptr(dev)))


def tc05_selftest(A, B, *, bf16=False, negate_a=False, a_in_tmem=False, a_mn=False, b_mn=False, d_col=0,
                  fp16=False):
    """D = op(A) @ B.T on one CTA through tcgen05 (diagnostic).  A (128,K),
    B (N,K) fp32 CUDA tensors, N <= 256; operands rounded to bf16, fp16 or
    (neither) tf32; the accumulator starts at TMEM column d_col (0, 64, 128
    or 192).  Returns (D, status)."""
    dev = _dev(A, B)
    N, K = B.shape
    if d_col not in (0, 64, 128, 192):
        raise ValueError("d_col must be 0, 64, 128 or 192")
    D = torch.empty((128, N), dtype=torch.float32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    mode = (1 if bf16 or fp16 else 0) | (256 if fp16 else 0) | (2 if negate_a else 0) | (4 if a_in_tmem else 0) | \
        (8 if a_mn else 0) | \
        (16 if b_mn else 0) | (32 if d_col & 64 else 0) | (64 if d_col & 128 else 0)
    check(lib().gdn_tc05_selftest(ptr(A), ptr(B), ptr(D), N, K, mode, ptr(status), stream_ptr(dev)))
    return D, status


def tc05_pair_selftest(A, B):
    """A @ B.T on a CTA pair through tcgen05 cta_group::2, M = 128 (diagnostic).
    A (128,K), B (N,K) fp32 CUDA tensors holding tf32 values.  Returns
    (raw, status): raw (2, 128, N/2) is each CTA's tensor memory, lane by
    lane."""
    dev = _dev(A, B)
    N, K = B.shape
    raw = torch.full((2, 128, N // 2), float("nan"), dtype=torch.float32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    check(lib().gdn_tc05_pair_selftest(ptr(A), ptr(B), ptr(raw), N, K, ptr(status), stream_ptr(dev)))
    return raw, status


def chunked_norm_fwd(q, k, v, a, b, A_log, dt_bias, z, gamma, state_in=None, state_out=None, out=None,
                     cu_seqlens=None, *, eps=1e-6, l2norm=True, out_head0=0, workspace=None):
    """Chunked prefill with the gated RMSNorm fused in (gdn_chunked_norm_fwd_ws).
    q, k, v as chunked_fwd; z (..., Hv, 128) bf16 with contiguous heads;
    gamma (128,) fp32.  out: bf16 (..., H_out, 128) with H_out >= out_head0 +
    Hv (allocated as (..., Hv, 128) when None).  Returns (out, state_out)."""
    Hk, Hv = q.shape[-2], v.shape[-2]
    for t in (q, k, v, z):
        if t.dtype != torch.bfloat16 or t.stride(-1) != 1 or t.stride(-2) != 128:
            raise ValueError("q, k, v, z must be bf16 with contiguous 128-wide heads")
    if cu_seqlens is not None:
        B, T = cu_seqlens.numel() - 1, q.shape[0]
        lead = (T,)
    else:
        B, T = q.shape[0], q.shape[1]
        lead = (B, T)
        if B > 1 and T > 0 and (q.stride(0) != T * q.stride(-3) or k.stride(0) != T * k.stride(-3)
                                or v.stride(0) != T * v.stride(-3) or z.stride(0) != T * z.stride(-3)):
            raise ValueError("batch rows must follow each other (token-major storage)")
    dev = _dev(a, b, A_log, dt_bias, z, gamma, state_in, state_out, out, cu_seqlens)
    if out is None:
        out = torch.empty(lead + (Hv, D), dtype=torch.bfloat16, device=dev)
    if out.dtype != torch.bfloat16 or out.stride(-1) != 1 or out.stride(-2) != 128:
        raise ValueError("out must be bf16 with contiguous 128-wide heads")
    if state_out is None:
        state_out = torch.empty((B, Hv, D, D), dtype=torch.float32, device=dev)
    need = chunked_workspace_bytes(B, T, Hv, cu_seqlens is not None)
    if workspace is None:
        workspace = torch.empty(need, dtype=torch.uint8, device=dev)
    check(lib().gdn_chunked_norm_fwd_ws(ptr(q), ptr(k), ptr(v), q.stride(-3), k.stride(-3), v.stride(-3), ptr(a),
                                        ptr(b), ptr(A_log), ptr(dt_bias), ptr(state_in), ptr(state_out), ptr(z),
                                        z.stride(-3), ptr(gamma), eps, ptr(out), out.stride(-3), out_head0,
                                        ptr(cu_seqlens), B, T, Hk, Hv, D, D,
                                        F_QK_L2NORM if l2norm else 0,
                                        ptr(workspace), workspace.numel(), stream_ptr(dev)))
    return out, state_out


def spec_verify(p, q, draft, u_accept, u_sample, err_flag=None):
    """On-device acceptance of a speculative block (gdn_spec_verify).  p
    (B, k+1, V), q (B, k, V) fp32; draft (B, k) int32; u_accept (B, k),
    u_sample (B,) fp32.  Returns (accept_len, commit_n, token), int32 (B,)."""
    B, k1, V = p.shape
    k = k1 - 1
    if q.shape != (B, k, V) or draft.shape != (B, k) or u_accept.shape != (B, k) or u_sample.shape != (B,):
        raise ValueError("shapes: p (B,k+1,V), q (B,k,V), draft (B,k), u_accept (B,k), u_sample (B,)")
    if draft.dtype != torch.int32:
        raise ValueError("draft must be int32")
    dev = _dev(p, q, draft, u_accept, u_sample, err_flag)
    outs = [torch.empty(B, dtype=torch.int32, device=dev) for _ in range(3)]
    if err_flag is None:
        err_flag = torch.zeros(1, dtype=torch.int32, device=dev)
    check(lib().gdn_spec_verify(ptr(p), ptr(q), ptr(draft), ptr(u_accept), ptr(u_sample), B, k, V,
                                ptr(outs[0]), ptr(outs[1]), ptr(outs[2]), ptr(err_flag), stream_ptr(dev)))
    return tuple(outs)


def conv1d_fwd(x, w, state_in=None, state_out=None, y=None, cu_seqlens=None, *, bf16_ops=False, silu=True):
    """Causal depthwise conv1d + SiLU (gdn_conv1d_fwd).  x (B,T,C) bf16, or
    packed (T,C) with cu_seqlens (B+1) int32; w (C,4) bf16; state_in
    (B,3,C) bf16 or None.  Returns (y, state_out)."""
    if cu_seqlens is not None:
        T, C = x.shape
        B = cu_seqlens.numel() - 1
        if cu_seqlens.dtype != torch.int32:
            raise ValueError("cu_seqlens must be int32")
    else:
        B, T, C = x.shape
    dev = _dev(x, w, state_in, state_out, y, cu_seqlens)
    if y is None:
        y = torch.empty_like(x)
    flags = (F_CONV_BF16_OPS if bf16_ops else 0) | (0 if silu else F_CONV_NO_SILU)
    check(lib().gdn_conv1d_fwd(ptr(x), ptr(w), ptr(state_in), ptr(state_out), ptr(y), ptr(cu_seqlens),
                               B, T, C, w.shape[1], flags, stream_ptr(dev)))
    return y, state_out


def gemm_bf16(A, B, C=None, n_f32=None, C32=None, f32_width=None):
    """C = A B^T on the tensor cores (gdn_gemm_bf16): A (M, K), B (N, K) bf16,
    fp32 accumulation, C (M, N) bf16.  With n_f32 set, columns n_f32 .. N-1
    go to C32 as fp32 (the bf16-rounded values), as a stack of (M, f32_width)
    matrices (default one (M, N - n_f32) matrix), and C has n_f32 columns.
    Returns C, or (C, C32) with n_f32."""
    M, K = A.shape
    N = B.shape[0]
    if B.shape[1] != K:
        raise ValueError("A and B must share K")
    dev = _dev(A, B, C, C32)
    nc = N if n_f32 is None else n_f32
    if C is None:
        C = torch.empty((M, nc), dtype=torch.bfloat16, device=dev)
    ld32 = 0
    if n_f32 is not None:
        ld32 = f32_width or (N - n_f32)
        nblk = -(-(N - n_f32) // ld32)
        if C32 is None:
            C32 = torch.empty((nblk, M, ld32) if f32_width else (M, ld32), dtype=torch.float32, device=dev)
    check(lib().gdn_gemm_bf16(ptr(A), ptr(B), ptr(C), ptr(C32), M, N, K, K, K, C.shape[1], ld32,
                              0 if n_f32 is None else n_f32, stream_ptr(dev)))
    return C if n_f32 is None else (C, C32)


def in_proj_conv(x, W, conv_w, state_in=None, state_out=None, y=None, cu_seqlens=None, B=None):
    """y = silu(conv1d(x W^T)) with the projection and the causal conv in one
    tensor-core kernel (gdn_in_proj_conv).  x (tokens, K) bf16 packed with
    cu_seqlens (B+1) int32, or (B, T, K); W (C, K) bf16; conv_w (C, 4) bf16;
    state_in / state_out (B, 3, C) bf16 or None.  Returns (y, state_out)."""
    if cu_seqlens is not None:
        T, K = x.shape
        Bq = cu_seqlens.numel() - 1
        if cu_seqlens.dtype != torch.int32:
            raise ValueError("cu_seqlens must be int32")
    else:
        Bq, T, K = x.shape
    C = W.shape[0]
    dev = _dev(x, W, conv_w, state_in, state_out, y, cu_seqlens)
    if y is None:
        y = torch.empty(tuple(x.shape[:-1]) + (C,), dtype=torch.bfloat16, device=dev)
    check(lib().gdn_in_proj_conv(ptr(x), ptr(W), ptr(conv_w), ptr(state_in), ptr(state_out), ptr(y),
                                 ptr(cu_seqlens), Bq, T, C, K, K, K, C, stream_ptr(dev)))
    return y, state_out


def conv_commit(state_prev, x, commit_n, state_out=None, err_flag=None):
    """Conv window after accepting commit_n[b] tokens of a recorded block."""
    B, T, C = x.shape
    dev = _dev(state_prev, x, commit_n, state_out, err_flag)
    if state_out is None:
        state_out = torch.empty((B, 3, C), dtype=torch.bfloat16, device=dev)
    check(lib().gdn_conv_commit(ptr(state_prev), ptr(x), ptr(commit_n), ptr(state_out), ptr(err_flag),
                                B, T, C, 4, stream_ptr(dev)))
    return state_out


def gated_rmsnorm_fwd(o, z, gamma, out=None, eps=1e-6, out_dtype=torch.bfloat16):
    """out = rms_norm(o, gamma, eps) * silu(z) over the last dim (128)."""
    dev = _dev(o, z, gamma, out)
    rows = o.numel() // D
    flags = (F_NORM_IN_BF16 if o.dtype == torch.bfloat16 else 0) | \
        (F_NORM_OUT_F32 if out_dtype == torch.float32 else 0)
    if out is None:
        out = torch.empty(o.shape, dtype=out_dtype, device=dev)
    check(lib().gdn_gated_rmsnorm_fwd(ptr(o), ptr(z), ptr(gamma), ptr(out), rows, D, eps, flags,
                                      stream_ptr(dev)))
    return out


def chunked_workspace_bytes(B, T, Hv, packed=False) -> int:
    """Workspace bytes for one pass of gdn_chunked_fwd_ws (gdn_chunked_workspace_bytes)."""
    return int(lib().gdn_chunked_workspace_bytes(B, T, Hv, 1 if packed else 0))


def chunked_workspace_min_bytes(B, Hv, has_state_out=True) -> int:
    """Smallest workspace gdn_chunked_fwd_ws accepts; smaller than one pass runs in windows."""
    return int(lib().gdn_chunked_workspace_min_bytes(B, Hv, 1 if has_state_out else 0))


def chunked_fwd(q, k, v, a, b, A_log, dt_bias, state_in=None, state_out=None, o=None, cu_seqlens=None, *,
                l2norm=True, o_dtype=torch.float32, B=None, T=None, split=False, workspace=None):
    """Chunked prefill.  q, k: (..., Hk, 128) bf16 views of token-major rows
    (any token stride); v: (..., Hv, 128).  Leading dims are (B, T) or, with
    cu_seqlens, (total,).  split=False runs gdn_chunked_fwd (one launch, no
    scratch); split=True runs gdn_chunked_fwd_ws on `workspace` (a uint8 CUDA
    tensor of at least chunked_workspace_bytes(...) bytes, allocated here
    when None).  Returns (o, state_out)."""
    Hk, Hv = q.shape[-2], v.shape[-2]
    for t in (q, k, v):
        if t.dtype != torch.bfloat16 or t.stride(-1) != 1 or t.stride(-2) != 128:
            raise ValueError("q, k, v must be bf16 with contiguous 128-wide heads")
    qs, ks, vs = q.stride(-3), k.stride(-3), v.stride(-3)
    if cu_seqlens is not None:
        B = cu_seqlens.numel() - 1
        T = q.shape[0]
        lead = (T,)
    else:
        B, T = q.shape[0], q.shape[1]
        lead = (B, T)
        if B > 1 and T > 0 and (q.stride(0) != T * qs or k.stride(0) != T * ks or v.stride(0) != T * vs):
            raise ValueError("batch rows must follow each other (token-major storage)")
    dev = _dev(a, b, A_log, dt_bias, state_in, state_out, o, cu_seqlens)
    if o is None:
        o = torch.empty(lead + (Hv, D), dtype=o_dtype, device=dev)
    if state_out is None:
        state_out = torch.empty((B, Hv, D, D), dtype=torch.float32, device=dev)
    flags = (F_QK_L2NORM if l2norm else 0) | (F_O_BF16 if o_dtype == torch.bfloat16 else 0)
    if not split:
        check(lib().gdn_chunked_fwd(ptr(q), ptr(k), ptr(v), qs, ks, vs, ptr(a), ptr(b), ptr(A_log), ptr(dt_bias),
                                    ptr(state_in), ptr(state_out), ptr(o), ptr(cu_seqlens), B, T, Hk, Hv, D, D,
                                    flags, stream_ptr(dev)))
        return o, state_out
    need = chunked_workspace_bytes(B, T, Hv, cu_seqlens is not None)
    if workspace is None:
        workspace = torch.empty(need, dtype=torch.uint8, device=dev)
    elif workspace.dtype != torch.uint8 or not workspace.is_contiguous():
        raise ValueError("workspace must be a contiguous uint8 tensor")
    check(lib().gdn_chunked_fwd_ws(ptr(q), ptr(k), ptr(v), qs, ks, vs, ptr(a), ptr(b), ptr(A_log), ptr(dt_bias),
                                   ptr(state_in), ptr(state_out), ptr(o), ptr(cu_seqlens), B, T, Hk, Hv, D, D,
                                   flags, ptr(workspace), workspace.numel(), stream_ptr(dev)))
    return o, state_out
