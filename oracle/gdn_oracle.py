"""CPU oracle for the Gated DeltaNet (GDN) hot path -- TEST INFRASTRUCTURE.

This module restates, in numpy, the reference's own algorithm for every
function on the GDN path of ggluo/Qwen3.8-27B-MLX.  It is the checker the CUDA
kernels are compared against; only ``tests/``, ``__graft_entry__.smoke()`` and
the ``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may use it.
The product never imports it and has no CPU fallback.

Parity status: pinned.  Every function below is checked against golden vectors
(``tests/golden/*.npz``) produced by running the reference's own Python
(python/qwen35.py) over a numpy stand-in for MLX, see tests/golden/gen_golden.py.
MLX's own last-bit rounding is not pinned (MLX is not installable here).

Layouts follow the reference: q,k (B,T,H,Dk); v (B,T,H,Dv); alpha,beta
(B,T,H); state (B,H,Dv,Dk) row-contiguous over Dk.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional

import numpy as np

try:  # bf16 rounding for the "bf16 per op" mode of the front end
    import ml_dtypes
    _BF16 = np.dtype(ml_dtypes.bfloat16)
except Exception:  # pragma: no cover - ml_dtypes ships with this image
    _BF16 = None

F32 = np.float32
EPS = 1e-6          # l2norm and rms_norm epsilon (ops.hpp:19-20; TextConfig.rms_norm_eps)
CHUNK = 64          # chunk size of chunked_delta (python/qwen35.py:365)
CHUNK_THRESHOLD = 16  # python/qwen35.py:338: L >= 16 takes the chunked form


def bf16_round(x) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even) and return
    them as float32."""
    x = np.asarray(x, F32)
    if _BF16 is not None:
        return x.astype(_BF16).astype(F32)
    u = x.view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(F32)


# ---------------------------------------------------------------------------
# element-wise helpers
# ---------------------------------------------------------------------------

def softplus(x):
    """logaddexp(0, x) (cpp/src/ops.cpp:22-25): max(x,0) + log1p(exp(-|x|))."""
    x = np.asarray(x, F32)
    return (np.maximum(x, F32(0)) + np.log1p(np.exp(-np.abs(x)))).astype(F32)


def sigmoid(x):
    x = np.asarray(x, F32)
    return (F32(1) / (F32(1) + np.exp(-x))).astype(F32)


def silu(x):
    """x * sigmoid(x) (cpp/src/ops.cpp:20)."""
    x = np.asarray(x, F32)
    return (x * sigmoid(x)).astype(F32)


def gates(a, b, A_log, dt_bias):
    """Decay and write strength of one GDN layer.

    beta  = sigmoid(b)
    alpha = exp(-exp(A_log) * softplus(a + dt_bias))
    as cpp/src/model.cpp:608-612 and python/qwen35.py:597-600 compute them;
    a, b are (..., H) float32, A_log and dt_bias are (H,).
    """
    a = np.asarray(a, F32)
    A = np.exp(np.asarray(A_log, F32))
    alpha = np.exp(-(A * softplus(a + np.asarray(dt_bias, F32)))).astype(F32)
    return alpha, sigmoid(b)


def l2norm(x, eps=EPS):
    """x * rsqrt(sum(x^2, -1) + eps) -- l2, not RMS (cpp/src/ops.cpp:27-30)."""
    x = np.asarray(x, F32)
    ss = np.sum(x * x, axis=-1, keepdims=True, dtype=F32)
    return (x * (F32(1) / np.sqrt(ss + F32(eps)))).astype(F32)


def l2norm_bf16(x, eps=EPS):
    """l2norm with MLX's per-op bf16 rounding: every intermediate of
    cpp/src/ops.cpp:27-30 rounded to bf16 (reductions accumulate in fp32)."""
    x = bf16_round(x)
    sq = bf16_round(x * x)
    ss = bf16_round(np.sum(sq, axis=-1, keepdims=True, dtype=F32))
    r = bf16_round(F32(1) / np.sqrt(bf16_round(ss + F32(eps))))
    return bf16_round(x * r)


# ---------------------------------------------------------------------------
# the recurrence, per token (the oracle of the decode / verify kernel)
# ---------------------------------------------------------------------------

def delta_reference(q, k, v, alpha, beta, S=None, collect=False, accum=F32):
    """Per-token gated delta rule, state laid out (B,H,Dv,Dk).

    Follows delta::run_reference (cpp/src/delta.cpp:175-204) and
    _delta_step / sequential_delta (python/qwen35.py:434-475), per step:
        kS    = sum_dk k[dk] * S[v,dk]
        S     = a * (S - b * (kS * k)) + b * (v * k)
        o[v]  = sum_dk q[dk] * S[v,dk]
    Returns (o (B,T,H,Dv), S_out (B,H,Dv,Dk)[, states (B,H,T,Dv,Dk)]).
    ``accum=np.float64`` evaluates everything in double precision.
    """
    q = np.asarray(q, accum)
    k = np.asarray(k, accum)
    v = np.asarray(v, accum)
    alpha = np.asarray(alpha, accum)
    beta = np.asarray(beta, accum)
    B, T, H, Dk = q.shape
    Dv = v.shape[-1]
    S = np.zeros((B, H, Dv, Dk), accum) if S is None else np.array(S, accum)
    o = np.zeros((B, T, H, Dv), accum)
    states = np.zeros((B, H, T, Dv, Dk), accum) if collect else None
    for t in range(T):
        kt = k[:, t][:, :, None, :]                     # (B,H,1,Dk)
        qt = q[:, t][:, :, None, :]
        vt = v[:, t][:, :, :, None]                     # (B,H,Dv,1)
        at = alpha[:, t][:, :, None, None]
        bt = beta[:, t][:, :, None, None]
        kS = np.sum(kt * S, axis=-1, keepdims=True)     # (B,H,Dv,1)
        S = at * (S - bt * (kS * kt)) + bt * (vt * kt)
        o[:, t] = np.sum(qt * S, axis=-1)
        if collect:
            states[:, :, t] = S
    cast = (lambda x: x.astype(F32)) if accum != F32 else (lambda x: x)
    if collect:
        return cast(o), cast(S), cast(states)
    return cast(o), cast(S)


def commit_index(n: int, T: int) -> int:
    """DeltaCache::commit(n) (cpp/src/model.cpp:439-457): 0 <= n <= T selects
    S_prev for n == 0, else the state after step n (states[n-1])."""
    if n < 0 or n > T:
        raise ValueError("DeltaCache::commit out of range")
    return n - 1


def spec_residual(p, q):
    """Normalised max(0, p - q), or p / sum(p) when that is empty
    (python/speculative.py:100-106)."""
    r = np.maximum(np.asarray(p, np.float64) - np.asarray(q, np.float64), 0.0)
    tot = r.sum()
    if tot <= 1e-12:
        return np.asarray(p, np.float64) / np.sum(p, dtype=np.float64)
    return r / tot


def spec_verify(p, q, draft, u_accept, u_sample):
    """Acceptance step of a speculative block for one sequence, as
    python/speculative.py:170-190 (cpp/src/session.cpp:495-511): accept draft
    i iff q_i[d_i] > 0 ? u_i q_i[d_i] <= p_i[d_i] : p_i[d_i] > 0; j = leading
    accepted drafts; the corrected token is drawn from p_k (j == k) or from
    the residual of row j -- here by inverse CDF with the uniform u_sample
    (the reference draws with MLX's categorical sampler).  p (k+1, V), q
    (k, V) fp32.  Returns (j, commit_n = j + 1, token)."""
    k = len(draft)
    j = 0
    while j < k:
        d = int(draft[j])
        pd, qd = np.float32(p[j][d]), np.float32(q[j][d])
        acc = (np.float32(u_accept[j]) * qd <= pd) if qd > 0 else (pd > 0)
        if not acc:
            break
        j += 1
    r = np.asarray(p[k], np.float64) if j == k else np.maximum(
        np.asarray(p[j], np.float64) - np.asarray(q[j], np.float64), 0.0)
    if j < k and not r.sum() > 1e-12:
        r = np.asarray(p[j], np.float64)
    cdf = np.cumsum(r)
    v = int(np.searchsorted(cdf, float(u_sample) * cdf[-1], side="right"))
    if v >= len(r):
        v = int(np.nonzero(r > 0)[0][-1])
    return j, j + 1, v


# ---------------------------------------------------------------------------
# the chunked (WY / UT) form, the oracle of the prefill kernel
# ---------------------------------------------------------------------------

def _unit_lower_inverse(Tm):
    """(I + A)^-1 for strictly-lower A by forward substitution over rows, as
    _invert_unit_lower (python/qwen35.py:350-362): row i of X is
    e_i - Tm[i, :i] @ X[:i]."""
    C = Tm.shape[-1]
    X = np.zeros_like(Tm)
    eye = np.eye(C, dtype=Tm.dtype)
    X[..., 0, :] = eye[0]
    for i in range(1, C):
        X[..., i, :] = eye[i] - np.einsum("...j,...jc->...c", Tm[..., i, :i], X[..., :i, :])
    return X


def chunked_delta(q, k, v, alpha, beta, S=None, C=CHUNK, clip=1e-6):
    """Chunked form of the gated delta rule (python/qwen35.py:365-431).

    Steps, per (b, h) and chunk of C tokens:
      1. pad T to a multiple of C with alpha=1, beta=0 (exact no-ops)   :381-388
      2. lcg = cumsum(log(clip(alpha, 1e-6, 1)))                          :400-401
      3. dr[i,j] = exp(lcg_i - lcg_j) on the lower triangle; the exponent
         is masked before exp                                             :406
      4. A = beta_i * dr * (K K^T) * strictly_lower; Tinv = (I + A)^-1     :408-409
      5. U0 = Tinv (beta v); Kt = Tinv (beta cumg k); M = dr * (Q K^T) * lower;
         Qeff = cumg q - M Kt; MU0 = M U0                                  :411-417
      6. serially over chunks with S as (Dk,Dv): y = MU0 + Qeff S;
         U = U0 - Kt S; S = cumg_last S + K^T (ratio_last * U)             :419-429
    Input and output state are (B,H,Dv,Dk), as the reference returns them.
    """
    q = np.asarray(q, F32)
    k = np.asarray(k, F32)
    v = np.asarray(v, F32)
    alpha = np.asarray(alpha, F32)
    beta = np.asarray(beta, F32)
    B, T, H, Dk = q.shape
    Dv = v.shape[-1]
    pad = (C - T % C) % C
    if pad:
        q = np.concatenate([q, np.zeros((B, pad, H, Dk), F32)], 1)
        k = np.concatenate([k, np.zeros((B, pad, H, Dk), F32)], 1)
        v = np.concatenate([v, np.zeros((B, pad, H, Dv), F32)], 1)
        alpha = np.concatenate([alpha, np.ones((B, pad, H), F32)], 1)
        beta = np.concatenate([beta, np.zeros((B, pad, H), F32)], 1)
    Tp = T + pad
    n = Tp // C

    def to_chunks(x, D):                    # (B,Tp,H,D) -> (B,H,n,C,D)
        return np.ascontiguousarray(x.reshape(B, n, C, H, D).transpose(0, 3, 1, 2, 4))

    qc, kc, vc = to_chunks(q, Dk), to_chunks(k, Dk), to_chunks(v, Dv)
    g = alpha.reshape(B, n, C, H).transpose(0, 3, 1, 2)
    bt = beta.reshape(B, n, C, H).transpose(0, 3, 1, 2)

    lcg = np.cumsum(np.log(np.clip(g, F32(clip), F32(1))), axis=-1, dtype=F32)
    cumg = np.exp(lcg)
    ii = np.arange(C)
    lower = (ii[:, None] >= ii[None, :])
    slower = (ii[:, None] > ii[None, :])
    expo = np.where(lower, lcg[..., :, None] - lcg[..., None, :], F32(-1e30))
    dr = np.exp(expo).astype(F32)

    KK = kc @ np.swapaxes(kc, -1, -2)
    A = (bt[..., :, None] * dr * KK * slower).astype(F32)
    Tinv = _unit_lower_inverse(A)
    U0 = Tinv @ (bt[..., :, None] * vc)
    Kt = Tinv @ ((bt * cumg)[..., :, None] * kc)
    M = (dr * (qc @ np.swapaxes(kc, -1, -2)) * lower).astype(F32)
    Qeff = cumg[..., :, None] * qc - M @ Kt
    MU0 = M @ U0
    cumg_last = cumg[..., -1]
    ratio_last = np.exp(lcg[..., -1, None] - lcg)

    St = np.zeros((B, H, Dk, Dv), F32) if S is None else np.ascontiguousarray(
        np.swapaxes(np.asarray(S, F32), -1, -2))
    ys = np.zeros((B, H, n, C, Dv), F32)
    for c in range(n):
        ys[:, :, c] = MU0[:, :, c] + Qeff[:, :, c] @ St
        Uc = U0[:, :, c] - Kt[:, :, c] @ St
        Us = ratio_last[:, :, c][..., None] * Uc
        St = cumg_last[:, :, c][..., None, None] * St + np.swapaxes(kc[:, :, c], -1, -2) @ Us
    y = ys.transpose(0, 2, 3, 1, 4).reshape(B, Tp, H, Dv)[:, :T]
    return np.ascontiguousarray(y, F32), np.ascontiguousarray(np.swapaxes(St, -1, -2), F32)


# ---------------------------------------------------------------------------
# front end and back end
# ---------------------------------------------------------------------------

def depthwise_conv(x, w, state=None, mode="f32"):
    """Causal depthwise conv1d, no bias (cpp/src/model.cpp:385-395,
    python/qwen35.py:642-660).

    x (B,T,C), w (C,K) (the stored (C,1,K) weight with the unit axis dropped),
    state (B,K-1,C) or None for zeros.  Returns (y, xp) where
    xp = concat(state, x) (B,T+K-1,C) and y[t,c] = sum_j xp[t+j,c] * w[c,j].

    mode "f32": exact fp32 products and sums of the given values.
    mode "bf16": MLX's per-op bf16 arithmetic -- each product rounded, the
    running sum (taps in order j = 0..K-1) rounded after every add.
    """
    x = np.asarray(x, F32)
    w = np.asarray(w, F32)
    B, T, Cc = x.shape
    K = w.shape[1]
    pad = np.zeros((B, K - 1, Cc), F32) if state is None else np.asarray(state, F32)
    xp = np.concatenate([pad, x], 1)
    if mode == "bf16":
        y = bf16_round(xp[:, 0:T] * w[:, 0])
        for j in range(1, K):
            y = bf16_round(y + bf16_round(xp[:, j:j + T] * w[:, j]))
        return y, xp
    y = xp[:, 0:T] * w[:, 0]
    for j in range(1, K):
        y = y + xp[:, j:j + T] * w[:, j]
    return y.astype(F32), xp


def gated_rmsnorm(o, z, gamma, eps=EPS):
    """Normalise first, then gate (cpp/src/model.cpp:350-354,
    python/qwen35.py:159-180): rms_norm(o, gamma, eps) * silu(z), in fp32,
    with MLX's rms_norm definition o * rsqrt(mean(o^2) + eps) * gamma.
    gamma is used as stored (not zero-centred, cpp/src/model.cpp:80-85)."""
    o = np.asarray(o, F32)
    ms = np.mean(o * o, axis=-1, keepdims=True, dtype=F32)
    h = o * (F32(1) / np.sqrt(ms + F32(eps))) * np.asarray(gamma, F32)
    return (h * silu(np.asarray(z, F32))).astype(F32)


# ---------------------------------------------------------------------------
# the GDN block minus its projections, with the decode cache
# ---------------------------------------------------------------------------

@dataclass
class DeltaCache:
    """Per-layer recurrent state with speculative rollback
    (python/qwen35.py:291-328, cpp/src/model.cpp:439-457)."""
    conv: Optional[np.ndarray] = None       # (B,K-1,C)
    state: Optional[np.ndarray] = None      # (B,H,Dv,Dk)
    offset: int = 0
    record: bool = False
    base_offset: int = 0
    pending: Optional[tuple] = None

    def commit(self, n: int):
        conv_input, S_prev, states = self.pending
        L = states.shape[2]
        idx = commit_index(n, L)
        st = S_prev if idx < 0 else states[:, :, idx]
        kw = conv_input.shape[1] - L
        self.state = np.ascontiguousarray(st)
        self.conv = np.ascontiguousarray(conv_input[:, n:n + kw])
        self.offset = self.base_offset + n
        self.pending = None
        self.record = False


@dataclass
class BlockWeights:
    conv_w: np.ndarray       # (C, K)
    A_log: np.ndarray        # (Hv,)
    dt_bias: np.ndarray      # (Hv,)
    gamma: np.ndarray        # (Dv,)
    nk: int = 16
    nv: int = 48
    dk: int = 128
    dv: int = 128


def gdn_block(qkv, z, a, b, wts: BlockWeights, cache: Optional[DeltaCache] = None,
              act="f32", chunked_at=CHUNK_THRESHOLD):
    """GatedDeltaNet.__call__ between its projections (python/qwen35.py:572-639;
    cpp/src/model.cpp:582-642).

    qkv (B,L,C) projection output with contiguous [q | k | v]; z (B,L,Hv*Dv);
    a, b (B,L,Hv) gate pre-activations.  Returns the normed output
    (B,L,Hv*Dv) before out_proj, in float32 (rounded to bf16 when act="bf16",
    the cast of cpp/src/model.cpp:627).

    act "f32":  every step in float32.
    act "bf16": the reference's MLX rounding with bf16 activations --
                conv/silu/l2norm/q-scale per op in bf16, then cast to fp32.
    Dispatch is the reference's CPU path: recording -> per-token with
    per-step states; L >= 16 -> chunked; else per-token.
    """
    nk, nv, dk, dv = wts.nk, wts.nv, wts.dk, wts.dv
    qkv = np.asarray(qkv, F32)
    B, L, Cc = qkv.shape
    rnd = bf16_round if act == "bf16" else (lambda x: np.asarray(x, F32))
    conv_state = None if cache is None else cache.conv
    S = None if cache is None else cache.state
    y, xp = depthwise_conv(rnd(qkv), rnd(wts.conv_w), conv_state,
                           mode="bf16" if act == "bf16" else "f32")
    if act == "bf16":
        y = bf16_round(y * bf16_round(sigmoid(y)))
    else:
        y = silu(y)
    nkd = nk * dk
    q = y[..., :nkd].reshape(B, L, nk, dk)
    k = y[..., nkd:2 * nkd].reshape(B, L, nk, dk)
    v = y[..., 2 * nkd:].reshape(B, L, nv, dv)
    scale = F32(dk ** -0.5)
    if act == "bf16":
        q = bf16_round(l2norm_bf16(q) * bf16_round(scale))
        k = l2norm_bf16(k)
    else:
        q = l2norm(q) * scale
        k = l2norm(k)
    rep = nv // nk
    q = np.repeat(q, rep, axis=2).astype(F32)
    k = np.repeat(k, rep, axis=2).astype(F32)
    v = v.astype(F32)
    alpha, beta = gates(rnd(a), rnd(b), wts.A_log, wts.dt_bias)
    if S is None:
        S = np.zeros((B, nv, dv, dk), F32)
    S_prev = S
    recording = cache is not None and cache.record
    states = None
    if recording:
        o, S, states = delta_reference(q, k, v, alpha, beta, S, collect=True)
    elif L >= chunked_at:
        o, S = chunked_delta(q, k, v, alpha, beta, S)
    else:
        o, S = delta_reference(q, k, v, alpha, beta, S)
    zz = rnd(np.asarray(z, F32)).reshape(B, L, nv, dv)
    out = gated_rmsnorm(o, zz, wts.gamma).reshape(B, L, nv * dv)
    out = rnd(out)
    if cache is not None:
        if recording:
            cache.base_offset = cache.offset
            cache.pending = (xp, S_prev, states)
        else:
            K = wts.conv_w.shape[1]
            cache.conv = xp[:, xp.shape[1] - (K - 1):]
            cache.state = S
            cache.offset += L
    return out


# ---------------------------------------------------------------------------
# helpers shared by the tests and the bench
# ---------------------------------------------------------------------------

def rel_err(a, b) -> float:
    """max|a-b| / max|b| (cpp/src/tests.cpp:38-45)."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    d = np.max(np.abs(b)) if b.size else 0.0
    return float(np.max(np.abs(a - b)) / (d if d > 0 else 1.0)) if a.size else 0.0


def rel_l2(a, b) -> float:
    """||a-b||_2 / ||b||_2 (the prefill tolerance's measure)."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    d = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (d if d > 0 else 1.0))


def synth_decode_inputs(rng, B, T, Hk=16, Hv=48, D=128, state_std=0.05):
    """Seeded inputs with the BASELINE config-0 distributions: q,k ~ N(0,1)
    bf16, l2-normalised per head, q scaled by D^-1/2; v ~ N(0,1) bf16; a,b ~
    N(0,1); A_log ~ U(0, ln 16); dt_bias ~ U(0,1); S0 ~ N(0, state_std).
    q, k, v are returned as bf16-representable float32."""
    q = bf16_round(l2norm(bf16_round(rng.standard_normal((B, T, Hk, D), dtype=F32))) * F32(D ** -0.5))
    k = bf16_round(l2norm(bf16_round(rng.standard_normal((B, T, Hk, D), dtype=F32))))
    v = bf16_round(rng.standard_normal((B, T, Hv, D), dtype=F32))
    a = rng.standard_normal((B, T, Hv), dtype=F32)
    b = rng.standard_normal((B, T, Hv), dtype=F32)
    A_log = rng.uniform(0.0, np.log(16.0), (Hv,)).astype(F32)
    dt_bias = rng.uniform(0.0, 1.0, (Hv,)).astype(F32)
    S0 = (rng.standard_normal((B, Hv, D, D), dtype=F32) * F32(state_std)).astype(F32)
    return dict(q=q, k=k, v=v, a=a, b=b, A_log=A_log, dt_bias=dt_bias, S0=S0)


def expand_heads(x, Hv):
    """repeat_interleave over the head axis: key head i serves value heads
    i*r .. i*r+r-1 (python/qwen35.py:592-594)."""
    r = Hv // x.shape[2]
    return np.repeat(np.asarray(x, F32), r, axis=2)


# ---------------------------------------------------------------------------
# the C restatement (gdn_oracle.c), for large cases and the timed CPU baseline
# ---------------------------------------------------------------------------

_C = None


def c_oracle():
    """Load liboracle_gdn.so (built by ``make -C oracle``)."""
    global _C
    if _C is None:
        import ctypes
        import os
        path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "liboracle_gdn.so")
        if not os.path.exists(path):
            raise RuntimeError(f"{path} is not built; run make -C oracle")
        lib = ctypes.CDLL(path)
        vp, i, ll = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong
        lib.oracle_gates.argtypes = [vp] * 6 + [ll, i]
        lib.oracle_recurrent.argtypes = [vp] * 9 + [i] * 6
        lib.oracle_gates.restype = None
        lib.oracle_recurrent.restype = None
        _C = lib
    return _C


def _p(x):
    import ctypes
    return None if x is None else ctypes.c_void_p(x.ctypes.data)


def recurrent_c(q, k, v, a, b, A_log, dt_bias, S_in=None, S_out=None, o=None, states=None,
                nthreads=0):
    """Decode / verify step with raw gates and unexpanded key heads, through
    the C oracle.  All arrays float32 and C-contiguous; q, k (B,T,Hk,D)."""
    B, T, Hk, D = q.shape
    Hv = v.shape[2]
    c = c_oracle()
    alpha = np.empty((B, T, Hv), F32)
    beta = np.empty((B, T, Hv), F32)
    c.oracle_gates(_p(a), _p(b), _p(A_log), _p(dt_bias), _p(alpha), _p(beta), B * T, Hv)
    if S_out is None:
        S_out = np.empty((B, Hv, D, D), F32)
    if o is None:
        o = np.empty((B, T, Hv, D), F32)
    c.oracle_recurrent(_p(q), _p(k), _p(v), _p(alpha), _p(beta), _p(S_in), _p(S_out), _p(o),
                       _p(states), B, T, Hk, Hv, D, nthreads)
    return o, S_out
