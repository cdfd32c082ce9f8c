"""Drop-in for the reference's python/delta_kernel.py, on the B200 library.

The reference module exposes ``available()`` and
``gated_delta_metal(q, k, v, alpha, beta, S, collect=False)``
(python/delta_kernel.py:122-165).  This module keeps both names and their
argument meaning -- q, k (B,L,H,Dk) already l2-normalised and head-expanded,
v (B,L,H,Dv), alpha, beta (B,L,H), S (B,H,Dv,Dk) or None -- and returns
``(o, S_out)`` or ``(o, S_out, [S_1 .. S_L])`` with ``collect=True``, as torch
tensors on the inputs' CUDA device.  The work runs in ``gdn_delta_run`` of
libgdn_b200.so; there is no other path.
"""
from __future__ import annotations

from typing import List

import torch

import gdn_b200 as _g


def available() -> bool:
    """True when a CUDA device is present and the library loads."""
    if not torch.cuda.is_available():
        return False
    try:
        _g.lib()
    except Exception:
        return False
    return True


def gated_delta_cuda(q, k, v, alpha, beta, S=None, collect: bool = False):
    """Per-token gated delta rule on the GPU; see the module docstring."""
    B, L, H, Dk = q.shape
    Dv = v.shape[-1]
    dev = q.device
    f = torch.float32
    q, k, v = (x.to(f).contiguous() for x in (q, k, v))
    alpha, beta = alpha.to(f).contiguous(), beta.to(f).contiguous()
    S = None if S is None else S.to(f).contiguous()
    o = torch.empty((B, L, H, Dv), dtype=f, device=dev)
    S_out = torch.empty((B, H, Dv, Dk), dtype=f, device=dev)
    states = torch.empty((B, H, L, Dv, Dk), dtype=f, device=dev) if collect else None
    _g.check(_g.lib().gdn_delta_run(_g.ptr(q), _g.ptr(k), _g.ptr(v), _g.ptr(alpha), _g.ptr(beta),
                                    _g.ptr(S), _g.ptr(o), _g.ptr(S_out), _g.ptr(states),
                                    B, L, H, Dk, Dv, _g.stream_ptr(dev)))
    if collect:
        seq: List[torch.Tensor] = [states[:, :, t] for t in range(L)]
        return o, S_out, seq
    return o, S_out


# the reference's name, for a literal swap of the import
gated_delta_metal = gated_delta_cuda
