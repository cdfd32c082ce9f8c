"""The C ABI library without a GPU: it loads, exports every function that
include/*.h declares, and rejects bad arguments with the documented status
codes before making any CUDA call.  CPU only -- no kernel is launched (the
pointers below are fake and never dereferenced)."""
import ctypes
import glob
import os
import re

import pytest
import torch

import gdn_b200 as G
from conftest import ROOT

FAKE = 1 << 40          # 16-byte aligned fake device address, never dereferenced


def declarations():
    """name -> list of parameter declarations, parsed from include/*.h."""
    out = {}
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for name, params in re.findall(r"\b(gdn_\w+)\s*\(([^;{]*?)\)\s*;", src):
            ps = [p.strip() for p in params.split(",") if p.strip() and p.strip() != "void"]
            out[name] = ps
    return out


def declared_functions():
    return sorted(declarations())


def test_library_exports_every_declared_symbol():
    L = G.lib()
    names = declared_functions()
    assert "gdn_recurrent_fwd" in names
    for n in names:
        assert hasattr(L, n), n
        assert n in G.SIGNATURES, f"{n} has no ctypes signature"


def test_ctypes_signatures_match_header_parameter_lists():
    """Every ctypes argtypes list has one entry per declared parameter, and
    pointers / integers sit where the header puts them."""
    for name, params in declarations().items():
        args = G.SIGNATURES[name]
        assert len(args) == len(params), (name, len(args), len(params))
        for decl, t in zip(params, args):
            is_ptr = "*" in decl
            assert (t is ctypes.c_void_p) == is_ptr, (name, decl, t)


def test_version():
    assert G.lib().gdn_version() >= 100


def rec(**kw):
    args = dict(q=FAKE, k=FAKE + 4096, v=FAKE + 8192, a=FAKE + 12288, b=FAKE + 16384,
                A_log=FAKE + 20480, dt_bias=FAKE + 24576, state_in=FAKE + (1 << 30),
                state_out=FAKE + (2 << 30), o=FAKE + (3 << 30), ckpt=None,
                B=1, T=1, Hk=16, Hv=48, Dk=128, Dv=128, flags=0)
    args.update(kw)
    p = lambda x: None if x is None else ctypes.c_void_p(x)  # noqa: E731
    return G.lib().gdn_recurrent_fwd(p(args["q"]), p(args["k"]), p(args["v"]), p(args["a"]), p(args["b"]),
                                     p(args["A_log"]), p(args["dt_bias"]), p(args["state_in"]),
                                     p(args["state_out"]), p(args["o"]), p(args["ckpt"]),
                                     args["B"], args["T"], args["Hk"], args["Hv"], args["Dk"], args["Dv"],
                                     args["flags"], None)


@pytest.mark.parametrize("kw,code", [
    (dict(Dk=64), G.GDN_ERR_SHAPE),
    (dict(Dv=96), G.GDN_ERR_SHAPE),
    (dict(Hk=5), G.GDN_ERR_SHAPE),
    (dict(B=-1), G.GDN_ERR_SHAPE),
    (dict(flags=0x100), G.GDN_ERR_FLAGS),
    (dict(q=None), G.GDN_ERR_NULL),
    (dict(o=None), G.GDN_ERR_NULL),
    (dict(A_log=None), G.GDN_ERR_NULL),
    (dict(state_out=None), G.GDN_ERR_NULL),
    (dict(state_in=FAKE + (1 << 30) + 4), G.GDN_ERR_ALIGN),
    (dict(k=FAKE + 4098), G.GDN_ERR_ALIGN),
    (dict(state_out=FAKE + (1 << 30) + 1024), G.GDN_ERR_ALIAS),
    (dict(ckpt=FAKE + (1 << 30) + 65536), G.GDN_ERR_ALIAS),
    (dict(o=FAKE + (2 << 30) + 64), G.GDN_ERR_ALIAS),
])
def test_bad_arguments_are_rejected(kw, code):
    assert rec(**kw) == code
    assert G.lib().gdn_last_error().decode() != ""


def test_batch_zero_is_a_no_op():
    assert rec(B=0) == G.GDN_OK
    assert G.lib().gdn_last_error().decode() == ""


def test_gates_direct_needs_no_gate_parameters():
    # rejected only for the state overlap, not for the missing A_log/dt_bias
    assert rec(flags=G.F_GATES_DIRECT, A_log=None, dt_bias=None,
               state_out=FAKE + (1 << 30) + 1024) == G.GDN_ERR_ALIAS


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU error path only")
def test_valid_call_without_gpu_reports_cuda_error_not_a_cpu_fallback():
    assert rec() == G.GDN_ERR_CUDA
    assert "gdn recurrent kernel launch" in G.lib().gdn_last_error().decode()
