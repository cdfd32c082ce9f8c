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


def spec(**kw):
    args = dict(p=FAKE, q=FAKE + (1 << 32), draft=FAKE + (2 << 32), u_accept=FAKE + (3 << 32),
                u_sample=FAKE + (4 << 32), B=2, k=3, V=1000, accept_len=FAKE + (5 << 32),
                commit_n=FAKE + (6 << 32), token=FAKE + (7 << 32), err=FAKE + (8 << 32))
    args.update(kw)
    p = lambda x: None if x is None else ctypes.c_void_p(x)  # noqa: E731
    return G.lib().gdn_spec_verify(p(args["p"]), p(args["q"]), p(args["draft"]), p(args["u_accept"]),
                                   p(args["u_sample"]), args["B"], args["k"], args["V"], p(args["accept_len"]),
                                   p(args["commit_n"]), p(args["token"]), p(args["err"]), None)


@pytest.mark.parametrize("kw,code", [
    (dict(k=0), G.GDN_ERR_SHAPE),
    (dict(k=33), G.GDN_ERR_SHAPE),
    (dict(V=0), G.GDN_ERR_SHAPE),
    (dict(V=4096 * 1024 + 1), G.GDN_ERR_SHAPE),
    (dict(B=-1), G.GDN_ERR_SHAPE),
    (dict(p=None), G.GDN_ERR_NULL),
    (dict(token=None), G.GDN_ERR_NULL),
    (dict(err=None), G.GDN_ERR_NULL),
    (dict(q=FAKE + (1 << 32) + 2), G.GDN_ERR_ALIGN),
    (dict(draft=FAKE + (2 << 32) + 1), G.GDN_ERR_ALIGN),
])
def test_spec_verify_bad_arguments_are_rejected(kw, code):
    assert spec(**kw) == code
    assert G.lib().gdn_last_error().decode() != ""


def test_spec_verify_batch_zero_is_a_no_op():
    assert spec(B=0) == G.GDN_OK
    assert G.lib().gdn_last_error().decode() == ""


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU error path only")
@pytest.mark.parametrize("V,what", [(1000, "spec verify launch"), (151936, "spec verify (cluster) launch")])
def test_spec_verify_without_gpu_reports_cuda_error_on_either_launch_path(V, what):
    """Below 64K vocabulary entries one CTA per sequence, from 64K on an
    8-CTA cluster per sequence: both report the failed launch, neither falls
    back to the CPU."""
    assert spec(V=V) == G.GDN_ERR_CUDA
    assert what in G.lib().gdn_last_error().decode()


def test_overlap_flag_is_refused_outside_the_dense_decode_entry():
    """GDN_F_OVERLAP_PREV (launch as a programmatic dependent of the previous
    kernel) is accepted by gdn_recurrent_fwd only; the checkpoint and pool
    entries refuse it before any CUDA call."""
    lib = G.lib()
    v = lambda x: ctypes.c_void_p(x)  # noqa: E731
    inputs = [v(FAKE), v(FAKE + 4096), v(FAKE + 8192), v(FAKE + 12288), v(FAKE + 16384), v(FAKE + 20480),
              v(FAKE + 24576)]
    rc = lib.gdn_recurrent_fwd_from_ckpt(*inputs, v(FAKE + (1 << 32)), v(FAKE + (2 << 32)), v(FAKE + (3 << 32)), 4,
                                         v(FAKE + (5 << 32)), v(FAKE + (6 << 32)), None, v(FAKE + (7 << 32)),
                                         1, 1, 16, 48, 128, 128, G.F_OVERLAP_PREV, None)
    assert rc == G.GDN_ERR_FLAGS
    rc = lib.gdn_recurrent_fwd_pool(*inputs, v(FAKE + (1 << 32)), v(FAKE + (2 << 32)), 4, None, None, 0,
                                    G.POOL_FINAL, v(FAKE + (3 << 32)), None, v(FAKE + (4 << 32)),
                                    1, 1, 16, 48, 128, 128, G.F_OVERLAP_PREV, None)
    assert rc == G.GDN_ERR_FLAGS


# ---------------------------------------------------------------------------
# the split chunked prefill (gdn_chunked_fwd_ws): argument checks and sizing
# ---------------------------------------------------------------------------

def chunked(**kw):
    C = 2 * 16 * 128 + 48 * 128                  # q | k | v rows of the conv output
    args = dict(q=FAKE, k=FAKE + 4096, v=FAKE + 8192, q_stride=C, k_stride=C, v_stride=C,
                a=FAKE + (1 << 33), b=FAKE + (2 << 33), A_log=FAKE + (3 << 33), dt_bias=FAKE + (4 << 33),
                state_in=None, state_out=FAKE + (5 << 33), o=FAKE + (6 << 33), cu=None,
                B=1, T=256, Hk=16, Hv=48, Dk=128, Dv=128, flags=G.F_QK_L2NORM,
                ws=FAKE + (8 << 33), ws_size=1 << 30)
    args.update(kw)
    p = lambda x: None if x is None else ctypes.c_void_p(x)  # noqa: E731
    return G.lib().gdn_chunked_fwd_ws(p(args["q"]), p(args["k"]), p(args["v"]), args["q_stride"],
                                      args["k_stride"], args["v_stride"], p(args["a"]), p(args["b"]),
                                      p(args["A_log"]), p(args["dt_bias"]), p(args["state_in"]),
                                      p(args["state_out"]), p(args["o"]), p(args["cu"]), args["B"], args["T"],
                                      args["Hk"], args["Hv"], args["Dk"], args["Dv"], args["flags"],
                                      p(args["ws"]), args["ws_size"], None)


@pytest.mark.parametrize("kw,code", [
    (dict(flags=0x40000), G.GDN_ERR_FLAGS),
    (dict(Dk=64), G.GDN_ERR_SHAPE),
    (dict(Hk=5), G.GDN_ERR_SHAPE),             # 48 value heads are not a multiple of 5 key heads
    (dict(T=-1), G.GDN_ERR_SHAPE),
    (dict(q_stride=16 * 128 - 8), G.GDN_ERR_SHAPE),   # rows narrower than the heads
    (dict(v_stride=48 * 128 - 8), G.GDN_ERR_SHAPE),
    (dict(k_stride=2 * 16 * 128 + 48 * 128 + 4), G.GDN_ERR_ALIGN),   # not whole 16-byte pieces
    (dict(q=FAKE + 8), G.GDN_ERR_ALIGN),
    (dict(state_out=FAKE + (5 << 33) + 4), G.GDN_ERR_ALIGN),
    (dict(q=None), G.GDN_ERR_NULL),
    (dict(A_log=None), G.GDN_ERR_NULL),
    (dict(o=None), G.GDN_ERR_NULL),
    (dict(state_in=FAKE + (5 << 33) + 4096), G.GDN_ERR_ALIAS),     # partial overlap of the two states
    (dict(o=FAKE + (5 << 33) + 65536), G.GDN_ERR_ALIAS),           # o inside state_out
])
def test_chunked_bad_arguments_are_rejected(kw, code):
    assert chunked(**kw) == code
    assert G.lib().gdn_last_error().decode() != ""


def test_chunked_batch_zero_is_a_no_op():
    assert chunked(B=0) == G.GDN_OK


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU error path only")
def test_chunked_valid_call_without_gpu_reports_cuda_error_not_a_cpu_fallback():
    assert chunked() == G.GDN_ERR_CUDA
    assert chunked(cu=FAKE + (7 << 33), B=3, T=700) == G.GDN_ERR_CUDA


def test_chunked_workspace_sizes():
    """One pass needs a record per (chunk, value head) on top of a fixed
    header; the smallest workspace (one chunk per sequence, windows) is far
    below it and holds the carried state when the call keeps none; a packed
    batch may need one partial chunk per sequence more than a uniform one."""
    one = G.chunked_workspace_bytes(1, 4096, 48)
    two = G.chunked_workspace_bytes(1, 8192, 48)
    assert 0 < one < two
    rec = (two - one) // (64 * 48)                       # bytes per (chunk, value head) record
    assert rec % 256 == 0 and 64 * 1024 < rec < 160 * 1024
    assert G.chunked_workspace_bytes(1, 4096, 24) < one
    mn = G.chunked_workspace_min_bytes(1, 48, True)
    assert 0 < mn < one
    assert G.chunked_workspace_min_bytes(1, 48, False) >= mn + 48 * 128 * 128 * 4
    assert G.chunked_workspace_bytes(8, 4096, 48, packed=True) >= G.chunked_workspace_bytes(8, 512, 48)
    assert G.chunked_workspace_bytes(0, 0, 48) >= 0
    assert G.lib().gdn_chunked_workspace_bytes(1, 64, 0, 0) == 0     # invalid sizes report 0


# ---------------------------------------------------------------------------
# conv1d, gated RMSNorm and the projection GEMM: argument checks
# ---------------------------------------------------------------------------

def conv(**kw):
    args = dict(x=FAKE, w=FAKE + (1 << 33), state_in=None, state_out=None, y=FAKE + (2 << 33), cu=None,
                B=2, T=100, C=640, K=4, flags=0)
    args.update(kw)
    p = lambda x: None if x is None else ctypes.c_void_p(x)  # noqa: E731
    return G.lib().gdn_conv1d_fwd(p(args["x"]), p(args["w"]), p(args["state_in"]), p(args["state_out"]),
                                  p(args["y"]), p(args["cu"]), args["B"], args["T"], args["C"], args["K"],
                                  args["flags"], None)


@pytest.mark.parametrize("kw,code", [
    (dict(K=3), G.GDN_ERR_SHAPE),
    (dict(C=644), G.GDN_ERR_SHAPE),                # channels in whole 16-byte vectors
    (dict(B=-1), G.GDN_ERR_SHAPE),
    (dict(flags=0x1), G.GDN_ERR_FLAGS),
    (dict(w=None), G.GDN_ERR_NULL),
    (dict(y=None), G.GDN_ERR_NULL),
    (dict(x=FAKE + 8), G.GDN_ERR_ALIGN),
    (dict(y=FAKE + 4096), G.GDN_ERR_ALIAS),       # y over x (the halo rows are re-read)
    (dict(state_out=FAKE + 64), G.GDN_ERR_ALIAS),  # the carried window over x
])
def test_conv_bad_arguments_are_rejected(kw, code):
    assert conv(**kw) == code
    assert G.lib().gdn_last_error().decode() != ""


def test_conv_batch_zero_is_a_no_op():
    assert conv(B=0) == G.GDN_OK


def norm(**kw):
    args = dict(o=FAKE, z=FAKE + (1 << 33), gamma=FAKE + (2 << 33), out=FAKE + (3 << 33), rows=4096, D=128,
                flags=0)
    args.update(kw)
    p = lambda x: None if x is None else ctypes.c_void_p(x)  # noqa: E731
    return G.lib().gdn_gated_rmsnorm_fwd(p(args["o"]), p(args["z"]), p(args["gamma"]), p(args["out"]),
                                         args["rows"], args["D"], ctypes.c_float(1e-6), args["flags"], None)


@pytest.mark.parametrize("kw,code", [
    (dict(D=64), G.GDN_ERR_SHAPE),
    (dict(rows=-1), G.GDN_ERR_SHAPE),
    (dict(flags=0x8000), G.GDN_ERR_FLAGS),
    (dict(gamma=None), G.GDN_ERR_NULL),
    (dict(z=FAKE + (1 << 33) + 4), G.GDN_ERR_ALIGN),
    (dict(out=FAKE + 1024), G.GDN_ERR_ALIAS),     # out partly over o
    (dict(out=FAKE + (1 << 33)), G.GDN_ERR_ALIAS),  # out over z
])
def test_norm_bad_arguments_are_rejected(kw, code):
    assert norm(**kw) == code


def test_norm_in_place_over_o_and_zero_rows_are_accepted():
    assert norm(rows=0) == G.GDN_OK
    if not torch.cuda.is_available():           # out == o passes the checks, then needs the GPU
        assert norm(out=FAKE) == G.GDN_ERR_CUDA


def gemm(**kw):
    args = dict(A=FAKE, B=FAKE + (1 << 33), C=FAKE + (2 << 33), C32=None, M=256, N=512, K=5120, lda=5120,
                ldb=5120, ldc=512, ld32=0, n_f32=0)
    args.update(kw)
    p = lambda x: None if x is None else ctypes.c_void_p(x)  # noqa: E731
    return G.lib().gdn_gemm_bf16(p(args["A"]), p(args["B"]), p(args["C"]), p(args["C32"]), args["M"], args["N"],
                                 args["K"], args["lda"], args["ldb"], args["ldc"], args["ld32"], args["n_f32"],
                                 None)


@pytest.mark.parametrize("kw,code", [
    (dict(K=5124, lda=5128, ldb=5128), G.GDN_ERR_SHAPE),   # K in whole 16-byte pieces
    (dict(lda=5112), G.GDN_ERR_SHAPE),                      # stride below K
    (dict(N=516, ldc=520), G.GDN_ERR_SHAPE),                # N a multiple of 8
    (dict(ldc=500), G.GDN_ERR_SHAPE),
    (dict(C32=FAKE + (3 << 33), n_f32=12, ld32=12), G.GDN_ERR_SHAPE),
    (dict(A=None), G.GDN_ERR_NULL),
    (dict(C=None), G.GDN_ERR_NULL),
    (dict(B=FAKE + (1 << 33) + 8), G.GDN_ERR_ALIGN),
])
def test_gemm_bad_arguments_are_rejected(kw, code):
    assert gemm(**kw) == code


def test_gemm_no_rows_is_a_no_op():
    assert gemm(M=0) == G.GDN_OK
