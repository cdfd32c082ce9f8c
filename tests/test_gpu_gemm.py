"""The block's projections on the tensor cores, through the C ABI:
gdn_gemm_bf16 (in_proj_z / in_proj_a / in_proj_b, out_proj) against an fp32
matmul of the same bf16 operands, and gdn_in_proj_conv (in_proj_qkv with the
causal conv + SiLU in its epilogue) against gdn_conv1d_fwd applied to
gdn_gemm_bf16's output.

Tolerances:
  * GEMM: every element within one bf16 rounding of the fp32 product
    (|C - ref| <= 2^-8 |ref| + 2^-8 * rms(ref) -- the second term covers the
    accumulation-order difference near zero); the fp32 columns hold exactly
    the bf16-rounded values of the same accumulators;
  * fused conv: bit-identical to the unfused pair (the same bf16 projection
    values, the same tap arithmetic), outputs and carried windows.
"""
import numpy as np
import pytest
import torch

import gdn_b200 as G

pytestmark = pytest.mark.gpu


def rand_bf16(shape, scale, g):
    return (torch.randn(shape, generator=g, device="cuda") * scale).bfloat16()


def ref_gemm(A, B):
    return A.float() @ B.float().t()


def within_one_rounding(C, ref):
    C, ref = C.float(), ref.float()
    tol = 2.0 ** -8 * ref.abs() + 2.0 ** -8 * ref.pow(2).mean().sqrt()
    return bool(((C - ref).abs() <= tol).all())


@pytest.fixture(autouse=True)
def _no_tf32():
    old = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32 = old


# shapes with fewer than 74 tiles of 256 x 256 run on single CTAs (128 x 256
# tiles), larger ones on CTA pairs (256 x 256, tcgen05 cta_group::2)
@pytest.mark.parametrize("M,N,K", [(1, 256, 64), (300, 520, 256), (129, 16, 128), (4096, 512, 6144),
                                   (777, 1024, 5120), (2048, 6144, 512), (3001, 2304, 1024)])
def test_gemm_matches_fp32_matmul(M, N, K):
    g = torch.Generator(device="cuda")
    g.manual_seed(M + N + K)
    A = rand_bf16((M, K), 1.0, g)
    B = rand_bf16((N, K), K ** -0.5, g)
    C = G.gemm_bf16(A, B)
    torch.cuda.synchronize()
    assert within_one_rounding(C, ref_gemm(A, B))
    assert G.take_device_error() == 0


def test_gemm_fp32_tail_columns():
    """z | a | b in one product: 6144 bf16 columns, then 96 as fp32 (the
    .astype(float32) of the gate projections)."""
    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    M, K = 1000, 5120
    A = rand_bf16((M, K), 1.0, g)
    B = rand_bf16((6240, K), K ** -0.5, g)
    C, C32 = G.gemm_bf16(A, B, n_f32=6144)
    torch.cuda.synchronize()
    ref = ref_gemm(A, B)
    assert C.shape == (M, 6144) and C32.shape == (M, 96) and C32.dtype == torch.float32
    assert within_one_rounding(C, ref[:, :6144])
    assert within_one_rounding(C32, ref[:, 6144:])
    assert torch.equal(C32, C32.bfloat16().float())          # bf16 values carried as fp32
    full = G.gemm_bf16(A, B)                                   # the same accumulators, all bf16
    assert torch.equal(full[:, :6144], C) and torch.equal(full[:, 6144:].float(), C32)
    # the fp32 tail as two stacked (M, 48) matrices: a then b, each contiguous
    C2, ab = G.gemm_bf16(A, B, n_f32=6144, f32_width=48)
    assert ab.shape == (2, M, 48) and torch.equal(C2, C)
    assert torch.equal(ab[0], C32[:, :48]) and torch.equal(ab[1], C32[:, 48:])


def test_gemm_rejects_bad_arguments():
    A = torch.zeros((8, 60), dtype=torch.bfloat16, device="cuda")
    B = torch.zeros((16, 60), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(G.GdnError):                            # K not a multiple of 8
        G.gemm_bf16(A, B)


@pytest.mark.parametrize("with_state", [True, False])
def test_in_proj_conv_uniform_matches_unfused(with_state):
    g = torch.Generator(device="cuda")
    g.manual_seed(11)
    Bq, T, K, N = 2, 300, 512, 1280
    x = rand_bf16((Bq, T, K), 1.0, g)
    W = rand_bf16((N, K), K ** -0.5, g)
    w = rand_bf16((N, 4), 0.5, g)
    st = rand_bf16((Bq, 3, N), 1.0, g) if with_state else None
    so_f = torch.empty((Bq, 3, N), dtype=torch.bfloat16, device="cuda")
    so_u = torch.empty_like(so_f)
    y_f, _ = G.in_proj_conv(x, W, w, state_in=st, state_out=so_f)
    p = G.gemm_bf16(x.view(Bq * T, K), W).view(Bq, T, N)
    y_u, _ = G.conv1d_fwd(p, w, state_in=st, state_out=so_u)
    torch.cuda.synchronize()
    assert torch.equal(y_f, y_u)
    assert torch.equal(so_f, so_u)
    assert G.take_device_error() == 0


@pytest.mark.parametrize("N", [768, 10240])
def test_in_proj_conv_packed_varlen_matches_unfused(N):
    """Sequences shorter than the 3-row window, empty ones, and ones that cross
    tile boundaries (125 tokens per CTA tile, 250 per CTA pair); N = 768 runs
    on single CTAs, N = 10240 on CTA pairs."""
    g = torch.Generator(device="cuda")
    g.manual_seed(12)
    lens = [100, 0, 257, 1, 2, 640, 125, 126, 250, 251, 249]
    K = 256
    tot = sum(lens)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]).astype(np.int32), device="cuda")
    x = rand_bf16((tot, K), 1.0, g)
    W = rand_bf16((N, K), K ** -0.5, g)
    w = rand_bf16((N, 4), 0.5, g)
    st = rand_bf16((len(lens), 3, N), 1.0, g)
    so_f = torch.full((len(lens), 3, N), 7.0, dtype=torch.bfloat16, device="cuda")
    so_u = torch.empty_like(so_f)
    y_f, _ = G.in_proj_conv(x, W, w, state_in=st, state_out=so_f, cu_seqlens=cu)
    y_u, _ = G.conv1d_fwd(G.gemm_bf16(x, W), w, state_in=st, state_out=so_u, cu_seqlens=cu)
    torch.cuda.synchronize()
    assert torch.equal(y_f, y_u)
    assert torch.equal(so_f, so_u)
    assert G.take_device_error() == 0


def test_in_proj_conv_config4_shape_spot_check():
    """The config-4 projection shape (hidden 5120 -> 10240 conv channels) on
    two packed sequences: bit-identical to the unfused pair."""
    g = torch.Generator(device="cuda")
    g.manual_seed(13)
    lens = [1500, 2222]
    K, N = 5120, 10240
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]).astype(np.int32), device="cuda")
    x = rand_bf16((sum(lens), K), 1.0, g)
    W = rand_bf16((N, K), K ** -0.5, g)
    w = rand_bf16((N, 4), 0.5, g)
    y_f, _ = G.in_proj_conv(x, W, w, cu_seqlens=cu)
    y_u, _ = G.conv1d_fwd(G.gemm_bf16(x, W), w, cu_seqlens=cu)
    torch.cuda.synchronize()
    assert torch.equal(y_f, y_u)
    assert G.take_device_error() == 0
