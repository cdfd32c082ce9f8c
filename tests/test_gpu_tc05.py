"""The tcgen05 tensor-core path (descriptors, TMEM alloc/ld/st, commit) on
the device, through the gdn_tc05_selftest diagnostic: D = op(A) @ B^T against
a float64 product of the same (tf32- or bf16-representable) operands.
Tolerance 1e-5 max-relative: the products are exact, only the fp32
accumulation order differs."""
import numpy as np
import pytest
import torch

import gdn_b200 as G
import gdn_oracle as O

pytestmark = pytest.mark.gpu


def tf32(x):
    return (x.view(torch.int32) & ~0x1FFF).view(torch.float32)


@pytest.mark.parametrize("N,K", [(64, 64), (128, 128), (64, 128), (16, 16)])
@pytest.mark.parametrize("mode", ["tf32", "bf16", "neg", "tmem", "bf16_a_mn", "bf16_b_mn", "bf16_ab_mn"])
def test_tc05_gemm(N, K, mode):
    g = torch.Generator(device="cuda").manual_seed(N * 1000 + K)
    A = torch.randn((128, K), generator=g, device="cuda")
    B = torch.randn((N, K), generator=g, device="cuda")
    if mode.startswith("bf16"):
        A, B = A.bfloat16().float(), B.bfloat16().float()
    else:
        A, B = tf32(A), tf32(B)
    D, st = G.tc05_selftest(A, B, bf16=mode.startswith("bf16"), negate_a=(mode == "neg"),
                            a_in_tmem=mode.startswith("tmem"), a_mn=mode in ("bf16_a_mn", "bf16_ab_mn"),
                            b_mn=mode in ("bf16_b_mn", "bf16_ab_mn"))
    torch.cuda.synchronize()
    ref = A.double().cpu().numpy() @ B.double().cpu().numpy().T
    if mode == "neg":
        ref = -ref
    assert int(st.item()) == 0
    assert O.rel_err(D.cpu().numpy(), ref) < 1e-5


def test_tf32_mn_major_is_refused():
    A = torch.zeros((128, 16), device="cuda")
    B = torch.zeros((16, 16), device="cuda")
    with pytest.raises(G.GdnError) as e:
        G.tc05_selftest(A, B, a_mn=True)
    assert e.value.code == G.GDN_ERR_FLAGS


@pytest.mark.parametrize("N,K,mode,d_col", [(128, 128, "tmem", 128), (192, 64, "tf32", 192), (192, 64, "tf32", 0),
                                            (256, 32, "tf32", 128), (128, 128, "tmem", 0), (64, 128, "tmem", 192)])
def test_tc05_wide_n_and_column_offsets(N, K, mode, d_col):
    """The accumulator shapes of the split prefill's scan kernel: N = 128 with
    A from tensor memory and N = 192 from shared memory, at column offsets."""
    g = torch.Generator(device="cuda").manual_seed(N * 7 + K + d_col)
    A = tf32(torch.randn((128, K), generator=g, device="cuda"))
    B = tf32(torch.randn((N, K), generator=g, device="cuda"))
    D, st = G.tc05_selftest(A, B, a_in_tmem=(mode == "tmem"), d_col=d_col)
    torch.cuda.synchronize()
    ref = A.double().cpu().numpy() @ B.double().cpu().numpy().T
    assert int(st.item()) == 0
    assert O.rel_err(D.cpu().numpy(), ref) < 1e-5


@pytest.mark.parametrize("N,K", [(64, 128), (128, 64), (256, 32), (64, 8)])
def test_tc05_pair_accumulator_layout(N, K):
    """The CTA-pair MMA (cta_group::2, M = 128) of the pair scan: CTA r's
    64 x N accumulator (rows 64r..64r+63 of D) lies at lane m, column n for
    n < N/2 and at lane 64 + m, column n - N/2 for the rest."""
    g = torch.Generator(device="cuda").manual_seed(N * 31 + K)
    A = tf32(torch.randn((128, K), generator=g, device="cuda"))
    B = tf32(torch.randn((N, K), generator=g, device="cuda"))
    raw, st = G.tc05_pair_selftest(A, B)
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    raw = raw.cpu().numpy()
    ref = A.double().cpu().numpy() @ B.double().cpu().numpy().T
    nh = N // 2
    D = np.empty((128, N))
    for r in range(2):
        D[64 * r:64 * r + 64, :nh] = raw[r, :64]
        D[64 * r:64 * r + 64, nh:] = raw[r, 64:]
    assert O.rel_err(D, ref) < 1e-5


def f16r(x):
    return x.half().float()


@pytest.mark.parametrize("N,K,b_mn", [(64, 128, True), (128, 128, False), (192, 64, False), (64, 64, True)])
def test_tc05_fp16(N, K, b_mn):
    """kind::f16 with fp16 operands, the scan's form: K-major A and B, and B
    MN-major (a K-major [dk][token] tile read as [token][dk]) for N = 64."""
    g = torch.Generator(device="cuda").manual_seed(N * 3 + K + (1 if b_mn else 0))
    A = f16r(torch.randn((128, K), generator=g, device="cuda"))
    B = f16r(torch.randn((N, K), generator=g, device="cuda"))
    D, st = G.tc05_selftest(A, B, fp16=True, b_mn=b_mn)
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    ref = A.double().cpu().numpy() @ B.double().cpu().numpy().T
    assert O.rel_err(D.cpu().numpy(), ref) < 1e-5
