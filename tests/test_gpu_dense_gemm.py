"""
The tcgen05 bf16 GEMMs of the dense projections (ll_gemm_bf16*) against a plain PyTorch fp32
reference of the same op: the bf16 operands' products summed in fp32 (exact products, so the
only difference is the order and rounding of the sums, ~1e-6 relative: the tensor cores' fp32
accumulation differs from sequential IEEE sums by up to ~1e-4 of the partial sums' size when
terms cancel), then rounded to bf16 when the output is bf16 (half a bf16 ulp, at most 2^-8
relative).

Covers both B layouts ([N][K] for F.linear, [K][N] for the input gradient), ragged M, N and K
(tile and K-block tails through the TMA's zero fill), one token, the two-output launch and the
two-pair sum, and the shapes of the shared expert and the latent block.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref(a, b, b_nk):
    af, bf = a.float(), b.float()
    return af @ (bf.t() if b_nk else bf)


def _gemm(a, b, b_nk, c_dtype):
    from lazylora_b200 import _lib as L
    lib = L.load()
    M, K = a.shape
    N = b.shape[0] if b_nk else b.shape[1]
    ld = (N + 7) // 8 * 8
    c = torch.empty((M, ld), dtype=torch.bfloat16 if c_dtype == 1 else torch.float32, device="cuda")[:, :N]
    rc = lib.ll_gemm_bf16(M, N, K, a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0), b_nk, c.data_ptr(), ld,
                          c_dtype, L.stream_ptr())
    assert rc == 0, L.load().ll_last_cuda_error()
    assert lib.ll_gemm_bf16_status(L.stream_ptr()) == 0
    return c


def _rel(x, y):
    return float((x.float() - y.float()).norm() / y.float().norm().clamp_min(1e-30))


@pytest.mark.parametrize("M,N,K", [(1, 64, 64), (5, 100, 72), (127, 256, 512), (128, 176, 1000), (300, 520, 7168),
                                   (1024, 6144, 7168), (1024, 7168, 3584)])
@pytest.mark.parametrize("b_nk", [1, 0])
def test_gemm_matches_fp32_reference(M, N, K, b_nk):
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N + K + b_nk)
    a = torch.randn(M, K, generator=g, device="cuda").to(torch.bfloat16)
    rows, cols = (N, K) if b_nk else (K, N)
    # rows 16-byte aligned: the leading dimension rounded up to 8 elements (a view when padded)
    b = torch.zeros(rows, (cols + 7) // 8 * 8, dtype=torch.bfloat16, device="cuda")[:, :cols]
    b.copy_((torch.randn(rows, cols, generator=g, device="cuda") * 0.05).to(torch.bfloat16))
    want = _ref(a, b, b_nk)
    got32 = _gemm(a, b, b_nk, 0)
    assert _rel(got32, want) < 1e-5, "fp32 output: summation order only"
    got16 = _gemm(a, b, b_nk, 1)
    err = (got16.float() - want).abs()
    atol = 1e-4 * float(want.pow(2).mean().sqrt())
    assert bool((err <= want.abs() * 2 ** -8 + atol).all()), "bf16 output within one rounding of the fp32 sum"


def test_linear_two_and_sum2():
    from lazylora_b200.core import dense as D
    g = torch.Generator(device="cuda").manual_seed(11)
    M, F, d = 300, 6144, 7168
    x = torch.randn(M, d, generator=g, device="cuda").to(torch.bfloat16)
    wg = (torch.randn(F, d, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    wu = (torch.randn(F, d, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    G, U = D.linear_two(x, wg, wu)
    assert _rel(G, _ref(x, wg, 1)) < 3e-3 and _rel(U, _ref(x, wu, 1)) < 3e-3
    assert torch.equal(G, D.linear(x, wg)) and torch.equal(U, D.linear(x, wu)), "same tiles, same bits"
    dG = torch.randn(M, F, generator=g, device="cuda").to(torch.bfloat16)
    dU = torch.randn(M, F, generator=g, device="cuda").to(torch.bfloat16)
    dx = D.matmul_sum2(dG, wg, dU, wu)
    want = dG.float() @ wg.float() + dU.float() @ wu.float()
    assert _rel(dx, want) < 3e-3
    err = (dx.float() - want).abs()
    atol = 1e-4 * float(want.pow(2).mean().sqrt())
    assert bool((err <= want.abs() * 2 ** -8 + atol).all()), "one rounding of the fp32 sum of both products"
    D.check_status()


def test_gemm_deterministic_and_refuses_bad_args():
    from lazylora_b200 import _lib as L
    from lazylora_b200.core import dense as D
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(200, 1024, generator=g, device="cuda").to(torch.bfloat16)
    w = torch.randn(700, 1024, generator=g, device="cuda").to(torch.bfloat16)
    assert torch.equal(D.linear(x, w), D.linear(x, w))
    lib = L.load()
    c = torch.empty(200, 704, dtype=torch.bfloat16, device="cuda")
    # leading dimension not a multiple of 8, misaligned pointer, bad dtype code
    assert lib.ll_gemm_bf16(200, 700, 1024, x.data_ptr(), 1020, w.data_ptr(), 1024, 1, c.data_ptr(), 704, 1,
                            L.stream_ptr()) != 0
    assert lib.ll_gemm_bf16(200, 700, 1024, x.data_ptr() + 2, 1024, w.data_ptr(), 1024, 1, c.data_ptr(), 704, 1,
                            L.stream_ptr()) != 0
    assert lib.ll_gemm_bf16(200, 700, 1024, x.data_ptr(), 1024, w.data_ptr(), 1024, 1, c.data_ptr(), 704, 2,
                            L.stream_ptr()) != 0
