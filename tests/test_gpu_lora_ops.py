"""
GPU checks of the LoRA product entry points (ll_lora_down, ll_lora_outer, ll_lora_add_bf16)
against plain PyTorch fp32 restatements of lora_layer.py:104-123's products (x A^T, the
adapter gradients, and the bf16 sum of a projection and its rounded delta).

Tolerances: the products are fp32 sums of bf16 inputs in another order than torch's, so they
agree to a few fp32 ulps of the sum (relative L2 1e-5). The bf16 add rounds the delta and the
sum to bf16 as the reference does; a different fp32 order inside the delta can move a rounding
by one bf16 ulp, so the result is held to 1e-3 relative L2 and 99 % of elements bit-equal.
Repeated calls are bitwise identical (fixed-order sums).
"""
import ctypes

import pytest
import torch

from lazylora_b200 import _lib as L

pytestmark = pytest.mark.gpu
WS = 16 * 1024 * 1024


def rel(a, b):
    return ((a.double() - b.double()).norm() / b.double().norm().clamp_min(1e-30)).item()


@pytest.fixture(scope="module")
def lib():
    return L.load()


def down(lib, X, B0, B1, n0, n, b_rows, ws_bytes=WS):
    M, K = X.shape
    ws = torch.empty(max(ws_bytes // 4, 4), dtype=torch.float32, device="cuda")
    C0 = torch.full((M, n0), float("nan"), device="cuda")
    C1 = torch.full((M, n - n0), float("nan"), device="cuda") if n > n0 else None
    rc = lib.ll_lora_down(X.data_ptr(), 1, M, K, B0.data_ptr(), B1.data_ptr() if B1 is not None else None, n0, n,
                          b_rows, ctypes.c_float(1.0), C0.data_ptr(), C1.data_ptr() if C1 is not None else None,
                          ws.data_ptr(), ws_bytes, L.stream_ptr())
    return rc, C0, C1


@pytest.mark.parametrize("M,K,r", [(1, 64, 4), (37, 1024, 8), (1024, 7168, 16), (300, 2048, 32)])
def test_lora_down_rows_pair(lib, M, K, r):
    g = torch.Generator(device="cuda").manual_seed(M + K)
    X = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    A0 = torch.randn(r, K, device="cuda", generator=g) / K ** 0.5
    A1 = torch.randn(r, K, device="cuda", generator=g) / K ** 0.5
    rc, C0, C1 = down(lib, X, A0, A1, r, 2 * r, 1)
    L.check(rc, "ll_lora_down")
    assert rel(C0, X.float() @ A0.t()) < 1e-5
    assert rel(C1, X.float() @ A1.t()) < 1e-5
    rc, D0, D1 = down(lib, X, A0, A1, r, 2 * r, 1)
    assert torch.equal(C0, D0) and torch.equal(C1, D1)


@pytest.mark.parametrize("M,K,r", [(5, 256, 4), (1024, 7168, 16), (64, 6144, 32)])
def test_lora_down_columns(lib, M, K, r):
    g = torch.Generator(device="cuda").manual_seed(K - M)
    X = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    B = torch.randn(K, r, device="cuda", generator=g) * 0.05
    rc, C0, _ = down(lib, X, B, None, r, r, 0)
    L.check(rc, "ll_lora_down")
    assert rel(C0, X.float() @ B) < 1e-5


def test_lora_down_small_workspace_fewer_splits(lib):
    g = torch.Generator(device="cuda").manual_seed(11)
    M, K, r = 512, 4096, 16
    X = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    A = torch.randn(r, K, device="cuda", generator=g) / K ** 0.5
    want = X.float() @ A.t()
    rc, C0, _ = down(lib, X, A, None, r, r, 1, ws_bytes=4 * M * r)          # one split fits
    L.check(rc, "ll_lora_down")
    assert rel(C0, want) < 1e-5
    rc, _, _ = down(lib, X, A, None, r, r, 1, ws_bytes=4 * M * r - 4)      # not even one
    assert rc == 4                                                           # LL_ERR_WORKSPACE


@pytest.mark.parametrize("N,C,r,transposed", [(16, 256, 4, False), (1024, 7168, 16, True), (1024, 6144, 16, False),
                                              (77, 2048, 32, True)])
def test_lora_outer(lib, N, C, r, transposed):
    g = torch.Generator(device="cuda").manual_seed(N * 3 + C)
    P = torch.randn(N, r, device="cuda", generator=g)
    Q = torch.randn(N, C, device="cuda", generator=g).to(torch.bfloat16)
    s = 2.0
    out = torch.full((C, r) if transposed else (r, C), float("nan"), device="cuda")
    ws = torch.empty(WS // 4, dtype=torch.float32, device="cuda")
    L.check(lib.ll_lora_outer(P.data_ptr(), Q.data_ptr(), 1, N, C, r, ctypes.c_float(s), int(transposed),
                              out.data_ptr(), ws.data_ptr(), WS, L.stream_ptr()), "ll_lora_outer")
    want = s * P.t() @ Q.float()
    assert rel(out, want.t() if transposed else want) < 1e-5


@pytest.mark.parametrize("N,C,r,two,r_rows", [(8, 256, 4, False, False), (1024, 7168, 16, False, False),
                                              (1024, 7168, 16, True, True), (45, 6144, 32, True, True),
                                              (33, 512, 8, False, True)])
def test_lora_add_bf16(lib, N, C, r, two, r_rows):
    g = torch.Generator(device="cuda").manual_seed(N + C + r)
    Y = torch.randn(N, C, device="cuda", generator=g).to(torch.bfloat16)
    Ls = [torch.randn(N, r, device="cuda", generator=g) for _ in range(2)]
    Rs = [torch.randn(r, C, device="cuda", generator=g) * 0.05 for _ in range(2)]
    s = 2.0
    Rarg = [R.contiguous() if r_rows else R.t().contiguous() for R in Rs]        # [r][C] or [C][r]
    out = Y.clone()
    L.check(lib.ll_lora_add_bf16(out.data_ptr(), Ls[0].data_ptr(), Rarg[0].data_ptr(),
                                 Ls[1].data_ptr() if two else None, Rarg[1].data_ptr() if two else None, r,
                                 int(r_rows), ctypes.c_float(s), N, C, out.data_ptr(), L.stream_ptr()),
            "ll_lora_add_bf16")
    want = Y.float() + (s * Ls[0] @ Rs[0]).to(torch.bfloat16).float()
    if two:
        want = want + (s * Ls[1] @ Rs[1]).to(torch.bfloat16).float()
    want = want.to(torch.bfloat16)
    assert rel(out.float(), want.float()) < 1e-3
    assert (out == want).float().mean().item() > 0.99
