"""
bf16 projections on the library's tcgen05 GEMM (ll_gemm_bf16*): the F.linear products around the
routed experts (the latent block's down / up projections, lazy_lora/trainer/lazy_trainer.py:
722-735, and the shared expert's three projections), forward and input-gradient backward.

bf16 operands, fp32 accumulation, bf16 output (round to nearest), as F.linear / torch.matmul of
bf16 tensors compute them on CUDA; sums run in another fixed order, so results agree to within
bf16 rounding, and are bitwise reproducible run to run. CUDA tensors only; no fallback.
"""
from typing import Optional

import torch

from .. import _lib as L


def _ok(t: torch.Tensor) -> torch.Tensor:
    """A 2-D bf16 CUDA tensor with unit inner stride, a leading dimension that is a multiple of
    8 elements and a 16-byte aligned start, copied when it is not."""
    if t.dtype != torch.bfloat16:
        t = t.to(torch.bfloat16)
    if t.dim() != 2 or t.stride(1) != 1 or t.stride(0) % 8 or t.stride(0) < t.shape[1] or t.data_ptr() % 16:
        t = t.contiguous()
    if t.stride(0) % 8:
        pad = torch.zeros((t.shape[0], (t.shape[1] + 7) // 8 * 8), dtype=t.dtype, device=t.device)
        pad[:, :t.shape[1]] = t
        t = pad[:, :t.shape[1]]
    return t


def _out(M: int, N: int, like: torch.Tensor, out: Optional[torch.Tensor]) -> torch.Tensor:
    if out is not None:
        if out.dtype != torch.bfloat16 or out.shape != (M, N) or out.stride(1) != 1 or out.stride(0) % 8 or \
                out.data_ptr() % 16:
            raise ValueError("out: bf16 [M, N] with unit inner stride, leading dimension a multiple of 8, "
                             "16-byte aligned")
        return out
    ld = (N + 7) // 8 * 8
    buf = torch.empty((M, ld), dtype=torch.bfloat16, device=like.device)
    return buf[:, :N]


def linear(x: torch.Tensor, w: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """x [M, K] . w^T with w [N, K] (F.linear without bias) -> bf16 [M, N]."""
    L.require_cuda(x, w)
    a, b = _ok(x), _ok(w)
    M, K = a.shape
    N = b.shape[0]
    if b.shape[1] != K:
        raise ValueError(f"linear: x {tuple(x.shape)} and w {tuple(w.shape)} do not match")
    c = _out(M, N, a, out)
    L.check(L.load().ll_gemm_bf16(M, N, K, a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0), 1, c.data_ptr(),
                                  c.stride(0), 1, L.stream_ptr()), "ll_gemm_bf16")
    return c


def matmul(g: torch.Tensor, w: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """g [M, K] . w with w [K, N] (the input gradient through F.linear's weight) -> bf16 [M, N]."""
    L.require_cuda(g, w)
    a, b = _ok(g), _ok(w)
    M, K = a.shape
    N = b.shape[1]
    if b.shape[0] != K:
        raise ValueError(f"matmul: g {tuple(g.shape)} and w {tuple(w.shape)} do not match")
    c = _out(M, N, a, out)
    L.check(L.load().ll_gemm_bf16(M, N, K, a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0), 0, c.data_ptr(),
                                  c.stride(0), 1, L.stream_ptr()), "ll_gemm_bf16")
    return c


def linear_two(x: torch.Tensor, w0: torch.Tensor, w1: torch.Tensor):
    """(x . w0^T, x . w1^T) in one launch, w0 and w1 [N, K] (the gate and up projections)."""
    L.require_cuda(x, w0, w1)
    a, b0, b1 = _ok(x), _ok(w0), _ok(w1)
    M, K = a.shape
    N = b0.shape[0]
    if b0.shape != (N, K) or b1.shape != (N, K) or b0.stride(0) != b1.stride(0):
        raise ValueError("linear_two: w0 and w1 must both be [N, K] with the same leading dimension")
    ld = (N + 7) // 8 * 8
    buf = torch.empty((2, M, ld), dtype=torch.bfloat16, device=x.device)
    c0, c1 = buf[0, :, :N], buf[1, :, :N]
    L.check(L.load().ll_gemm_bf16_two_outputs(M, N, K, a.data_ptr(), a.stride(0), b0.data_ptr(), b1.data_ptr(),
                                              b0.stride(0), 1, c0.data_ptr(), c1.data_ptr(), ld, 1, L.stream_ptr()),
            "ll_gemm_bf16_two_outputs")
    return c0, c1


def matmul_sum2(g0: torch.Tensor, w0: torch.Tensor, g1: torch.Tensor, w1: torch.Tensor) -> torch.Tensor:
    """g0 . w0 + g1 . w1 with w [K, N], summed in fp32 before the one rounding to bf16
    (dx = dG W_g + dU W_u)."""
    L.require_cuda(g0, w0, g1, w1)
    a0, b0, a1, b1 = _ok(g0), _ok(w0), _ok(g1), _ok(w1)
    M, K0 = a0.shape
    K1 = a1.shape[1]
    N = b0.shape[1]
    if a1.shape[0] != M or b0.shape[0] != K0 or b1.shape != (K1, N):
        raise ValueError("matmul_sum2: shapes do not match")
    c = _out(M, N, a0, None)
    L.check(L.load().ll_gemm_bf16_sum2(M, N, a0.data_ptr(), K0, a0.stride(0), b0.data_ptr(), b0.stride(0), 0,
                                       a1.data_ptr(), K1, a1.stride(0), b1.data_ptr(), b1.stride(0), 0, c.data_ptr(),
                                       c.stride(0), 1, L.stream_ptr()), "ll_gemm_bf16_sum2")
    return c


def check_status():
    """Raise if a bounded wait inside one of these GEMMs ran out since the last check."""
    L.check(L.load().ll_gemm_bf16_status(L.stream_ptr()), "ll_gemm_bf16")
