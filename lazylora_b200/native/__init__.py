"""
Drop-in for lazy_lora.native: `kernel()` returns an object with the same `gemm`, `gemm_t`
and `dequant` methods as lazy_lora/native/__init__.py:19-74 (MXFP4Kernel), running on the
B200 through the C ABI instead of the OpenMP C file.

Differences from the reference, on purpose:
  * tensors live on the GPU (inputs on the CPU are refused, not silently moved);
  * `kernel()` raises when the CUDA library cannot be loaded instead of returning None,
    because there is no CPU fallback behind it (LAZYLORA_NO_NATIVE=1 raises as well);
  * `gemm` accepts any K that is a multiple of 32 (the reference's stack tile stops at
    K = 4096, mxfp4_gemm.c:72).
Arithmetic: the weights decode exactly (fp16, scale bytes within 36 of the matrix maximum),
activation rows are rounded to fp16 after a power-of-two row scaling, products accumulate in
fp32 on the tensor cores: ~2^-12 relative per element against the reference's fp32.
"""
import os

import torch

from .. import _lib as L


def _pad_scales(scales: torch.Tensor):
    """Scale rows padded to a multiple of 16 bytes (TMA strides), plus the stride."""
    R, G = scales.shape
    stride = (G + 15) // 16 * 16
    if stride == G and scales.is_contiguous():
        return scales, stride
    out = torch.zeros((R, stride), dtype=torch.uint8, device=scales.device)
    out[:, :G] = scales
    return out, stride


class MXFP4Kernel:
    def __init__(self, lib):
        self.lib = lib

    def threads(self) -> int:
        return int(self.lib.ll_mxfp4_threads())

    def gemm(self, x, packed, scales):
        """y[M, R] = x[M, K] @ W^T for packed W[R, K]. x is made a contiguous fp32 tensor."""
        L.require_cuda(x, packed, scales)
        x = x.contiguous().float()
        M, K = x.shape
        R = packed.shape[0]
        assert packed.shape[1] * 2 == K and scales.shape == (R, K // 32), (packed.shape, scales.shape, K)
        packed = packed.contiguous()
        sc, stride = _pad_scales(scales)
        y = torch.empty((M, R), dtype=torch.float32, device=x.device)
        nbytes = self.lib.ll_mxfp4_workspace_bytes(M, K, R)
        ws = torch.empty(nbytes, dtype=torch.uint8, device=x.device)
        L.check(self.lib.ll_mxfp4_gemm(y.data_ptr(), x.data_ptr(), packed.data_ptr(), sc.data_ptr(), M, K, R,
                                       stride, ws.data_ptr(), nbytes, L.stream_ptr()), "ll_mxfp4_gemm")
        return y

    def gemm_t(self, dy, packed, scales):
        """y[M, K] = dy[M, R] @ W for packed W[R, K] (fresh zeros accumulated into, as the reference)."""
        L.require_cuda(dy, packed, scales)
        dy = dy.contiguous().float()
        M, R = dy.shape
        K = packed.shape[1] * 2
        assert packed.shape[0] == R and scales.shape == (R, K // 32)
        packed = packed.contiguous()
        sc, stride = _pad_scales(scales)
        if R % 32:
            pad = (R + 31) // 32 * 32
            dy = torch.nn.functional.pad(dy, (0, pad - R))
            packed = torch.nn.functional.pad(packed, (0, 0, 0, pad - R))
            sc = torch.nn.functional.pad(sc, (0, 0, 0, pad - R))
            R = pad
        y = torch.zeros((M, K), dtype=torch.float32, device=dy.device)
        nbytes = self.lib.ll_mxfp4_workspace_bytes(M, K, R)
        ws = torch.empty(nbytes, dtype=torch.uint8, device=dy.device)
        L.check(self.lib.ll_mxfp4_gemm_t(y.data_ptr(), dy.data_ptr(), packed.data_ptr(), sc.data_ptr(), M, K, R,
                                         stride, ws.data_ptr(), nbytes, L.stream_ptr()), "ll_mxfp4_gemm_t")
        return y

    def dequant(self, packed, scales, out_dtype=torch.float32):
        """W[R, K] from the packed bytes, exact (fp32 like the reference; bf16/fp16 on request)."""
        L.require_cuda(packed, scales)
        R = packed.shape[0]
        K = packed.shape[1] * 2
        packed = packed.contiguous()
        scales = scales.contiguous()
        code = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}[out_dtype]
        w = torch.empty((R, K), dtype=out_dtype, device=packed.device)
        L.check(self.lib.ll_mxfp4_dequant(w.data_ptr(), packed.data_ptr(), scales.data_ptr(), K, R,
                                          scales.shape[1], code, L.stream_ptr()), "ll_mxfp4_dequant")
        return w


_kernel = None


def kernel() -> MXFP4Kernel:
    """The B200 kernel object. Raises (never returns None) when it cannot be used."""
    global _kernel
    if os.environ.get("LAZYLORA_NO_NATIVE", "") == "1":
        raise RuntimeError("LAZYLORA_NO_NATIVE=1: lazylora_b200 has no non-native path to fall back to")
    if _kernel is None:
        if not torch.cuda.is_available():
            raise RuntimeError("lazylora_b200 needs a CUDA device (B200, sm_100a)")
        _kernel = MXFP4Kernel(L.load())
    return _kernel
