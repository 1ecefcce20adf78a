"""
The allocation-free GEMM entry point, ll_mxfp4_gemm_noalloc.

It exists for callers that cannot allocate device memory (a binding holding raw pointers
and no device allocator, or code running where allocation is not allowed): instead of a
caller-sized workspace it uses a static device array inside the library. These checks call
it through the C ABI and compare it with the allocating entry point, ll_mxfp4_gemm, on the
same inputs, for calls in a row of different sizes (each later call finds an earlier call's
leftovers in the shared array), within the GEMM tolerance of the other parity tests
(rel-L2 1e-3); and
check that a size beyond the static array is refused with an error, not run.

This file is named to be collected last, so a run that stops at the first failure has
already run every other test.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 1e-3


def _rel_l2(a, b):
    return float((a.double() - b.double()).norm() / b.double().norm())


def test_noalloc_gemm_matches_workspace_gemm():
    from lazylora_b200 import _lib as L
    lib = L.load()
    g = torch.Generator().manual_seed(11)
    K, R = 7168, 512
    packed = torch.randint(0, 256, (R, K // 2), dtype=torch.uint8, generator=g).cuda()
    scales = torch.randint(112, 126, (R, K // 32), dtype=torch.uint8, generator=g).cuda()
    scales[5, 3] = 255                                    # a damaged group contributes nothing
    stream = torch.cuda.current_stream().cuda_stream
    # calls in a row over the shared array: a three-chunk call (300 rows of 128-row chunks),
    # then smaller ones that must not read the larger call's leftovers (chunk list, rows), one
    # of them not a multiple of 16 rows, then the three-chunk size again
    for call, M in enumerate((300, 48, 37, 300)):
        x = torch.randn(M, K, generator=g).cuda()
        want = torch.empty((M, R), dtype=torch.float32, device="cuda")
        nbytes = lib.ll_mxfp4_workspace_bytes(M, K, R)
        ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
        rc = lib.ll_mxfp4_gemm(want.data_ptr(), x.data_ptr(), packed.data_ptr(), scales.data_ptr(), M, K, R,
                               K // 32, ws.data_ptr(), nbytes, stream)
        assert rc == 0, lib.ll_last_cuda_error()
        got = torch.full((M, R), float("nan"), dtype=torch.float32, device="cuda")
        rc = lib.ll_mxfp4_gemm_noalloc(got.data_ptr(), x.data_ptr(), packed.data_ptr(), scales.data_ptr(), M, K, R,
                                       K // 32, stream)
        assert rc == 0, lib.ll_last_cuda_error()
        torch.cuda.synchronize()
        assert torch.isfinite(got).all(), f"call {call} (M={M})"
        assert _rel_l2(got, want) <= TOL, f"call {call} (M={M})"


def test_noalloc_gemm_refuses_sizes_beyond_its_array():
    from lazylora_b200 import _lib as L
    lib = L.load()
    M, K, R = 1024, 7168, 128                             # 14.7 MB of activations > 8 MiB
    dummy = torch.zeros(16, dtype=torch.uint8, device="cuda")
    rc = lib.ll_mxfp4_gemm_noalloc(dummy.data_ptr(), dummy.data_ptr(), dummy.data_ptr(), dummy.data_ptr(), M, K, R,
                                   K // 32, torch.cuda.current_stream().cuda_stream)
    assert rc == 4                                        # LL_ERR_WORKSPACE
    assert b"scratch" in lib.ll_last_cuda_error()
