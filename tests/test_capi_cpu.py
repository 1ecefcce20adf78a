"""
CPU-side checks of the drop-in boundary: the library loads without a GPU and exports every
function include/lazylora_b200.h declares; the Python mirrors refuse CPU tensors instead of
falling back; the synthetic generator follows the documented distributions.
"""
import ctypes
import os
import re

import pytest
import torch

from lazylora_b200 import _lib, build
from lazylora_b200.synthetic import CONFIGS, make_layer

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "lazylora_b200.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(ll_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    build.build()
    return ctypes.CDLL(build.LIB)


def test_header_symbols_exported(lib):
    names = declared_functions()
    assert len(names) >= 15
    for n in names:
        assert hasattr(lib, n), f"{n} declared in include/lazylora_b200.h but not exported"


def test_binding_covers_header():
    assert set(declared_functions()) == set(_lib.exported_symbols())


def test_status_strings_without_gpu():
    L = _lib.load()
    assert L.ll_status_string(0) == b"ok"
    assert b"timed out" in L.ll_status_string(3)


def test_no_cpu_fallback():
    from lazylora_b200.native import MXFP4Kernel
    k = MXFP4Kernel(_lib.load())
    with pytest.raises(ValueError):
        k.gemm(torch.zeros(2, 32), torch.zeros(4, 16, dtype=torch.uint8), torch.zeros(4, 1, dtype=torch.uint8))


def test_kernel_raises_without_gpu_or_when_disabled(monkeypatch):
    import lazylora_b200.native as native
    monkeypatch.setenv("LAZYLORA_NO_NATIVE", "1")
    with pytest.raises(RuntimeError):
        native.kernel()


def test_workspace_sizes():
    L = _lib.load()
    d = _lib.MoELayerDesc()
    d.d, d.f, d.E, d.r = 7168, 2048, 896, 16
    n = L.ll_moe_workspace_bytes(ctypes.byref(d), 1024, 8)
    assert 0.5e9 < n < 2e9          # the activations of one 1024-token layer
    assert L.ll_mxfp4_workspace_bytes(16, 7168, 2048) > 16 * 7168 * 2


def test_synthetic_distributions():
    cfg = CONFIGS["tiny"]
    inp = make_layer(cfg)
    s = inp["w1s"]
    assert int(s.min()) >= 117 and int(s.max()) <= 121
    p = inp["w2p"]
    assert p.dtype == torch.uint8 and p.shape == (cfg.E, cfg.d, cfg.f // 2)
    # deterministic
    inp2 = make_layer(cfg)
    assert torch.equal(inp["w1p"], inp2["w1p"]) and torch.equal(inp["x"], inp2["x"])


def test_lora_entry_points_check_arguments_without_gpu():
    """Shape and workspace checks of the LoRA products return before any CUDA call."""
    L = _lib.load()
    p = ctypes.c_void_p(16)                      # never dereferenced: the checks come first
    one = ctypes.c_float(1.0)
    # K % 8 != 0
    assert L.ll_lora_down(p, 1, 4, 12, p, None, 4, 4, 1, one, p, None, p, 1 << 20, None) == 1
    # n0 > n; columns form with n0 != n
    assert L.ll_lora_down(p, 1, 4, 64, p, None, 8, 4, 1, one, p, None, p, 1 << 20, None) == 1
    assert L.ll_lora_down(p, 1, 4, 64, p, None, 4, 8, 0, one, p, None, p, 1 << 20, None) == 1
    # a pair of row blocks without the second matrix
    assert L.ll_lora_down(p, 1, 4, 64, p, None, 4, 8, 1, one, p, None, p, 1 << 20, None) == 1
    # workspace below one split of M x n
    assert L.ll_lora_down(p, 1, 64, 64, p, None, 16, 16, 1, one, p, None, p, 4 * 64 * 16 - 4, None) == 4
    assert L.ll_lora_down(p, 1, 0, 64, p, None, 16, 16, 1, one, p, None, p, 0, None) == 0     # M = 0
    # C % 4 != 0; workspace below r x C
    assert L.ll_lora_outer(p, p, 1, 8, 30, 4, one, 0, p, p, 1 << 20, None) == 1
    assert L.ll_lora_outer(p, p, 1, 8, 32, 4, one, 0, p, p, 4 * 32 * 4 - 4, None) == 4
    # rank outside {4, 8, 16, 32}
    assert L.ll_lora_add_bf16(p, p, p, None, None, 12, 1, one, 8, 64, p, None) == 1
    assert L.ll_lora_add_bf16(p, p, p, None, None, 16, 1, one, 0, 64, p, None) == 0          # N = 0


def test_shared_expert_refuses_cpu_tensors():
    """The shared expert has no CPU path: CPU weights are refused, not computed on the host."""
    from lazylora_b200.trainer.shared_expert import SharedExpert
    d, F, r = 64, 96, 4
    W = lambda o, i: torch.zeros(o, i, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        SharedExpert(W(F, d), W(F, d), W(d, F), torch.zeros(r, d), torch.zeros(F, r), torch.zeros(r, d),
                     torch.zeros(F, r), torch.zeros(r, F), torch.zeros(d, r), 2.0)
