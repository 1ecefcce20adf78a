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
