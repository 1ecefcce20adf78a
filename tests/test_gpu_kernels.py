"""
GPU parity of the drop-in kernels and the router against the CPU oracle (oracle/), through
the C ABI. Bars: dequant bit-exact; GEMMs rel-L2 <= 1e-3 (fp16 operands, fp32 accumulate;
the layer bar is 2e-3); router selection bit-exact on identical scores.
"""
import pytest
import torch

from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def kern():
    from lazylora_b200.native import kernel
    return kernel()


@pytest.fixture(scope="module")
def ok():
    return O.MXFP4Checker("oracle")


def _weights(R, K, gen, lo=110, hi=130, damaged=True):
    packed = torch.randint(0, 256, (R, K // 2), dtype=torch.uint8, generator=gen)
    scales = torch.randint(lo, hi + 1, (R, K // 32), dtype=torch.uint8, generator=gen)
    if damaged and R > 2:
        scales[1, 0] = 253
        scales[2, -1] = 255
    return packed, scales


def test_dequant_bit_exact(kern, ok):
    g = torch.Generator().manual_seed(1)
    # every scale byte 0..255 across the rows of one matrix
    R, K = 256, 64
    packed = torch.randint(0, 256, (R, K // 2), dtype=torch.uint8, generator=g)
    scales = torch.stack([torch.arange(256, dtype=torch.uint8), torch.arange(256, dtype=torch.uint8).flip(0)], 1)
    want = ok.dequant(packed, scales)
    got = kern.dequant(packed.cuda(), scales.cuda()).cpu()
    assert torch.equal(got.view(torch.int32), want.view(torch.int32))
    assert torch.all(got.view(R, 2, 32)[scales >= 253] == 0)
    # bf16 output is exact for every byte; fp16 within 104..140
    got16 = kern.dequant(packed.cuda(), scales.cuda(), out_dtype=torch.bfloat16).cpu()
    assert torch.equal(got16, want.to(torch.bfloat16))
    p2, s2 = _weights(64, 512, g, 104, 140, damaged=False)
    assert torch.equal(kern.dequant(p2.cuda(), s2.cuda(), out_dtype=torch.float16).cpu(),
                       ok.dequant(p2, s2).to(torch.float16))


@pytest.mark.parametrize("M,K,R", [(1, 32, 128), (5, 256, 200), (37, 1024, 384), (130, 2048, 256),
                                   (16, 7168, 256), (9, 3584, 3072)])
def test_gemm(kern, ok, M, K, R):
    g = torch.Generator().manual_seed(M * 7 + K + R)
    packed, scales = _weights(R, K, g)
    x = torch.randn(M, K, generator=g)
    want = ok.gemm(x, packed, scales)
    got = kern.gemm(x.cuda(), packed.cuda(), scales.cuda()).cpu()
    assert O.rel_l2(got, want) < 1e-3


@pytest.mark.parametrize("M,K,R", [(1, 128, 32), (5, 256, 200), (37, 1024, 384), (130, 2048, 256),
                                   (16, 7168, 256), (9, 3584, 3072)])
def test_gemm_t(kern, ok, M, K, R):
    g = torch.Generator().manual_seed(M * 11 + K + R)
    packed, scales = _weights(R, K, g)
    dy = torch.randn(M, R, generator=g)
    want = ok.gemm_t(dy, packed, scales)
    got = kern.gemm_t(dy.cuda(), packed.cuda(), scales.cuda()).cpu()
    assert O.rel_l2(got, want) < 1e-3


def test_gemm_wide_scale_range(kern, ok):
    """Scale bytes spanning 36 binades below the maximum still decode exactly (decode bias)."""
    g = torch.Generator().manual_seed(3)
    packed, scales = _weights(128, 512, g, 150 - 36, 150, damaged=False)
    x = torch.randn(4, 512, generator=g)
    assert O.rel_l2(kern.gemm(x.cuda(), packed.cuda(), scales.cuda()).cpu(), ok.gemm(x, packed, scales)) < 1e-3


def test_route_select_bit_exact():
    from lazylora_b200.core.moe_router import route_select
    g = torch.Generator().manual_seed(4)
    for (T, E, k) in [(6, 8, 2), (64, 896, 8), (33, 896, 16), (5, 1500, 8)]:
        scores = torch.sigmoid(torch.randn(T, E, generator=g))
        bias = torch.randn(E, generator=g) * 0.05
        sfc = scores + bias
        want_i, want_w = O.route_select(scores, sfc, k)
        got_i, got_w = route_select(scores.cuda(), sfc.cuda(), k)
        assert torch.equal(got_i.cpu(), want_i)
        ulp = (got_w.cpu() - want_w).abs() / torch.finfo(torch.float32).eps / want_w.abs()
        assert float(ulp.max()) <= 1.0


def test_route_select_block_path_equals_warp_path():
    """Up to 256 tokens the selection runs a block per token (8 warps over slices of the
    experts, then a merge); above that a warp per token. The first rows of a 300-token batch
    select the same ids with the same weight bits either way, also with many tied scores
    (scores rounded to 1/64: ties broken to the lower id) and k = 16, 32."""
    from lazylora_b200.core.moe_router import route_select
    g = torch.Generator().manual_seed(14)
    for (E, k, tied) in [(896, 8, False), (896, 8, True), (384, 16, True), (1024, 32, False), (64, 8, True)]:
        scores = torch.sigmoid(torch.randn(300, E, generator=g))
        if tied:
            scores = torch.round(scores * 64) / 64
        sfc = scores + (0 if tied else torch.randn(E, generator=g) * 0.05)
        big_i, big_w = route_select(scores.cuda(), sfc.cuda(), k)          # warp per token
        small_i, small_w = route_select(scores[:37].cuda(), sfc[:37].cuda(), k)   # block per token
        assert torch.equal(small_i, big_i[:37]), (E, k, tied)
        assert torch.equal(small_w.view(torch.int32), big_w[:37].view(torch.int32)), (E, k, tied)
        if not tied:    # (torch.topk leaves the order of ties unspecified)
            want_i, _ = O.route_select(scores[:37], sfc[:37], k)
            assert torch.equal(small_i.cpu(), want_i), (E, k, tied)


def test_router_forward_matches_reference_routing():
    from lazylora_b200.core.moe_router import KimiK3MoERouter
    g = torch.Generator().manual_seed(5)
    T, d, E, k = 256, 7168, 896, 8
    x = torch.randn(T, d, generator=g)
    W = torch.randn(E, d, generator=g) * 0.02
    b = torch.randn(E, generator=g) * 0.01
    want_i, want_w = O.route(x, W, b, k)
    r = KimiK3MoERouter(hidden_size=d, num_experts=E, top_k=k)
    got_i, got_w = r.forward(x.cuda(), weight=W.cuda(), bias=b.cuda())
    got_i, got_w = got_i.cpu(), got_w.cpu()
    # logits differ from the CPU GEMM in the last bits: any selection difference must be a near-tie
    sfc = torch.sigmoid(torch.nn.functional.linear(x, W)) + b
    mism = 0
    for t in range(T):
        if set(got_i[t].tolist()) != set(want_i[t].tolist()):
            mism += 1
            srt = sfc[t].sort(descending=True).values
            assert float(srt[k - 1] - srt[k]) < 1e-5 * float(srt[k - 1].abs()) + 1e-7
    assert mism <= 2
    same = (got_i == want_i).all(-1)
    assert O.rel_l2(got_w[same], want_w[same]) < 1e-5


def test_router_fixture(golden_dir):
    import numpy as np
    import os
    from lazylora_b200.core.moe_router import KimiK3MoERouter
    fx = np.load(os.path.join(golden_dir, "fx_router.npz"))
    x = torch.from_numpy(fx["in"]).cuda()
    r = KimiK3MoERouter(hidden_size=x.shape[-1], num_experts=int(fx["n_experts"]), top_k=int(fx["top_k"]))
    idx, w = r.forward(x, weight=torch.from_numpy(fx["gate_weight"]).cuda(), bias=torch.from_numpy(fx["bias"]).cuda())
    got = {(i, int(e)): float(v) for i, (ee, ww) in enumerate(zip(idx.tolist(), w.tolist())) for e, v in zip(ee, ww)}
    want = {(i, int(e)): float(v) for i, (ee, ww) in enumerate(zip(fx["topk_idx"].astype(int).tolist(),
                                                                     fx["topk_weight"].tolist())) for e, v in zip(ee, ww)}
    assert sorted(got) == sorted(want)
    for key in want:
        assert abs(got[key] - want[key]) <= 1e-5 + 1e-4 * abs(want[key])


def test_router_prepared_planes_bit_exact():
    """The weight split made once (ll_route_prepare) and reused (ll_route_topk_prepared) routes
    exactly as the per-call split (ll_route_topk), for bf16 and fp32 activations; the router
    module re-splits when its weight changes."""
    import ctypes
    from lazylora_b200 import _lib as L
    from lazylora_b200.core.moe_router import KimiK3MoERouter
    lib = L.load()
    g = torch.Generator().manual_seed(8)
    T, d, E, k = 40, 7168, 896, 8
    W = (torch.randn(E, d, generator=g) * 0.02).cuda()
    b = (torch.randn(E, generator=g) * 0.01).cuda()
    planes = torch.empty((3, E, d), dtype=torch.bfloat16, device="cuda")
    assert lib.ll_route_prepare(W.data_ptr(), E, d, planes.data_ptr(), L.stream_ptr()) == 0
    for xd in (torch.float32, torch.bfloat16):
        x = torch.randn(T, d, generator=g).cuda().to(xd)
        code = 0 if xd == torch.float32 else 1
        nb = lib.ll_route_workspace_bytes(T, d, E)
        ws = torch.empty(nb, dtype=torch.uint8, device="cuda")
        out = []
        for prepared in (False, True):
            idx = torch.empty((T, k), dtype=torch.int64, device="cuda")
            w = torch.empty((T, k), dtype=torch.float32, device="cuda")
            if prepared:
                rc = lib.ll_route_topk_prepared(x.data_ptr(), code, planes.data_ptr(), b.data_ptr(), T, d, E, k, 1,
                                                ctypes.c_float(1.0), idx.data_ptr(), w.data_ptr(), None, ws.data_ptr(),
                                                nb, L.stream_ptr())
            else:
                rc = lib.ll_route_topk(x.data_ptr(), code, W.data_ptr(), b.data_ptr(), T, d, E, k, 1,
                                       ctypes.c_float(1.0), idx.data_ptr(), w.data_ptr(), None, ws.data_ptr(), nb,
                                       L.stream_ptr())
            assert rc == 0, lib.ll_last_cuda_error()
            out.append((idx, w))
        assert torch.equal(out[0][0], out[1][0]) and torch.equal(out[0][1], out[1][1])
    r = KimiK3MoERouter(hidden_size=d, num_experts=E, top_k=k)
    x = torch.randn(T, d, generator=g).cuda().to(torch.bfloat16)
    with torch.no_grad():
        r.weight.copy_(W)
        r.bias.copy_(b)
    i0, _ = r.forward(x)
    with torch.no_grad():
        r.weight.mul_(-1.0)                                  # a changed weight is split again
    i1, _ = r.forward(x)
    want, _ = KimiK3MoERouter.forward(KimiK3MoERouter(hidden_size=d, num_experts=E, top_k=k), x, weight=-W, bias=b)
    assert torch.equal(i1, want) and not torch.equal(i0, i1)
