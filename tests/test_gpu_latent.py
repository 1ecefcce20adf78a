"""
GPU parity of the latent routed-expert block (down-projection, routed experts at the latent
width, RMSNorm of their fp32 sum, up-projection; lazy_lora/trainer/lazy_trainer.py:722-735)
against the CPU restatement in oracle/latent_oracle.py, forward and backward.

Tolerances: fp32 quantities (the routed sum, its gradient, grad_w, the LoRA gradients) within
relative L2 2e-3, the bar the path's other outputs meet. The block's input and output are bf16
(the reference casts to bf16 before each projection): one bf16 ulp is 2^-8 = 3.9e-3 relative,
and two fp32 accumulation orders round a share of the elements to neighbouring bf16 values, so
the bf16 outputs (out, grad_x) are held to 5e-3.
"""
import pytest
import torch

from lazylora_b200.synthetic import CONFIGS, make_layer
from oracle import latent_oracle as LO
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu

TOL = 2e-3
TOL_BF16 = 5e-3


def _case(d_h, cfg, seed=11):
    gen = torch.Generator().manual_seed(seed)
    inp = make_layer(cfg)
    d_l = cfg.d
    down_w = (torch.randn(d_l, d_h, generator=gen) / d_h ** 0.5).to(torch.bfloat16)
    up_w = (torch.randn(d_h, d_l, generator=gen) / d_l ** 0.5).to(torch.bfloat16)
    norm_w = 1.0 + 0.1 * torch.randn(d_l, generator=gen)
    x = torch.randn(cfg.T, d_h, generator=gen).to(torch.bfloat16)
    router_w = torch.randn(cfg.E, d_h, generator=gen) * 0.05
    idx, w = O.route(x.float(), router_w, torch.zeros(cfg.E), cfg.k)
    g = torch.randn(cfg.T, d_h, generator=gen).to(torch.bfloat16)
    return inp, down_w, up_w, norm_w, x, idx, w, g


@pytest.mark.parametrize("d_h,case", [(512, "tiny"), (2048, "small")])
def test_latent_block_matches_oracle(d_h, case):
    from lazylora_b200.trainer.latent_moe import LatentRoutedMoE
    from lazylora_b200.trainer.routed_experts import RoutedExpertsLayer
    cfg = CONFIGS[case]
    inp, down_w, up_w, norm_w, x, idx, w, g = _case(d_h, cfg)
    k = O.MXFP4Checker()
    layer_o = O.Layer.from_inputs(inp, cfg.scaling)
    want = LO.latent_block(k, layer_o, x, down_w, up_w, norm_w, idx, w, grad_out=g)

    layer = RoutedExpertsLayer.from_inputs(inp, cfg.scaling)
    blk = LatentRoutedMoE(layer, down_w.cuda(), up_w.cuda(), norm_w.cuda())
    out = blk.forward(x.cuda(), idx.cuda(), w.cuda())
    gx, gw, grads = blk.backward(g.cuda())
    layer.check_status(cfg.T, cfg.k)
    assert out.dtype == torch.bfloat16 and gx.dtype == torch.bfloat16
    assert O.rel_l2(out.cpu(), want["out"]) < TOL_BF16
    assert O.rel_l2(gx.cpu(), want["grad_x"]) < TOL_BF16
    assert O.rel_l2(gw.cpu(), want["grad_w"]) < TOL
    for key, lo in (("dA_g", layer_o.gate.grad_A), ("dB_g", layer_o.gate.grad_B), ("dA_u", layer_o.up.grad_A),
                    ("dB_u", layer_o.up.grad_B), ("dA_d", layer_o.down.grad_A), ("dB_d", layer_o.down.grad_B)):
        assert O.rel_l2(grads[key].cpu(), lo) < TOL, key


def test_rmsnorm_kernels_match_torch():
    """The row kernels against the reference formula and its autograd gradient, fp32 and
    bf16 outputs, a row width that is not a multiple of the block."""
    import ctypes
    from lazylora_b200 import _lib as L
    lib = L.load()
    gen = torch.Generator().manual_seed(2)
    N, D = 37, 3584 + 40
    x = torch.randn(N, D, generator=gen) * 3.0
    wn = 1.0 + 0.2 * torch.randn(D, generator=gen)
    gy = torch.randn(N, D, generator=gen)
    xr = x.clone().requires_grad_(True)
    y = LO.rmsnorm(xr, wn)
    (gx_want,) = torch.autograd.grad(y, xr, gy)
    xd, wd, gyd = x.cuda(), wn.cuda(), gy.cuda()
    y32 = torch.empty(N, D, device="cuda")
    ybf = torch.empty(N, D, dtype=torch.bfloat16, device="cuda")
    rstd = torch.empty(N, device="cuda")
    gx = torch.empty(N, D, device="cuda")
    s = L.stream_ptr()
    L.check(lib.ll_rmsnorm_forward(xd.data_ptr(), wd.data_ptr(), N, D, ctypes.c_float(1e-5), y32.data_ptr(), 0,
                                   rstd.data_ptr(), s), "fwd")
    L.check(lib.ll_rmsnorm_forward(xd.data_ptr(), wd.data_ptr(), N, D, ctypes.c_float(1e-5), ybf.data_ptr(), 1,
                                   None, s), "fwd bf16")
    L.check(lib.ll_rmsnorm_backward(xd.data_ptr(), wd.data_ptr(), rstd.data_ptr(), gyd.data_ptr(), 0, N, D,
                                    gx.data_ptr(), s), "bwd")
    torch.cuda.synchronize()
    assert O.rel_l2(y32.cpu(), y.detach()) < 1e-6
    assert O.rel_l2(ybf.float().cpu(), y.detach().to(torch.bfloat16).float()) < 4e-3
    assert O.rel_l2(gx.cpu(), gx_want) < 1e-5


@pytest.mark.parametrize("case", ["tiny", "small"])
def test_fused_combine_norm_matches_separate_passes(case):
    """ll_moe_forward_rmsnorm: its fp32 output is ll_moe_forward's bit for bit (the same sums),
    and its normed rows and rstd are the row kernel's on that output (the squares summed in
    another fixed order: rstd within 1e-6, the bf16 rows within one rounding)."""
    import ctypes
    from lazylora_b200 import _lib as L
    from lazylora_b200.trainer.routed_experts import RoutedExpertsLayer
    cfg = CONFIGS[case]
    inp, _, _, norm_w, _, _, _, _ = _case(256, cfg)
    layer = RoutedExpertsLayer.from_inputs(inp, cfg.scaling)
    h = inp["x"].cuda()
    idx, w = O.route(inp["x"].float(), inp["router_w"], inp["router_b"], cfg.k)
    idx, w = idx.cuda(), w.cuda()
    nw = norm_w.cuda()
    out_a = layer.forward(h, idx, w)
    out_b, normed, rstd = layer.forward_rmsnorm(h, idx, w, nw, 1e-5)
    layer.check_status(cfg.T, cfg.k)
    assert torch.equal(out_a, out_b)
    lib = L.load()
    T, D = out_a.shape
    y = torch.empty(T, D, dtype=torch.bfloat16, device="cuda")
    r2 = torch.empty(T, device="cuda")
    L.check(lib.ll_rmsnorm_forward(out_a.data_ptr(), nw.data_ptr(), T, D, ctypes.c_float(1e-5), y.data_ptr(), 1,
                                   r2.data_ptr(), L.stream_ptr()), "ll_rmsnorm_forward")
    assert float(((rstd - r2).abs() / r2).max()) < 1e-6
    want = (out_a * r2[:, None] * nw[None, :])
    err = (normed.float() - want).abs()
    assert bool((err <= want.abs() * 2 ** -8 + 1e-6).all())
