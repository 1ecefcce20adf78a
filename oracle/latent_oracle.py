"""
CPU oracle for the latent routed-expert block of a Kimi K3 MoE layer. TEST INFRASTRUCTURE ONLY
(imported by tests/ as the checker; the product package never imports it).

Restates lazy_lora/trainer/lazy_trainer.py:722-735 (the routed half of _moe_forward) on CPU:

  h_latent = linear32(x, routed_expert_down_proj)       lazy_lora/core/linear32.py:17-35
  routed   = routed experts (fp32 sum)                   moe_oracle.experts_forward
  normed   = RMSNormFunction.forward(routed, norm_w)     lazy_lora/streaming/trunk_streamer.py:27-31
  out      = linear32(normed.to(bf16), routed_expert_up_proj)

and its backward the way autograd runs it there: _Linear32.backward (grad_x = grad_out.float()
@ W.float(), cast to the input's dtype), the cast and the RMSNorm ops differentiated in fp32,
RoutedExpertsFunction.backward (moe_oracle.experts_backward; its grad_h is cast to h_latent's
dtype), then the down projection's _Linear32.backward.
"""
from typing import Callable, Dict

import torch

from . import moe_oracle as O


def linear32(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """x @ w.T with the product in fp32, result in x's dtype (linear32.py:20-22)."""
    return torch.nn.functional.linear(x.float(), w.float()).to(x.dtype)


def linear32_grad_x(g: torch.Tensor, w: torch.Tensor, x_dtype) -> torch.Tensor:
    """_Linear32.backward: grad_out.float() @ W.float(), cast to the input's dtype (linear32.py:25-28)."""
    return torch.matmul(g.float(), w.float()).to(x_dtype)


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
    """RMSNormFunction.forward on a tensor (trunk_streamer.py:27-31)."""
    variance = x.pow(2).mean(-1, keepdim=True)
    return x * torch.rsqrt(variance + eps) * w


def latent_block_with(experts_fwd: Callable, experts_bwd: Callable, x, down_w, up_w, norm_w, idx, w,
                      grad_out=None, eps: float = 1e-5) -> Dict[str, torch.Tensor]:
    """The block's composition around any routed-expert sweep: experts_fwd(h, idx, w) -> fp32
    [N, d_l] (the routed sum) and experts_bwd(h, idx, w, g) -> (grad_h, grad_w).

    Forward: h_latent = linear32(x, down_w); routed = experts_fwd(h_latent); normed =
    rmsnorm(routed) cast to the up-projection's dtype; out = linear32(normed, up_w).
    Backward, the order autograd runs it in the reference's replay: the up-projection's
    _Linear32.backward, the cast and the RMSNorm differentiated in fp32, the routed experts'
    manual backward, the down-projection's _Linear32.backward."""
    h_lat = linear32(x, down_w)
    routed = experts_fwd(h_lat, idx, w)
    res = {"h_latent": h_lat, "routed": routed}
    routed_req = routed.clone().requires_grad_(True)
    normed = rmsnorm(routed_req, norm_w.to(routed.dtype), eps)
    normed_c = normed.to(up_w.dtype)
    out = linear32(normed_c, up_w)
    res["out"] = out.detach()
    if grad_out is None:
        return res
    g_normed = linear32_grad_x(grad_out, up_w, normed_c.dtype)
    (g_routed,) = torch.autograd.grad(normed_c, routed_req, g_normed)
    g_h, g_w = experts_bwd(h_lat, idx, w, g_routed.float())
    res["grad_x"] = linear32_grad_x(g_h, down_w, x.dtype)
    res["grad_w"] = g_w
    res["grad_routed"] = g_routed
    return res


def latent_block(k: "O.MXFP4Checker", layer: "O.Layer", x, down_w, up_w, norm_w, idx, w, grad_out=None,
                 eps: float = 1e-5) -> Dict[str, torch.Tensor]:
    """Forward (and, with grad_out, backward) of the latent routed block with MXFP4 experts.
    x bf16 [N, d_h]; down_w [d_l, d_h], up_w [d_h, d_l] bf16; norm_w [d_l]. LoRA gradients
    accumulate into layer.{gate, up, down}."""
    return latent_block_with(lambda h, i, ww: O.experts_forward(k, layer, h, i, ww),
                             lambda h, i, ww, g: O.experts_backward(k, layer, h, i, ww, g),
                             x, down_w, up_w, norm_w, idx, w, grad_out, eps)


def dense_experts_forward(h, idx, w, experts, beta: float = O.SITU_BETA, linear_beta: float = O.SITU_LINEAR_BETA):
    """_routed_experts_forward (lazy_trainer.py:806-834) with dense fp32 expert weights
    experts[e] = (W1 [f, d], W3 [f, d], W2 [d, f]) and no LoRA: the form the reference's vendored
    MoE-block fixture records (lazy_lora/tests/test_reference_ops.py:259-309). Differentiable."""
    out = torch.zeros(h.shape, dtype=torch.float32)
    for e in O.active_experts(idx):
        if e < 0:
            continue
        mask = idx == e
        rows = mask.any(-1).nonzero().squeeze(-1)
        xe = h.float().index_select(0, rows)
        W1, W3, W2 = experts[e]
        act = O.situ_glu_forward(torch.nn.functional.linear(xe, W1), torch.nn.functional.linear(xe, W3),
                                 beta, linear_beta)
        tw = (w.index_select(0, rows) * mask.index_select(0, rows).to(w.dtype)).sum(-1, keepdim=True)
        out = out.index_add(0, rows, torch.nn.functional.linear(act, W2) * tw)
    return out


def dense_experts_backward(h, idx, w, g, experts, beta: float = O.SITU_BETA,
                           linear_beta: float = O.SITU_LINEAR_BETA):
    """(grad_h, grad_w) of dense_experts_forward for upstream gradient g, by autograd."""
    hr = h.detach().float().clone().requires_grad_(True)
    wr = w.detach().clone().requires_grad_(True)
    out = dense_experts_forward(hr, idx, wr, experts, beta, linear_beta)
    gh, gw = torch.autograd.grad(out, (hr, wr), g)
    return gh, gw
