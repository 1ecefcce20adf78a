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
from typing import Dict

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


def latent_block(k: "O.MXFP4Checker", layer: "O.Layer", x, down_w, up_w, norm_w, idx, w, grad_out=None,
                 eps: float = 1e-5) -> Dict[str, torch.Tensor]:
    """Forward (and, with grad_out, backward) of the latent routed block. x bf16 [N, d_h];
    down_w [d_l, d_h], up_w [d_h, d_l] bf16; norm_w [d_l]. LoRA gradients accumulate into
    layer.{gate, up, down}."""
    h_lat = linear32(x, down_w)                                   # bf16 [N, d_l]
    routed = O.experts_forward(k, layer, h_lat, idx, w)           # fp32 [N, d_l]
    res = {"h_latent": h_lat, "routed": routed}
    routed_req = routed.clone().requires_grad_(True)
    normed = rmsnorm(routed_req, norm_w.to(routed.dtype), eps)
    normed_bf = normed.to(up_w.dtype)
    out = linear32(normed_bf, up_w)                               # bf16 [N, d_h]
    res["out"] = out
    if grad_out is None:
        return res
    g_normed_bf = linear32_grad_x(grad_out, up_w, normed_bf.dtype)
    (g_routed,) = torch.autograd.grad(normed_bf, routed_req, g_normed_bf)
    g_h, g_w = O.experts_backward(k, layer, h_lat, idx, w, g_routed.float())
    res["grad_x"] = linear32_grad_x(g_h, down_w, x.dtype)
    res["grad_w"] = g_w
    res["grad_routed"] = g_routed
    return res
