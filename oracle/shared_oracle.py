"""
CPU oracle for the shared expert of a Kimi K3 MoE layer. TEST INFRASTRUCTURE ONLY (imported
by tests/ as the checker; the product package never imports it).

Restates lazy_lora/trainer/lazy_trainer.py:702-707 on CPU with the reference's building
blocks and lets torch autograd produce the backward, as the reference's replay does:

  linear32           lazy_lora/core/linear32.py:17-35 (fp32 product, result in x's dtype;
                     backward grad_out.float() @ W.float(), cast to x's dtype)
  forward_lora_only  lazy_lora/core/lora_layer.py:104-123 (bf16 input cast to fp32,
                     (x A^T) B^T * scaling, cast back to bf16)
  situ_glu_forward   lazy_lora/core/situ_activation.py:47-75 (fp32 inside, input dtype out)
"""
from typing import Dict

import torch
import torch.nn.functional as F

from . import moe_oracle as O


class _Linear32(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight):
        ctx.save_for_backward(weight)
        ctx.x_dtype = x.dtype
        return F.linear(x.float(), weight.float()).to(x.dtype)

    @staticmethod
    def backward(ctx, grad_out):
        (weight,) = ctx.saved_tensors
        return torch.matmul(grad_out.float(), weight.float()).to(ctx.x_dtype), None


def lora_delta(x, A, B, scaling):
    xd = x.to(A.dtype)
    return (F.linear(F.linear(xd, A), B) * scaling).to(x.dtype)


def situ_glu(gate, up, beta: float = O.SITU_BETA, linear_beta: float = O.SITU_LINEAR_BETA):
    g, u = gate.float(), up.float()
    a = beta * torch.tanh(g / beta) * torch.sigmoid(g)
    return (a * (linear_beta * torch.tanh(u / linear_beta))).to(gate.dtype)


def shared_expert(x, W_g, W_u, W_d, ad: Dict[str, torch.Tensor], scaling: float, grad_out=None):
    """Forward (and with grad_out, backward) of the shared expert. x bf16 [N, d]; W bf16;
    ad: A_g, B_g, A_u, B_u, A_d, B_d fp32. Returns out, and grad_x plus the six LoRA grads."""
    xr = x.detach().clone().requires_grad_(True)
    P = {k: v.detach().clone().requires_grad_(True) for k, v in ad.items()}
    s_gate = _Linear32.apply(xr, W_g) + lora_delta(xr, P["A_g"], P["B_g"], scaling)
    s_up = _Linear32.apply(xr, W_u) + lora_delta(xr, P["A_u"], P["B_u"], scaling)
    h = situ_glu(s_gate, s_up)
    out = _Linear32.apply(h, W_d) + lora_delta(h, P["A_d"], P["B_d"], scaling)
    res = {"out": out.detach()}
    if grad_out is not None:
        out.backward(grad_out)
        res["grad_x"] = xr.grad
        for k in ("A_g", "B_g", "A_u", "B_u", "A_d", "B_d"):
            res["d" + k] = P[k].grad
    return res
