"""
The latent routed-expert block of a Kimi K3 MoE layer on the GPU.

Kimi K3 runs its routed experts in a narrower latent space (lazy_lora/trainer/
lazy_trainer.py:697-736): the normed hidden state is projected down (routed_expert_down_proj,
[d_l, d_h] bf16), the routed experts run on the latent rows and their fp32 sum is RMS-normed
(routed_expert_norm, trunk_streamer.py:27-31), cast to bf16 and projected back up
(routed_expert_up_proj, [d_h, d_l]). Here:

  * the two dense projections are plain bf16 GEMMs with fp32 accumulation, as F.linear
    computes them on CUDA in the reference, on this library's tcgen05 GEMM (core.dense);
  * the routed experts are a RoutedExpertsLayer at width d_l (this library's grouped MXFP4
    kernels);
  * the RMSNorm is fused into the routed experts' final combine (ll_moe_forward_rmsnorm: each
    token's rows summed, then normalised, written straight to bf16 for the up-projection, and
    its rsqrt kept); its gradient is this library's row kernel (ll_rmsnorm_backward).

The backward follows the autograd graph of the reference: the up-projection's input gradient,
the RMSNorm gradient for a frozen norm weight, the routed experts' backward (its grad_h cast to
h_latent's bf16), the down-projection's input gradient. The projections and the norm weight are
frozen (LoRA training); the routed experts' LoRA gradients come back as from the layer.
"""
from typing import Dict, Tuple

import torch

from .. import _lib as L
from ..core import dense
from .routed_experts import RoutedExpertsLayer


class LatentRoutedMoE:
    """down_w [d_l, d_h], up_w [d_h, d_l] (bf16, frozen), norm_w [d_l]; layer: the routed
    experts at width d_l."""

    def __init__(self, layer: RoutedExpertsLayer, down_w: torch.Tensor, up_w: torch.Tensor, norm_w: torch.Tensor,
                 eps: float = 1e-5):
        L.require_cuda(down_w, up_w, norm_w)
        d_l, d_h = down_w.shape
        if tuple(up_w.shape) != (d_h, d_l) or tuple(norm_w.shape) != (d_l,) or layer.d != d_l:
            raise ValueError("down_w [d_l, d_h], up_w [d_h, d_l], norm_w [d_l] and a layer of width d_l")
        self.layer = layer
        self.down_w = down_w.to(torch.bfloat16).contiguous()
        self.up_w = up_w.to(torch.bfloat16).contiguous()
        self.norm_w = norm_w.to(torch.float32).contiguous()
        self.eps = float(eps)
        self.lib = L.load()
        self._saved = None

    def forward(self, x: torch.Tensor, idx: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        """routed_out [N, d_h] bf16 for the normed hidden state x [N, d_h]."""
        L.require_cuda(x, idx, w)
        xb = x.reshape(-1, self.down_w.shape[1]).to(torch.bfloat16)
        h_lat = dense.linear(xb, self.down_w).contiguous()                # bf16 [N, d_l]
        # the routed experts, their combine and the RMSNorm of the fp32 sum in the same final pass
        routed, normed, rstd = self.layer.forward_rmsnorm(h_lat, idx, w, self.norm_w, self.eps)
        out = dense.linear(normed, self.up_w).contiguous()                 # bf16 [N, d_h]
        self._saved = (h_lat, routed, rstd, idx, w)
        return out

    def backward(self, grad_out: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor, Dict[str, torch.Tensor]]:
        """(grad_x [N, d_h] bf16, grad_w [N, k] fp32, LoRA gradients) of the last forward."""
        if self._saved is None:
            raise RuntimeError("backward before forward")
        h_lat, routed, rstd, idx, w = self._saved
        N, D = routed.shape
        g_normed = dense.matmul(grad_out.reshape(N, -1).to(torch.bfloat16), self.up_w).contiguous()  # bf16 [N, d_l]
        g_routed = torch.empty((N, D), dtype=torch.float32, device=routed.device)
        L.check(self.lib.ll_rmsnorm_backward(routed.data_ptr(), self.norm_w.data_ptr(), rstd.data_ptr(),
                                             g_normed.data_ptr(), 1, N, D, g_routed.data_ptr(), L.stream_ptr()),
                "ll_rmsnorm_backward")
        g_h, g_w, grads = self.layer.backward(h_lat, idx, w, g_routed)
        grad_x = dense.matmul(g_h.to(torch.bfloat16), self.down_w).contiguous()             # bf16 [N, d_h]
        return grad_x, g_w, grads
