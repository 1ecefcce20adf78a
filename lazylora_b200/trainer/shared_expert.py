"""
The shared expert of a Kimi K3 MoE layer on the GPU: a dense SiTU-GLU MLP (d -> F -> d, bf16
weights, frozen) with a rank-r LoRA adapter on each of its three projections
(lazy_lora/trainer/lazy_trainer.py:702-707):

    s_gate = linear32(x, W_g) + lora_g(x),  s_up = linear32(x, W_u) + lora_u(x)
    h      = situ_glu(s_gate, s_up)
    out    = linear32(h, W_d) + lora_d(h)

The three projections are bf16 GEMMs with fp32 accumulation (cuBLAS through torch.matmul, as
F.linear runs them on CUDA in the reference); the LoRA products are small fp32 GEMMs; the
element-wise middle — both LoRA deltas added in bf16 and the SiTU-GLU, and in the backward the
down adapter's input-gradient term plus the SiTU-GLU gradient — is one kernel each way
(ll_shared_glu_forward / ll_shared_glu_backward). The backward returns dL/dx and the six LoRA
gradients, following the autograd graph of the reference's forward (lora_layer.py:104-123:
the adapter casts its bf16 input to fp32 and its fp32 delta back to bf16).
"""
import ctypes
from typing import Dict, Tuple

import torch

from .. import _lib as L


class SharedExpert:
    """W_g, W_u [F, d], W_d [d, F] (bf16, frozen); adapters A_g, A_u [r, d], B_g, B_u [F, r],
    A_d [r, F], B_d [d, r] (fp32); scaling = alpha / r."""

    def __init__(self, W_g, W_u, W_d, A_g, B_g, A_u, B_u, A_d, B_d, scaling: float):
        L.require_cuda(W_g, W_u, W_d, A_g, B_g, A_u, B_u, A_d, B_d)
        self.F, self.d = W_g.shape
        self.r = A_g.shape[0]
        if tuple(W_u.shape) != (self.F, self.d) or tuple(W_d.shape) != (self.d, self.F):
            raise ValueError("W_g, W_u [F, d], W_d [d, F]")
        if self.r not in (4, 8, 16, 32):
            raise ValueError("LoRA rank 4, 8, 16 or 32")
        bf = lambda t: t.to(torch.bfloat16).contiguous()
        f32 = lambda t: t.to(torch.float32).contiguous()
        self.W_g, self.W_u, self.W_d = bf(W_g), bf(W_u), bf(W_d)
        self.A_g, self.B_g, self.A_u, self.B_u = f32(A_g), f32(B_g), f32(A_u), f32(B_u)
        self.A_d, self.B_d = f32(A_d), f32(B_d)
        self.s = float(scaling)
        self.lib = L.load()
        self._saved = None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """out [N, d] bf16 for x [N, d]."""
        L.require_cuda(x)
        xb = x.reshape(-1, self.d).to(torch.bfloat16).contiguous()
        N, F = xb.shape[0], self.F
        G = torch.matmul(xb, self.W_g.t())
        U = torch.matmul(xb, self.W_u.t())
        xf = xb.float()
        xa_g = torch.matmul(xf, self.A_g.t()).contiguous()
        xa_u = torch.matmul(xf, self.A_u.t()).contiguous()
        SG = torch.empty((N, F), dtype=torch.bfloat16, device=x.device)
        SU = torch.empty_like(SG)
        H = torch.empty_like(SG)
        L.check(self.lib.ll_shared_glu_forward(G.data_ptr(), U.data_ptr(), xa_g.data_ptr(), xa_u.data_ptr(),
                                               self.B_g.data_ptr(), self.B_u.data_ptr(), ctypes.c_float(self.s),
                                               N, F, self.r, SG.data_ptr(), SU.data_ptr(), H.data_ptr(),
                                               L.stream_ptr()), "ll_shared_glu_forward")
        ha = torch.matmul(H.float(), self.A_d.t())                                  # [N, r]
        out = torch.matmul(H, self.W_d.t()) + (torch.matmul(ha, self.B_d.t()) * self.s).to(torch.bfloat16)
        self._saved = (xf, xa_g, xa_u, SG, SU, H, ha)
        return out

    def backward(self, g: torch.Tensor) -> Tuple[torch.Tensor, Dict[str, torch.Tensor]]:
        """(dL/dx [N, d] bf16, {dA_g, dB_g, dA_u, dB_u, dA_d, dB_d} fp32) of the last forward."""
        if self._saved is None:
            raise RuntimeError("backward before forward")
        xf, xa_g, xa_u, SG, SU, H, ha = self._saved
        N, F, s = xf.shape[0], self.F, self.s
        gb = g.reshape(N, self.d).to(torch.bfloat16).contiguous()
        gf = gb.float()
        gB = torch.matmul(gf, self.B_d).contiguous()                                # [N, r]
        grads = {"dB_d": s * torch.matmul(gf.t(), ha), "dA_d": s * torch.matmul(gB.t(), H.float())}
        Dh = torch.matmul(gb, self.W_d)                                             # [N, F] bf16
        DSG = torch.empty((N, F), dtype=torch.bfloat16, device=g.device)
        DSU = torch.empty_like(DSG)
        L.check(self.lib.ll_shared_glu_backward(Dh.data_ptr(), gB.data_ptr(), self.A_d.data_ptr(),
                                                ctypes.c_float(s), SG.data_ptr(), SU.data_ptr(), N, F, self.r,
                                                DSG.data_ptr(), DSU.data_ptr(), L.stream_ptr()),
                "ll_shared_glu_backward")
        dg, du = DSG.float(), DSU.float()
        gg = torch.matmul(dg, self.B_g)                                             # [N, r]
        gu = torch.matmul(du, self.B_u)
        grads["dB_g"] = s * torch.matmul(dg.t(), xa_g)
        grads["dA_g"] = s * torch.matmul(gg.t(), xf)
        grads["dB_u"] = s * torch.matmul(du.t(), xa_u)
        grads["dA_u"] = s * torch.matmul(gu.t(), xf)
        dx = (torch.matmul(DSG, self.W_g).float() + torch.matmul(DSU, self.W_u).float()
              + (s * torch.matmul(gg, self.A_g)).to(torch.bfloat16).float()
              + (s * torch.matmul(gu, self.A_u)).to(torch.bfloat16).float())
        return dx.to(torch.bfloat16), grads
