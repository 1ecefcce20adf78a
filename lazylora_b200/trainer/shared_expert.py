"""
The shared expert of a Kimi K3 MoE layer on the GPU: a dense SiTU-GLU MLP (d -> F -> d, bf16
weights, frozen) with a rank-r LoRA adapter on each of its three projections
(lazy_lora/trainer/lazy_trainer.py:702-707):

    s_gate = linear32(x, W_g) + lora_g(x),  s_up = linear32(x, W_u) + lora_u(x)
    h      = situ_glu(s_gate, s_up)
    out    = linear32(h, W_d) + lora_d(h)

The three projections are bf16 GEMMs with fp32 accumulation, as F.linear runs them on CUDA in
the reference, on the library's tcgen05 GEMM (core.dense: gate and up in one launch; no
cuBLAS). The LoRA products read the bf16 activations
directly (ll_lora_down, ll_lora_outer: fixed-order split-K sums) instead of fp32 copies; the
element-wise middle — both LoRA deltas added in bf16 and the SiTU-GLU, and in the backward the
down adapter's input-gradient term plus the SiTU-GLU gradient — is one kernel each way
(ll_shared_glu_forward / ll_shared_glu_backward); the down projection's delta, and the gate/up
adapters' input-gradient terms, are added to the bf16 GEMM outputs in place
(ll_lora_add_bf16). The backward returns dL/dx and the six LoRA gradients, following the
autograd graph of the reference's forward (lora_layer.py:104-123: the adapter casts its bf16
input to fp32 and its fp32 delta back to bf16); the two gate/up input-gradient products are
summed in one fp32 accumulator and rounded to bf16 once. The LoRA products and adapter gradients
run on a second stream beside the bf16 GEMMs (events order each consumer after its producer), so
the small latency-bound kernels fill the GEMMs' gaps instead of adding to the step.
"""
import ctypes
from typing import Dict, Tuple

import torch

from .. import _lib as L
from ..core import dense


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
        self._ws = None
        self._side = None

    def _side_stream(self, device) -> torch.cuda.Stream:
        """The stream the LoRA products run on, beside the bf16 GEMMs on the caller's stream."""
        if self._side is None or self._side.device != device:
            self._side = torch.cuda.Stream(device=device)
        return self._side

    def _workspace(self, N: int, device) -> torch.Tensor:
        """Split-K partials of the LoRA products: 24 MB covers the splits that fill the GPU at the
        shapes here, plus one full [N, 2r] product for a single split. Allocated on, and used only
        by, the side stream, so its memory is reused in that stream's order."""
        need = 24 * 1024 * 1024 + 4 * N * 2 * self.r
        if self._ws is None or self._ws.numel() * 4 < need or self._ws.device != device:
            with torch.cuda.stream(self._side_stream(device)):
                self._ws = torch.empty(need // 4, dtype=torch.float32, device=device)
        return self._ws

    def _down(self, X, B0, B1, n0, n, b_rows, C0, C1, ws):
        L.check(self.lib.ll_lora_down(X.data_ptr(), 1, X.shape[0], X.shape[1], B0.data_ptr(),
                                      B1.data_ptr() if B1 is not None else None, n0, n, b_rows, ctypes.c_float(1.0),
                                      C0.data_ptr(), C1.data_ptr() if C1 is not None else None, ws.data_ptr(),
                                      ws.numel() * 4, L.stream_ptr()), "ll_lora_down")

    def _outer(self, P, Q, transposed, out, ws):
        L.check(self.lib.ll_lora_outer(P.data_ptr(), Q.data_ptr(), 1, Q.shape[0], Q.shape[1], self.r,
                                       ctypes.c_float(self.s), 1 if transposed else 0, out.data_ptr(), ws.data_ptr(),
                                       ws.numel() * 4, L.stream_ptr()), "ll_lora_outer")

    def _add(self, Y, L0, R0, L1, R1, r_rows):
        L.check(self.lib.ll_lora_add_bf16(Y.data_ptr(), L0.data_ptr(), R0.data_ptr(),
                                          L1.data_ptr() if L1 is not None else None,
                                          R1.data_ptr() if R1 is not None else None, self.r, r_rows,
                                          ctypes.c_float(self.s), Y.shape[0], Y.shape[1], Y.data_ptr(),
                                          L.stream_ptr()), "ll_lora_add_bf16")

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """out [N, d] bf16 for x [N, d]. The LoRA products run on a side stream while the bf16
        GEMMs run on the caller's stream; the caller's stream waits for them before returning."""
        L.require_cuda(x)
        xb = x.reshape(-1, self.d).to(torch.bfloat16).contiguous()
        N, F, r, dev = xb.shape[0], self.F, self.r, x.device
        main, side = torch.cuda.current_stream(dev), self._side_stream(dev)
        ws = self._workspace(N, dev)
        xa_g = torch.empty((N, r), dtype=torch.float32, device=dev)
        xa_u = torch.empty_like(xa_g)
        ha = torch.empty((N, r), dtype=torch.float32, device=dev)                    # H A_d^T
        side.wait_stream(main)
        if N:
            with torch.cuda.stream(side):
                self._down(xb, self.A_g, self.A_u, r, 2 * r, 1, xa_g, xa_u, ws)
        G, U = dense.linear_two(xb, self.W_g, self.W_u)
        G, U = G.contiguous(), U.contiguous()
        SG = torch.empty((N, F), dtype=torch.bfloat16, device=dev)
        SU = torch.empty_like(SG)
        H = torch.empty_like(SG)
        main.wait_stream(side)
        L.check(self.lib.ll_shared_glu_forward(G.data_ptr(), U.data_ptr(), xa_g.data_ptr(), xa_u.data_ptr(),
                                               self.B_g.data_ptr(), self.B_u.data_ptr(), ctypes.c_float(self.s),
                                               N, F, r, SG.data_ptr(), SU.data_ptr(), H.data_ptr(),
                                               L.stream_ptr()), "ll_shared_glu_forward")
        side.wait_stream(main)
        if N:
            with torch.cuda.stream(side):
                self._down(H, self.A_d, None, r, r, 1, ha, None, ws)
        out = dense.linear(H, self.W_d).contiguous()
        main.wait_stream(side)
        if N:
            self._add(out, ha, self.B_d, None, None, 0)
        self._saved = (xb, xa_g, xa_u, SG, SU, H, ha)
        return out

    def backward(self, g: torch.Tensor) -> Tuple[torch.Tensor, Dict[str, torch.Tensor]]:
        """(dL/dx [N, d] bf16, {dA_g, dB_g, dA_u, dB_u, dA_d, dB_d} fp32) of the last forward. The
        LoRA products and adapter gradients run on the side stream beside the three input-gradient
        GEMMs; everything is ordered before the caller's stream continues."""
        if self._saved is None:
            raise RuntimeError("backward before forward")
        xb, xa_g, xa_u, SG, SU, H, ha = self._saved
        N, F, d, r, s, dev = xb.shape[0], self.F, self.d, self.r, self.s, xb.device
        gb = g.reshape(N, d).to(torch.bfloat16).contiguous()
        f32 = lambda *shape: torch.empty(shape, dtype=torch.float32, device=dev)
        grads = {"dB_d": f32(d, r), "dA_d": f32(r, F), "dB_g": f32(F, r), "dA_g": f32(r, d),
                 "dB_u": f32(F, r), "dA_u": f32(r, d)}
        if N == 0:
            for t in grads.values():
                t.zero_()
            return torch.empty((0, d), dtype=torch.bfloat16, device=dev), grads
        main, side = torch.cuda.current_stream(dev), self._side_stream(dev)
        ws = self._workspace(N, dev)
        gB = f32(N, r)                                                               # g B_d
        gg, gu = f32(N, r), f32(N, r)                                                # dSG B_g, dSU B_u
        DSG = torch.empty((N, F), dtype=torch.bfloat16, device=dev)
        DSU = torch.empty_like(DSG)
        side.wait_stream(main)
        with torch.cuda.stream(side):
            self._down(gb, self.B_d, None, r, r, 0, gB, None, ws)
            gB_ready = side.record_event()
            self._outer(ha, gb, True, grads["dB_d"], ws)
            self._outer(gB, H, False, grads["dA_d"], ws)
        Dh = dense.matmul(gb, self.W_d).contiguous()                                 # [N, F] bf16
        main.wait_event(gB_ready)
        L.check(self.lib.ll_shared_glu_backward(Dh.data_ptr(), gB.data_ptr(), self.A_d.data_ptr(),
                                                ctypes.c_float(s), SG.data_ptr(), SU.data_ptr(), N, F, r,
                                                DSG.data_ptr(), DSU.data_ptr(), L.stream_ptr()),
                "ll_shared_glu_backward")
        side.wait_stream(main)
        with torch.cuda.stream(side):
            self._down(DSG, self.B_g, None, r, r, 0, gg, None, ws)
            self._down(DSU, self.B_u, None, r, r, 0, gu, None, ws)
            gu_ready = side.record_event()
            self._outer(xa_g, DSG, True, grads["dB_g"], ws)
            self._outer(gg, xb, False, grads["dA_g"], ws)
            self._outer(xa_u, DSU, True, grads["dB_u"], ws)
            self._outer(gu, xb, False, grads["dA_u"], ws)
        dx = dense.matmul_sum2(DSG, self.W_g, DSU, self.W_u).contiguous()
        main.wait_event(gu_ready)
        self._add(dx, gg, self.A_g, gu, self.A_u, 1)
        main.wait_stream(side)
        return dx, grads
