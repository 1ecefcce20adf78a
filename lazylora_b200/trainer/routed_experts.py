"""
The routed-expert map of one MoE layer on the B200: drop-in for the expert sweep of
LazyLoRATrainer (lazy_lora/trainer/lazy_trainer.py:45-77 RoutedExpertsFunction,
:806-834 _routed_experts_forward, :836-880 _routed_experts_backward).

`RoutedExpertsLayer` holds one layer's expert weights resident in HBM in the reference's
MXFP4 format (packed [E, rows, cols/2] + E8M0 scales [E, rows, cols/32]), the three LoRA
adapters shared by all experts, and the workspace in which the forward leaves what the
backward needs. `forward` / `backward` are one C-ABI call each; no expert loop runs in
Python and nothing falls back to the CPU.

`RoutedExpertsFunction` keeps the reference's autograd signature, calling
`trainer._routed_experts_forward(...)` / `trainer._routed_experts_backward(...)`; the
`B200ExpertEngine` below implements those two methods over RoutedExpertsLayer objects, so
the reference trainer can route its sweep here by delegating to an engine instance.
"""
from typing import Dict, Optional

import ctypes

import torch

from .. import _lib as L


def _pad_scale_rows(s: torch.Tensor) -> torch.Tensor:
    """[E, rows, G] scale bytes with rows padded to a multiple of 16 bytes (TMA strides)."""
    G = s.shape[-1]
    stride = (G + 15) // 16 * 16
    if stride == G:
        return s.contiguous()
    out = torch.zeros(s.shape[:-1] + (stride,), dtype=torch.uint8, device=s.device)
    out[..., :G] = s
    return out


TRANSPOSED = ("w1t", "w3t", "w2t", "s1t", "s3t", "s2t")


class RoutedExpertsLayer:
    """Expert weights + shared LoRA of one layer, resident on one GPU.

    The backward reads transposed copies of the weights, built once per weight load.
    prepare_backward=False defers that build to the first backward (a forward-only user never
    pays it); `transposed` supplies the buffers for it: a dict of the six tensors (or a
    callable returning one) whose leading dimension is at least E, e.g. one set per staging
    slot of a streamer, reused by every group copied into that slot."""

    def __init__(self, w1p, w1s, w3p, w3s, w2p, w2s, A_g, B_g, A_u, B_u, A_d, B_d, lora_scaling: float,
                 transposed=None, prepare_backward: bool = True):
        L.require_cuda(w1p, w1s, w3p, w3s, w2p, w2s, A_g, B_g, A_u, B_u, A_d, B_d)
        self.lib = L.load()
        E, f, dh = w1p.shape
        d = dh * 2
        assert w3p.shape == (E, f, dh) and w2p.shape == (E, d, f // 2), "packed shapes"
        assert w1s.shape == (E, f, d // 32) and w2s.shape == (E, d, f // 32), "scale shapes"
        self.E, self.d, self.f, self.r = E, d, f, A_g.shape[0]
        self.lora_scaling = float(lora_scaling)
        self.w1p, self.w3p, self.w2p = w1p.contiguous(), w3p.contiguous(), w2p.contiguous()
        self.w1s, self.w3s, self.w2s = _pad_scale_rows(w1s), _pad_scale_rows(w3s), _pad_scale_rows(w2s)
        self.A_g, self.B_g = A_g.float().contiguous(), B_g.float().contiguous()
        self.A_u, self.B_u = A_u.float().contiguous(), B_u.float().contiguous()
        self.A_d, self.B_d = A_d.float().contiguous(), B_d.float().contiguous()
        self.beta = torch.zeros((E, 2), dtype=torch.int32, device=w1p.device)
        # the forward GEMMs' weight scales, laid out for the block-scaled MMA by ll_moe_prepare
        sf = lambda R, C: torch.empty(int(self.lib.ll_mxfp4_sf_bytes(E, R, C)), dtype=torch.uint8,
                                      device=w1p.device)
        self.w1sf, self.w3sf, self.w2sf = sf(f, d), sf(f, d), sf(d, f)
        self.w1t = self.w3t = self.w2t = self.s1t = self.s3t = self.s2t = None
        self._tbufs = transposed
        self.desc = L.MoELayerDesc()
        self._fill_desc()
        # the decode bias alone (the forward needs nothing else)
        L.check(self.lib.ll_moe_prepare(ctypes.byref(self.desc), self.beta.data_ptr(), L.stream_ptr()), "ll_moe_prepare")
        self._ws: Optional[torch.Tensor] = None
        self._ws_key = None
        if prepare_backward:
            self.prepare_backward()

    def transposed_shapes(self) -> Dict[str, tuple]:
        """(shape, dtype) of the six transposed copies the backward reads."""
        E, d, f = self.E, self.d, self.f
        u8, f16 = torch.uint8, torch.float16
        return {"w1t": ((E, d, f // 2), u8), "w3t": ((E, d, f // 2), u8), "w2t": ((E, f, d // 2), u8),
                "s1t": ((E, d // 32, f), f16), "s3t": ((E, d // 32, f), f16), "s2t": ((E, f // 32, d), f16)}

    def prepare_backward(self):
        """Build the transposed weight copies the backward GEMMs read (once per weight load)."""
        if self.w1t is not None:
            return
        bufs = self._tbufs() if callable(self._tbufs) else self._tbufs
        dev = self.w1p.device
        for name, (shape, dt) in self.transposed_shapes().items():
            if bufs is None:
                t = torch.empty(shape, dtype=dt, device=dev)
            else:
                b = bufs[name]
                if b.dtype != dt or b.device != dev or b.shape[0] < shape[0] or tuple(b.shape[1:]) != shape[1:]:
                    raise ValueError(f"transposed buffer {name}: need {shape} {dt} on {dev}, got "
                                     f"{tuple(b.shape)} {b.dtype} on {b.device}")
                t = b[:shape[0]]
            setattr(self, name, t)
        self._fill_desc()
        L.check(self.lib.ll_moe_prepare(ctypes.byref(self.desc), self.beta.data_ptr(), L.stream_ptr()), "ll_moe_prepare")

    @classmethod
    def from_inputs(cls, inp: Dict[str, torch.Tensor], lora_scaling: float, device="cuda", **kw):
        t = {k: v.to(device) for k, v in inp.items() if k in (
            "w1p", "w1s", "w3p", "w3s", "w2p", "w2s", "A_g", "B_g", "A_u", "B_u", "A_d", "B_d")}
        return cls(t["w1p"], t["w1s"], t["w3p"], t["w3s"], t["w2p"], t["w2s"], t["A_g"], t["B_g"],
                   t["A_u"], t["B_u"], t["A_d"], t["B_d"], lora_scaling, **kw)

    def _fill_desc(self):
        D = self.desc
        D.d, D.f, D.E, D.r, D.lora_scaling = self.d, self.f, self.E, self.r, self.lora_scaling
        D.w1p, D.w1s, D.w3p, D.w3s = self.w1p.data_ptr(), self.w1s.data_ptr(), self.w3p.data_ptr(), self.w3s.data_ptr()
        D.w2p, D.w2s = self.w2p.data_ptr(), self.w2s.data_ptr()
        D.s13_stride, D.s2_stride = self.w1s.shape[-1], self.w2s.shape[-1]
        D.beta = self.beta.data_ptr()
        D.w1sf, D.w3sf, D.w2sf = self.w1sf.data_ptr(), self.w3sf.data_ptr(), self.w2sf.data_ptr()
        D.A_g, D.B_g, D.A_u, D.B_u = self.A_g.data_ptr(), self.B_g.data_ptr(), self.A_u.data_ptr(), self.B_u.data_ptr()
        D.A_d, D.B_d = self.A_d.data_ptr(), self.B_d.data_ptr()
        for name in TRANSPOSED:
            t = getattr(self, name)
            setattr(D, name, t.data_ptr() if t is not None else 0)

    def set_lora(self, A_g, B_g, A_u, B_u, A_d, B_d):
        """Point the layer at (updated) adapter tensors, e.g. after an optimizer step."""
        self.A_g, self.B_g = A_g.detach().float().contiguous(), B_g.detach().float().contiguous()
        self.A_u, self.B_u = A_u.detach().float().contiguous(), B_u.detach().float().contiguous()
        self.A_d, self.B_d = A_d.detach().float().contiguous(), B_d.detach().float().contiguous()
        self._fill_desc()

    def last_launch_count(self) -> int:
        """Kernels the last forward or backward call on this thread launched."""
        return int(self.lib.ll_last_launch_count())

    def lora_shapes(self) -> Dict[str, tuple]:
        """Shapes of the six LoRA gradients backward returns."""
        d, f, r = self.d, self.f, self.r
        return {"dA_g": (r, d), "dB_g": (f, r), "dA_u": (r, d), "dB_u": (f, r), "dA_d": (r, f), "dB_d": (d, r)}

    def workspace(self, T: int, k: int) -> torch.Tensor:
        n = self.lib.ll_moe_workspace_bytes(ctypes.byref(self.desc), T, k)
        if self._ws is None or self._ws.numel() < n:
            self._ws = torch.empty(n, dtype=torch.uint8, device=self.w1p.device)
        return self._ws

    @staticmethod
    def _dtype_code(t: torch.Tensor) -> int:
        if t.dtype == torch.float32:
            return 0
        if t.dtype == torch.bfloat16:
            return 1
        raise TypeError(f"activations must be float32 or bfloat16, got {t.dtype}")

    accepts_rows_hint = True

    def forward(self, x: torch.Tensor, idx: torch.Tensor, w: torch.Tensor, rows_hint: Optional[int] = None) -> torch.Tensor:
        """out[T, d] fp32 = sum over each token's k experts (ascending id) of w * expert(x).
        rows_hint: how many of the T*k slots are routed (>= 0), when many are -1."""
        L.require_cuda(x, idx, w)
        self.desc.rows_hint = int(rows_hint) if rows_hint else 0
        x = x.contiguous()
        idx = idx.to(torch.int64).contiguous()
        w = w.to(torch.float32).contiguous()
        T, k = idx.shape
        ws = self.workspace(T, k)
        out = torch.empty((T, self.d), dtype=torch.float32, device=x.device)
        L.check(self.lib.ll_moe_forward(ctypes.byref(self.desc), T, k, x.data_ptr(), self._dtype_code(x),
                                        idx.data_ptr(), w.data_ptr(), out.data_ptr(), ws.data_ptr(), ws.numel(),
                                        L.stream_ptr()), "ll_moe_forward")
        self._ws_key = (x.data_ptr(), idx.data_ptr(), w.data_ptr(), T, k)
        return out

    def forward_rmsnorm(self, x: torch.Tensor, idx: torch.Tensor, w: torch.Tensor, norm_w: torch.Tensor, eps: float,
                        rows_hint: Optional[int] = None):
        """forward() whose combine also RMS-normalises each token's row (the latent block's norm):
        (out [T, d] fp32, normed [T, d] bf16, rstd [T] fp32)."""
        L.require_cuda(x, idx, w, norm_w)
        self.desc.rows_hint = int(rows_hint) if rows_hint else 0
        x = x.contiguous()
        idx = idx.to(torch.int64).contiguous()
        w = w.to(torch.float32).contiguous()
        nw = norm_w.to(torch.float32).contiguous()
        T, k = idx.shape
        ws = self.workspace(T, k)
        out = torch.empty((T, self.d), dtype=torch.float32, device=x.device)
        normed = torch.empty((T, self.d), dtype=torch.bfloat16, device=x.device)
        rstd = torch.empty((T,), dtype=torch.float32, device=x.device)
        L.check(self.lib.ll_moe_forward_rmsnorm(ctypes.byref(self.desc), T, k, x.data_ptr(), self._dtype_code(x),
                                                idx.data_ptr(), w.data_ptr(), nw.data_ptr(), ctypes.c_float(eps),
                                                out.data_ptr(), normed.data_ptr(), rstd.data_ptr(), ws.data_ptr(),
                                                ws.numel(), L.stream_ptr()), "ll_moe_forward_rmsnorm")
        self._ws_key = (x.data_ptr(), idx.data_ptr(), w.data_ptr(), T, k)
        return out, normed, rstd

    def backward(self, x, idx, w, g, forward_done: bool = None, rows_hint: Optional[int] = None):
        """(grad_h [T,d], grad_w [T,k], {dA_g, dB_g, dA_u, dB_u, dA_d, dB_d}), all fp32.
        rows_hint: as given to the forward (used when the forward is recomputed here)."""
        L.require_cuda(x, idx, w, g)
        x = x.contiguous()
        idx = idx.to(torch.int64).contiguous()
        w = w.to(torch.float32).contiguous()
        g = g.contiguous()
        T, k = idx.shape
        key = (x.data_ptr(), idx.data_ptr(), w.data_ptr(), T, k)
        if forward_done is None:
            forward_done = self._ws_key == key
        if not forward_done:        # the workspace does not hold this forward: recompute it
            self.forward(x, idx, w, rows_hint=rows_hint)
        self.prepare_backward()
        ws = self.workspace(T, k)
        dev = x.device
        grad_h = torch.empty((T, self.d), dtype=torch.float32, device=dev)
        grad_w = torch.empty((T, k), dtype=torch.float32, device=dev)
        grads = {
            "dA_g": torch.empty_like(self.A_g), "dB_g": torch.empty_like(self.B_g),
            "dA_u": torch.empty_like(self.A_u), "dB_u": torch.empty_like(self.B_u),
            "dA_d": torch.empty_like(self.A_d), "dB_d": torch.empty_like(self.B_d),
        }
        L.check(self.lib.ll_moe_backward(
            ctypes.byref(self.desc), T, k, x.data_ptr(), self._dtype_code(x), idx.data_ptr(), w.data_ptr(),
            g.data_ptr(), self._dtype_code(g), grad_h.data_ptr(), grad_w.data_ptr(),
            grads["dA_g"].data_ptr(), grads["dB_g"].data_ptr(), grads["dA_u"].data_ptr(), grads["dB_u"].data_ptr(),
            grads["dA_d"].data_ptr(), grads["dB_d"].data_ptr(), ws.data_ptr(), ws.numel(), L.stream_ptr()),
            "ll_moe_backward")
        return grad_h, grad_w, grads

    def permutation(self, T: int, k: int):
        """(offsets [E+1], perm_token [P], perm_slot [P]) int32 of the last forward."""
        ws = self.workspace(T, k)
        dev = self.w1p.device
        off = torch.empty(self.E + 1, dtype=torch.int32, device=dev)
        tok = torch.empty(T * k, dtype=torch.int32, device=dev)
        slot = torch.empty(T * k, dtype=torch.int32, device=dev)
        L.check(self.lib.ll_moe_permutation(ctypes.byref(self.desc), T, k, ws.data_ptr(), off.data_ptr(),
                                            tok.data_ptr(), slot.data_ptr(), L.stream_ptr()), "ll_moe_permutation")
        n = int(off[-1])
        return off, tok[:n], slot[:n]

    def check_status(self, T: int, k: int):
        """Raise if a device-side bounded wait ran out during the last forward/backward (syncs)."""
        ws = self.workspace(T, k)
        L.check(self.lib.ll_moe_status(ctypes.byref(self.desc), T, k, ws.data_ptr(), L.stream_ptr()), "ll_moe_status")


def _accumulate(p: torch.Tensor, g: torch.Tensor):
    g = g.to(p.dtype)
    if p.grad is None:
        p.grad = g.clone()
    else:
        p.grad.add_(g)


class B200ExpertEngine:
    """
    Implements the two trainer methods RoutedExpertsFunction calls, over device-resident
    layers: `layers[layer_idx]` is a RoutedExpertsLayer. LoRA gradients are accumulated into
    bundle.{gate,up,down}_lora.lora_{A,B}.grad as LazyLoRALinear.accumulate_grad does
    (lazy_lora/core/lora_layer.py:258-290).
    """

    def __init__(self, layers: Dict[int, RoutedExpertsLayer]):
        self.layers = layers

    def _sync_lora(self, layer: RoutedExpertsLayer, bundle):
        if bundle is None:
            return
        layer.set_lora(bundle.gate_lora.lora_A, bundle.gate_lora.lora_B, bundle.up_lora.lora_A,
                       bundle.up_lora.lora_B, bundle.down_lora.lora_A, bundle.down_lora.lora_B)

    def _routed_experts_forward(self, layer_idx, bundle, h_latent, topk_indices, topk_weights, active_experts=None):
        layer = self.layers[layer_idx]
        self._sync_lora(layer, bundle)
        return layer.forward(h_latent, topk_indices, topk_weights)

    def _routed_experts_backward(self, layer_idx, bundle, h_latent, topk_indices, topk_weights, active_experts,
                                 grad_out):
        layer = self.layers[layer_idx]
        self._sync_lora(layer, bundle)
        grad_h, grad_w, g = layer.backward(h_latent, topk_indices, topk_weights, grad_out.float())
        if bundle is not None:
            _accumulate(bundle.gate_lora.lora_A, g["dA_g"])
            _accumulate(bundle.gate_lora.lora_B, g["dB_g"])
            _accumulate(bundle.up_lora.lora_A, g["dA_u"])
            _accumulate(bundle.up_lora.lora_B, g["dB_u"])
            _accumulate(bundle.down_lora.lora_A, g["dA_d"])
            _accumulate(bundle.down_lora.lora_B, g["dB_d"])
        return grad_h.to(h_latent.dtype), grad_w.to(topk_weights.dtype)


class RoutedExpertsFunction(torch.autograd.Function):
    """Same signature and contract as lazy_lora/trainer/lazy_trainer.py:45-77."""

    @staticmethod
    def forward(ctx, h_latent, topk_weights, topk_indices, trainer, layer_idx, bundle, active_experts, cached=None):
        if cached is not None:
            out = cached.to(torch.float32)
        else:
            out = trainer._routed_experts_forward(layer_idx, bundle, h_latent, topk_indices, topk_weights,
                                                  active_experts)
        ctx.save_for_backward(h_latent, topk_weights, topk_indices)
        ctx.trainer, ctx.layer_idx, ctx.bundle, ctx.active_experts = trainer, layer_idx, bundle, active_experts
        return out

    @staticmethod
    def backward(ctx, grad_out):
        h_latent, topk_weights, topk_indices = ctx.saved_tensors
        grad_h, grad_w = ctx.trainer._routed_experts_backward(
            ctx.layer_idx, ctx.bundle, h_latent, topk_indices, topk_weights, ctx.active_experts, grad_out)
        return grad_h, grad_w, None, None, None, None, None, None
