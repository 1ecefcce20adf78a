"""
CPU oracle for the routed-expert hot path. TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference leg may import
this module, and only as the checker or the timed CPU baseline. The product package
(lazylora_b200) never imports it and has no CPU fallback.

It restates, on CPU tensors and with the same torch CPU operators the reference calls, the
reference's algorithm for the path:

  route              lazy_lora/core/moe_router.py:80-100     (KimiK3MoERouter.forward)
  active_experts     lazy_lora/core/moe_router.py:125-135    (get_active_expert_set)
  permutation        lazy_lora/trainer/lazy_trainer.py:823-827 (mask / nonzero per expert)
  situ_glu_forward   lazy_lora/core/situ_activation.py:47-75
  situ_glu_backward  lazy_lora/core/situ_activation.py:78-134
  LoRA               lazy_lora/core/lora_layer.py:104-139, 178-226, 258-290
  expert_forward     lazy_lora/trainer/lazy_trainer.py:762-791 (packed branch)
  experts_forward    lazy_lora/trainer/lazy_trainer.py:806-834
  experts_backward   lazy_lora/trainer/lazy_trainer.py:836-880

The MXFP4 GEMMs go through a C library: either this repository's restatement
(oracle/_build/libmxfp4_oracle.so, from mxfp4_oracle.c) or the reference's own kernel
compiled from its source (oracle/_ref/libmxfp4_ref.so, "reference" kind). The reference
kernel only supports K <= 4096 (lazy_lora/native/mxfp4_gemm.c:72), so `gemm` splits K into
chunks of 3584 and sums them in fp32 when it drives that library at K = 7168.

Parity of this oracle is pinned by tests/test_oracle.py against the golden vectors in
tests/golden/ (made by tests/golden/make_golden.py from the reference itself, plus the
reference's vendored router / SiTU-GLU / MoE-block fixtures).
"""
import ctypes
import os
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "libmxfp4_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libmxfp4_ref.so")
REF_K_CHUNK = 3584          # largest K the reference's stack tile takes, multiple of 32


def build(ref_root: Optional[str] = None) -> None:
    """Compile the checkers: oracle/_build always, and oracle/_ref from the reference tree at
    `ref_root` (default: the LAZYLORA_REFERENCE_ROOT environment variable) when it exists."""
    import subprocess
    ref_root = ref_root or os.environ.get("LAZYLORA_REFERENCE_ROOT", "")
    subprocess.run(["make", "-s", "-C", HERE, f"REF_ROOT={ref_root}"], check=True)


class MXFP4Checker:
    """gemm / gemm_t / dequant on CPU tensors, the semantics of lazy_lora/native/__init__.py:36-74."""

    def __init__(self, kind: str = "oracle"):
        path = ORACLE_SO if kind == "oracle" else REF_SO
        if not os.path.exists(path):
            build()
        self.kind = kind
        lib = ctypes.CDLL(path)
        f32 = ctypes.POINTER(ctypes.c_float)
        u8 = ctypes.POINTER(ctypes.c_uint8)
        pre = "oracle_" if kind == "oracle" else ""
        self._gemm = getattr(lib, pre + "mxfp4_gemm")
        self._gemm_t = getattr(lib, pre + "mxfp4_gemm_t")
        self._deq = getattr(lib, pre + "mxfp4_dequant")
        self._thr = getattr(lib, "oracle_threads" if kind == "oracle" else "mxfp4_threads")
        for fn in (self._gemm, self._gemm_t):
            fn.argtypes = [f32, f32, u8, u8, ctypes.c_int, ctypes.c_int, ctypes.c_int]
            fn.restype = None
        self._deq.argtypes = [f32, u8, u8, ctypes.c_int, ctypes.c_int]
        self._deq.restype = None
        self._thr.restype = ctypes.c_int
        self.lib = lib

    @staticmethod
    def _p(t, ct):
        return ctypes.cast(t.data_ptr(), ctypes.POINTER(ct))

    def threads(self) -> int:
        return int(self._thr())

    def _gemm_raw(self, x, packed, scales):
        M, K = x.shape
        R = packed.shape[0]
        y = torch.empty((M, R), dtype=torch.float32)
        self._gemm(self._p(y, ctypes.c_float), self._p(x, ctypes.c_float),
                   self._p(packed, ctypes.c_uint8), self._p(scales, ctypes.c_uint8), M, K, R)
        return y

    def gemm(self, x, packed, scales):
        """y[M, R] = x[M, K] @ W^T for packed W[R, K]."""
        x = x.contiguous().float()
        M, K = x.shape
        R = packed.shape[0]
        assert packed.shape[1] * 2 == K and scales.shape == (R, K // 32), (packed.shape, scales.shape, K)
        packed, scales = packed.contiguous(), scales.contiguous()
        if self.kind == "oracle" or K <= 4096:
            return self._gemm_raw(x, packed, scales)
        y = None
        for k0 in range(0, K, REF_K_CHUNK):
            k1 = min(K, k0 + REF_K_CHUNK)
            part = self._gemm_raw(x[:, k0:k1].contiguous(), packed[:, k0 // 2:k1 // 2].contiguous(),
                                  scales[:, k0 // 32:k1 // 32].contiguous())
            y = part if y is None else y + part
        return y

    def gemm_t(self, dy, packed, scales):
        """y[M, K] = dy[M, R] @ W for packed W[R, K] (the C call accumulates into zeros)."""
        dy = dy.contiguous().float()
        M, R = dy.shape
        K = packed.shape[1] * 2
        assert packed.shape[0] == R and scales.shape == (R, K // 32)
        y = torch.zeros((M, K), dtype=torch.float32)
        self._gemm_t(self._p(y, ctypes.c_float), self._p(dy, ctypes.c_float),
                     self._p(packed.contiguous(), ctypes.c_uint8),
                     self._p(scales.contiguous(), ctypes.c_uint8), M, K, R)
        return y

    def dequant(self, packed, scales):
        R = packed.shape[0]
        K = packed.shape[1] * 2
        w = torch.empty((R, K), dtype=torch.float32)
        self._deq(self._p(w, ctypes.c_float), self._p(packed.contiguous(), ctypes.c_uint8),
                  self._p(scales.contiguous(), ctypes.c_uint8), K, R)
        return w


# ------------------------------------------------------------------------------ routing

def route(x, weight, bias, top_k: int, renormalize: bool = True, routed_scaling_factor: float = 1.0):
    """(topk_indices int64 [N,k], topk_weights f32 [N,k]) as moe_router.py:80-100 computes them."""
    x_flat = x.reshape(-1, weight.shape[1]).to(torch.float32)
    logits = F.linear(x_flat, weight.to(torch.float32))
    scores = torch.sigmoid(logits)
    sfc = scores + bias.to(torch.float32).unsqueeze(0) if bias is not None else scores
    return route_select(scores, sfc, top_k, renormalize, routed_scaling_factor)


def route_select(scores, scores_for_choice, top_k: int, renormalize: bool = True,
                 routed_scaling_factor: float = 1.0):
    """The selection half of the router (moe_router.py:92-99) given its fp32 scores."""
    _, idx = torch.topk(scores_for_choice, k=top_k, dim=-1, sorted=True)
    w = torch.gather(scores, dim=-1, index=idx)
    if top_k > 1 and renormalize:
        w = w / (w.sum(dim=-1, keepdim=True) + 1e-20)
    return idx, w * routed_scaling_factor


def router_logits(x, weight):
    return F.linear(x.reshape(-1, weight.shape[1]).to(torch.float32), weight.to(torch.float32))


def active_experts(idx) -> List[int]:
    """moe_router.py:125-135: sorted unique expert ids."""
    return sorted(int(e) for e in torch.unique(idx).tolist())


def permutation(idx, E: int):
    """
    The reference's per-expert gather (lazy_trainer.py:823-827) as one stable permutation:
    (offsets [E+1] int64, token [P] int64, slot [P] int64). Pairs are ordered by expert id,
    tokens ascending within an expert, which is the row order `mask.any(-1).nonzero()` gives.
    """
    N, k = idx.shape
    offsets = torch.zeros(E + 1, dtype=torch.int64)
    toks, slots = [], []
    for e in range(E):
        mask = idx == e
        rows = mask.any(dim=-1).nonzero(as_tuple=False).squeeze(-1)
        offsets[e + 1] = offsets[e] + rows.numel()
        if rows.numel():
            toks.append(rows)
            slots.append(mask[rows].to(torch.int64).argmax(dim=-1))
    token = torch.cat(toks) if toks else torch.zeros(0, dtype=torch.int64)
    slot = torch.cat(slots) if slots else torch.zeros(0, dtype=torch.int64)
    return offsets, token, slot


# ---------------------------------------------------------------------------- SiTU-GLU

SITU_BETA = 4.0
SITU_LINEAR_BETA = 25.0


def situ_glu_forward(gate, up, beta: float = SITU_BETA, linear_beta: Optional[float] = SITU_LINEAR_BETA):
    dtype = gate.dtype
    g = gate.to(torch.float32)
    u = up.to(torch.float32)
    a = beta * torch.tanh(g / beta) * torch.sigmoid(g)
    if linear_beta is not None:
        u = linear_beta * torch.tanh(u / linear_beta)
    return (a * u).to(dtype)


def situ_glu_backward(grad_output, gate, up, beta: float = SITU_BETA,
                      linear_beta: Optional[float] = SITU_LINEAR_BETA):
    dtype = grad_output.dtype
    go = grad_output.to(torch.float32)
    g = gate.to(torch.float32)
    u = up.to(torch.float32)
    t = torch.tanh(g / beta)
    s = torch.sigmoid(g)
    a = beta * t * s
    da = (1.0 - t * t) * s + beta * t * s * (1.0 - s)
    if linear_beta is not None:
        tu = torch.tanh(u / linear_beta)
        u_out = linear_beta * tu
        du = 1.0 - tu * tu
    else:
        u_out = u
        du = torch.ones_like(u)
    return (go * u_out * da).to(dtype), (go * a * du).to(dtype)


# -------------------------------------------------------------------------------- LoRA

@dataclass
class LoRA:
    """One rank-r adapter: A [r, in], B [out, r], fp32, scaling alpha / r (lora_layer.py:48-102)."""
    A: torch.Tensor
    B: torch.Tensor
    scaling: float
    grad_A: Optional[torch.Tensor] = None
    grad_B: Optional[torch.Tensor] = None

    def forward_lora_only(self, x):
        orig = x.dtype
        xd = x.to(self.A.dtype) if x.dtype != self.A.dtype else x
        delta = F.linear(F.linear(xd, self.A), self.B) * self.scaling
        return delta.to(orig) if delta.dtype != orig else delta

    def compute_lora_gradients(self, grad_output, input_activation, dx_base):
        in_f, out_f = self.A.shape[1], self.B.shape[0]
        x_flat = input_activation.reshape(-1, in_f).to(self.A.dtype)
        dy_flat = grad_output.reshape(-1, out_f).to(self.A.dtype)
        h = F.linear(x_flat, self.A)
        grad_B = self.scaling * torch.matmul(dy_flat.t(), h)
        dh = self.scaling * F.linear(dy_flat, self.B.t())
        grad_A = torch.matmul(dh.t(), x_flat)
        dx_lora = F.linear(dh, self.A.t())
        grad_input = (dx_base.reshape(-1, in_f).to(self.A.dtype) + dx_lora).view_as(input_activation)
        if grad_input.dtype != input_activation.dtype:
            grad_input = grad_input.to(input_activation.dtype)
        return grad_A, grad_B, grad_input

    def accumulate_grad(self, gA, gB):
        self.grad_A = gA.clone() if self.grad_A is None else self.grad_A + gA
        self.grad_B = gB.clone() if self.grad_B is None else self.grad_B + gB


@dataclass
class Layer:
    """Packed expert weights [E, rows, cols] plus the three shared adapters of one layer."""
    w1p: torch.Tensor
    w1s: torch.Tensor
    w3p: torch.Tensor
    w3s: torch.Tensor
    w2p: torch.Tensor
    w2s: torch.Tensor
    gate: LoRA
    up: LoRA
    down: LoRA

    @staticmethod
    def from_inputs(inp: Dict[str, torch.Tensor], scaling: float) -> "Layer":
        return Layer(inp["w1p"], inp["w1s"], inp["w3p"], inp["w3s"], inp["w2p"], inp["w2s"],
                     LoRA(inp["A_g"].float(), inp["B_g"].float(), scaling),
                     LoRA(inp["A_u"].float(), inp["B_u"].float(), scaling),
                     LoRA(inp["A_d"].float(), inp["B_d"].float(), scaling))


def expert_forward(k: MXFP4Checker, layer: Layer, e: int, x):
    """gate, up, situ, down for the rows x of expert e (lazy_trainer.py:762-791, packed branch)."""
    xf = x.float()
    gate = k.gemm(xf, layer.w1p[e], layer.w1s[e])
    up = k.gemm(xf, layer.w3p[e], layer.w3s[e])
    gate = gate + layer.gate.forward_lora_only(x).float()
    up = up + layer.up.forward_lora_only(x).float()
    situ = situ_glu_forward(gate, up)
    down = k.gemm(situ, layer.w2p[e], layer.w2s[e])
    down = down + layer.down.forward_lora_only(situ).float()
    return gate, up, situ, down


def experts_forward(k: MXFP4Checker, layer: Layer, h, idx, w, experts: Optional[List[int]] = None):
    """sum_e w_e(token) * expert_e(h), experts in ascending id order (lazy_trainer.py:806-834)."""
    out = torch.zeros(h.shape, dtype=torch.float32)
    for e in (active_experts(idx) if experts is None else experts):
        mask = idx == e
        rows = mask.any(dim=-1).nonzero(as_tuple=False).squeeze(-1)
        if rows.numel() == 0:
            continue
        x = h.index_select(0, rows)
        _g, _u, _s, down = expert_forward(k, layer, e, x)
        tw = (w.index_select(0, rows) * mask.index_select(0, rows).to(w.dtype)).sum(dim=-1, keepdim=True)
        out.index_add_(0, rows, down * tw.float())
    return out


def experts_backward(k: MXFP4Checker, layer: Layer, h, idx, w, grad_out,
                     experts: Optional[List[int]] = None):
    """(grad_h, grad_w); LoRA gradients accumulate into layer.{gate,up,down} (lazy_trainer.py:836-880)."""
    grad_h = torch.zeros(h.shape, dtype=torch.float32)
    grad_w = torch.zeros(w.shape, dtype=torch.float32)
    for e in (active_experts(idx) if experts is None else experts):
        mask = idx == e
        rows = mask.any(dim=-1).nonzero(as_tuple=False).squeeze(-1)
        if rows.numel() == 0:
            continue
        x = h.index_select(0, rows)
        g_out = grad_out.index_select(0, rows).float()
        m = mask.index_select(0, rows)
        gate, up, situ, e_down = expert_forward(k, layer, e, x)
        dot = (g_out * e_down).sum(dim=-1, keepdim=True)
        grad_w.index_add_(0, rows, dot * m.to(dot.dtype))
        tw = (w.index_select(0, rows) * m.to(w.dtype)).sum(dim=-1, keepdim=True)
        d_down = g_out * tw.float()
        gA, gB, d_situ = layer.down.compute_lora_gradients(
            d_down, situ, dx_base=k.gemm_t(d_down, layer.w2p[e], layer.w2s[e]))
        layer.down.accumulate_grad(gA, gB)
        d_gate, d_up = situ_glu_backward(d_situ, gate, up)
        gA, gB, d_in_g = layer.gate.compute_lora_gradients(
            d_gate, x, dx_base=k.gemm_t(d_gate, layer.w1p[e], layer.w1s[e]))
        layer.gate.accumulate_grad(gA, gB)
        gA, gB, d_in_u = layer.up.compute_lora_gradients(
            d_up, x, dx_base=k.gemm_t(d_up, layer.w3p[e], layer.w3s[e]))
        layer.up.accumulate_grad(gA, gB)
        grad_h.index_add_(0, rows, d_in_g.float() + d_in_u.float())
    return grad_h.to(h.dtype), grad_w.to(w.dtype)


def run_layer(k: MXFP4Checker, inp: Dict[str, torch.Tensor], top_k: int, scaling: float,
              backward: bool = True) -> Dict[str, torch.Tensor]:
    """Route, forward and (optionally) backward one layer; returns every golden tensor."""
    layer = Layer.from_inputs(inp, scaling)
    x = inp["x"].float()
    idx, w = route(x, inp["router_w"], inp["router_b"], top_k)
    E = inp["w1p"].shape[0]
    offsets, token, slot = permutation(idx, E)
    res = {"idx": idx, "w": w, "offsets": offsets, "perm_token": token, "perm_slot": slot}
    res["out"] = experts_forward(k, layer, x, idx, w)
    if backward:
        gh, gw = experts_backward(k, layer, x, idx, w, inp["g"].float())
        res.update(grad_h=gh, grad_w=gw,
                   dA_g=layer.gate.grad_A, dB_g=layer.gate.grad_B,
                   dA_u=layer.up.grad_A, dB_u=layer.up.grad_B,
                   dA_d=layer.down.grad_A, dB_d=layer.down.grad_B)
    return res


def rel_l2(got, want) -> float:
    got = got.double().reshape(-1)
    want = want.double().reshape(-1)
    return float((got - want).norm() / (want.norm() + 1e-300))
