"""
KimiK3MoERouter on the B200: same constructor and forward contract as
lazy_lora/core/moe_router.py:23-135, with the logits, sigmoid, biased top-k selection,
gather and renormalisation done by the library's router kernels (ll_route_topk_prepared; the
frozen weight's split into bf16 planes, ll_route_prepare, is kept between calls; up to 8 tokens,
ll_route_topk on the fp32 weight itself).

Ties in the selection go to the lower expert id. torch's CPU topk leaves the order of equal
values unspecified, so on inputs with exact ties the order (not the set) may differ.
"""
from typing import List, Optional, Tuple

import torch

from .. import _lib as L


class KimiK3MoERouter(torch.nn.Module):
    def __init__(self, hidden_size: int = 7168, num_experts: int = 896, top_k: int = 16,
                 routed_scaling_factor: float = 1.0, renormalize: bool = True, use_bias: bool = True,
                 device="cuda"):
        super().__init__()
        self.weight = torch.nn.Parameter(torch.empty(num_experts, hidden_size, device=device))
        self.bias = torch.nn.Parameter(torch.zeros(num_experts, device=device)) if use_bias else None
        torch.nn.init.normal_(self.weight, std=0.02)
        self.hidden_size = hidden_size
        self.num_experts = num_experts
        self.top_k = top_k
        self.routed_scaling_factor = routed_scaling_factor
        self.renormalize = renormalize
        self.use_bias = use_bias
        self._ws = None
        self._planes = None         # (key of the weight split, bf16 planes [3][E][d])

    def forward(self, x: torch.Tensor, weight: Optional[torch.Tensor] = None,
                bias: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
        """(topk_indices int64 [N, k], topk_weights fp32 [N, k]) for x [..., hidden]."""
        lib = L.load()
        weight = self.weight if weight is None else weight
        bias = self.bias if bias is None else bias
        L.require_cuda(x, weight, bias)
        xf = x.reshape(-1, self.hidden_size)
        if xf.dtype not in (torch.float32, torch.bfloat16):
            xf = xf.float()
        xf = xf.contiguous()
        b = None if bias is None else bias.detach().to(torch.float32).contiguous()
        T, E, k = xf.shape[0], self.num_experts, self.top_k
        nbytes = lib.ll_route_workspace_bytes(T, self.hidden_size, E)
        if self._ws is None or self._ws.numel() < nbytes or self._ws.device != xf.device:
            self._ws = torch.empty(nbytes, dtype=torch.uint8, device=xf.device)
        # the (frozen) weight's bf16 planes, split once and again only when the weight changes
        key = (weight.data_ptr(), weight._version, weight.dtype, tuple(weight.shape), weight.device)
        if self._planes is None or self._planes[0] != key:
            w = weight.detach().to(torch.float32).contiguous()
            planes = torch.empty((3, E, self.hidden_size), dtype=torch.bfloat16, device=w.device)
            L.check(lib.ll_route_prepare(w.data_ptr(), E, self.hidden_size, planes.data_ptr(), L.stream_ptr()),
                    "ll_route_prepare")
            self._planes = (key, planes)
        planes = self._planes[1]
        idx = torch.empty((T, k), dtype=torch.int64, device=xf.device)
        tw = torch.empty((T, k), dtype=torch.float32, device=xf.device)
        if T <= 8 and weight.dtype == torch.float32 and weight.is_contiguous() and weight.data_ptr() % 16 == 0:
            # a few tokens: the logits are a matrix-vector product on CUDA cores, which reads the
            # fp32 weight itself (two thirds of the planes' bytes; the same logits, bit for bit)
            L.check(lib.ll_route_topk(xf.data_ptr(), 0 if xf.dtype == torch.float32 else 1, weight.data_ptr(),
                                      L.ptr(b), T, self.hidden_size, E, k, int(self.renormalize),
                                      float(self.routed_scaling_factor), idx.data_ptr(), tw.data_ptr(), None,
                                      self._ws.data_ptr(), nbytes, L.stream_ptr()),
                    "ll_route_topk")
            return idx, tw
        L.check(lib.ll_route_topk_prepared(xf.data_ptr(), 0 if xf.dtype == torch.float32 else 1, planes.data_ptr(),
                                           L.ptr(b), T, self.hidden_size, E, k, int(self.renormalize),
                                           float(self.routed_scaling_factor), idx.data_ptr(), tw.data_ptr(), None,
                                           self._ws.data_ptr(), nbytes, L.stream_ptr()),
                "ll_route_topk_prepared")
        return idx, tw

    @staticmethod
    def get_active_expert_set(topk_indices: torch.Tensor) -> List[int]:
        """Sorted unique expert ids (moe_router.py:125-135)."""
        return sorted(int(e) for e in torch.unique(topk_indices).cpu().tolist())


def route_select(scores: torch.Tensor, scores_for_choice: torch.Tensor, top_k: int, renormalize: bool = True,
                 routed_scaling_factor: float = 1.0):
    """Selection half of the router (moe_router.py:92-99) from given fp32 scores."""
    lib = L.load()
    L.require_cuda(scores, scores_for_choice)
    s = scores.float().contiguous()
    c = scores_for_choice.float().contiguous()
    T, E = s.shape
    idx = torch.empty((T, top_k), dtype=torch.int64, device=s.device)
    w = torch.empty((T, top_k), dtype=torch.float32, device=s.device)
    L.check(lib.ll_route_select(s.data_ptr(), c.data_ptr(), T, E, top_k, int(renormalize),
                                float(routed_scaling_factor), idx.data_ptr(), w.data_ptr(), L.stream_ptr()),
            "ll_route_select")
    return idx, w
