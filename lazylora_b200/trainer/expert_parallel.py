"""
Expert-parallel routed-expert layer: one process per GPU, experts split over the ranks.

The reference runs every routed expert in one process (lazy_lora/trainer/lazy_trainer.py
:806-880); this module spreads one layer's experts over n ranks of a torch.distributed
process group (NCCL on GPUs) and keeps the single-GPU layer (`RoutedExpertsLayer`, the
ll_moe_forward / ll_moe_backward calls) unchanged on each rank:

  expert e lives on rank floor(e * n / E)        (ll_ep_experts_of_rank)
  forward   plan (ll_ep_plan) -> exchange row counts -> gather this rank's token rows once
            per destination rank (ll_ep_gather_rows) -> all-to-all of the rows and of their
            k-slot headers (local expert id or -1, routing weight) -> local layer forward on
            the rows received -> all-to-all of the fp32 partial outputs back -> sum of each
            token's partials in ascending rank order (ll_ep_combine)
  backward  the same exchange for the upstream gradient rows, local layer backward,
            grad_h partials back and summed, grad_w slots gathered from the rank that owns
            each slot's expert (ll_ep_combine_slots), and one all-reduce (sum) of the six
            LoRA gradients (the adapters are shared by all experts)

All data crossing ranks goes through NCCL all-to-all / all-reduce into local HBM before any
kernel reads it. The result equals the single-GPU layer on the concatenated tokens up to the
fp32 summation order of the partial outputs.

The index kernels and the exchange order are separated (`ops`), so the same orchestration
runs with another implementation of the four index operations.
"""
from typing import Dict, List, Optional, Tuple

import ctypes

import torch
import torch.distributed as dist

from .. import _lib as L

LORA_GRADS = ("dA_g", "dB_g", "dA_u", "dB_u", "dA_d", "dB_d")


def experts_of_rank(E: int, n: int, rank: int) -> Tuple[int, int]:
    """(first expert id, expert count) of `rank`: contiguous blocks, expert e on rank floor(e*n/E)."""
    if not (0 <= rank < n) or E <= 0:
        raise ValueError("bad rank / expert count")
    lo = (rank * E + n - 1) // n
    hi = ((rank + 1) * E + n - 1) // n
    return lo, hi - lo


class CudaEPOps:
    """The four index operations as this library's CUDA kernels (C ABI)."""

    def __init__(self):
        self.lib = L.load()
        self.launches = 0      # kernels launched so far (for launch accounting)

    def plan(self, idx: torch.Tensor, w: torch.Tensor, E: int, n: int):
        L.require_cuda(idx, w)
        T, k = idx.shape
        dev = idx.device
        counts = torch.empty(n + 1, dtype=torch.int32, device=dev)
        pos = torch.empty((T, n), dtype=torch.int32, device=dev)
        cap = max(T * n, 1)
        send_tok = torch.empty(cap, dtype=torch.int32, device=dev)
        send_idx = torch.empty((cap, k), dtype=torch.int64, device=dev)
        send_w = torch.empty((cap, k), dtype=torch.float32, device=dev)
        L.check(self.lib.ll_ep_plan(T, k, E, n, idx.data_ptr(), w.data_ptr(), counts.data_ptr(), pos.data_ptr(),
                                    send_tok.data_ptr(), send_idx.data_ptr(), send_w.data_ptr(), L.stream_ptr()),
                "ll_ep_plan")
        self.launches += 1
        return counts, pos, send_tok, send_idx, send_w

    def gather_rows(self, src: torch.Tensor, tok: torch.Tensor, rows: int) -> torch.Tensor:
        src = src.contiguous()
        out = torch.empty((rows,) + tuple(src.shape[1:]), dtype=src.dtype, device=src.device)
        row_bytes = src[0].numel() * src.element_size() if src.shape[0] else 0
        if rows:
            L.check(self.lib.ll_ep_gather_rows(out.data_ptr(), src.data_ptr(), tok.data_ptr(), rows, row_bytes,
                                               L.stream_ptr()), "ll_ep_gather_rows")
            self.launches += 1
        return out

    def combine(self, part: torch.Tensor, pos: torch.Tensor, T: int, d: int) -> torch.Tensor:
        out = torch.empty((T, d), dtype=torch.float32, device=pos.device)
        n = pos.shape[1]
        L.check(self.lib.ll_ep_combine(out.data_ptr(), part.data_ptr() if part.numel() else None, pos.data_ptr(), T,
                                       n, d, L.stream_ptr()), "ll_ep_combine")
        self.launches += T > 0
        return out

    def combine_slots(self, part: torch.Tensor, pos: torch.Tensor, idx: torch.Tensor, E: int) -> torch.Tensor:
        T, k = idx.shape
        out = torch.empty((T, k), dtype=torch.float32, device=idx.device)
        L.check(self.lib.ll_ep_combine_slots(out.data_ptr(), part.data_ptr() if part.numel() else None,
                                             pos.data_ptr(), idx.data_ptr(), T, k, E, pos.shape[1], L.stream_ptr()),
                "ll_ep_combine_slots")
        self.launches += T > 0
        return out


class ExpertParallelLayer:
    """One MoE layer whose experts are split over the ranks of `group`.

    local_layer: this rank's experts (a RoutedExpertsLayer over experts_of_rank(E, n, rank)),
    with forward(x, idx, w) -> out and backward(x, idx, w, g) -> (grad_h, grad_w, grads).
    E: the layer's total expert count (the ids the router returns).
    """

    def __init__(self, local_layer, E: int, group=None, ops=None):
        self.local = local_layer
        self.E = int(E)
        self.group = group
        self.n = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.first, self.count = experts_of_rank(self.E, self.n, self.rank)
        if getattr(local_layer, "E", self.count) != self.count:
            raise ValueError(f"rank {self.rank} owns {self.count} experts, local layer has {local_layer.E}")
        self.ops = ops if ops is not None else CudaEPOps()
        self._ctx = None
        self.local_launches = 0    # kernels the local layer launched in the last forward + backward

    # ---------------------------------------------------------------- exchanges
    def _a2a(self, out: torch.Tensor, inp: torch.Tensor, out_splits: List[int], in_splits: List[int]):
        dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)
        return out

    def _dispatch(self, rows_src: torch.Tensor, ctx) -> torch.Tensor:
        send = self.ops.gather_rows(rows_src, ctx["send_tok"], ctx["S"])
        recv = torch.empty((ctx["R"],) + tuple(rows_src.shape[1:]), dtype=rows_src.dtype, device=rows_src.device)
        return self._a2a(recv, send, ctx["recv_counts"], ctx["send_counts"])

    def _return(self, rows: torch.Tensor, ctx, width: int) -> torch.Tensor:
        back = torch.empty((ctx["S"], width), dtype=rows.dtype, device=rows.device)
        return self._a2a(back, rows.contiguous(), ctx["send_counts"], ctx["recv_counts"])

    # ---------------------------------------------------------------- forward
    def forward(self, x: torch.Tensor, idx: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        """out [T, d] fp32 for this rank's T tokens (all k experts, wherever they live)."""
        idx = idx.to(torch.int64).contiguous()
        w = w.to(torch.float32).contiguous()
        x = x.contiguous()
        T, k = idx.shape
        d = x.shape[1]
        counts, pos, send_tok, send_idx, send_w = self.ops.plan(idx, w, self.E, self.n)
        # every rank sends each rank (rows for it, invalid ids here), so a bad id on any rank
        # fails all ranks after the same collective instead of leaving the others waiting
        sc = torch.stack([counts[:self.n], counts[self.n].expand(self.n)], dim=1).contiguous()
        rc = torch.empty_like(sc)
        self._a2a(rc, sc, [1] * self.n, [1] * self.n)
        send_counts = [int(c) for c in counts[:self.n].tolist()]
        rc_h = rc.tolist()
        recv_counts = [int(c) for c, _ in rc_h]
        bad = [r for r, (_, b) in enumerate(rc_h) if b]
        if bad:
            raise ValueError(f"routed expert ids outside [0, {self.E}) on rank(s) {bad}")
        S, R = sum(send_counts), sum(recv_counts)
        ctx = dict(T=T, k=k, d=d, pos=pos, send_tok=send_tok, S=S, R=R, send_counts=send_counts,
                   recv_counts=recv_counts, idx=idx)
        x_recv = self._dispatch(x, ctx)
        idx_recv = self._a2a(torch.empty((R, k), dtype=torch.int64, device=idx.device), send_idx[:S],
                             recv_counts, send_counts)
        w_recv = self._a2a(torch.empty((R, k), dtype=torch.float32, device=w.device), send_w[:S],
                           recv_counts, send_counts)
        self.local_launches = 0
        if R:
            kw = {}
            if getattr(self.local, "accepts_rows_hint", False):   # size the token tiles by the routed slots
                kw["rows_hint"] = int((idx_recv >= 0).sum().item())
            out_recv = self.local.forward(x_recv, idx_recv, w_recv, **kw)
            self.local_launches += self._local_count()
        else:
            out_recv = torch.zeros((0, d), dtype=torch.float32, device=x.device)
        part = self._return(out_recv, ctx, d)
        out = self.ops.combine(part, pos, T, d)
        ctx.update(x_recv=x_recv, idx_recv=idx_recv, w_recv=w_recv)
        self._ctx = ctx
        return out

    # ---------------------------------------------------------------- backward
    def backward(self, g: torch.Tensor):
        """(grad_h [T,d], grad_w [T,k], LoRA grads summed over all ranks) for the last forward."""
        ctx = self._ctx
        if ctx is None:
            raise RuntimeError("backward before forward")
        g = g.contiguous()
        d, k = ctx["d"], ctx["k"]
        g_recv = self._dispatch(g, ctx)
        if ctx["R"]:
            gh_recv, gw_recv, grads = self.local.backward(ctx["x_recv"], ctx["idx_recv"], ctx["w_recv"], g_recv)
            self.local_launches += self._local_count()
        else:
            gh_recv = torch.zeros((0, d), dtype=torch.float32, device=g.device)
            gw_recv = torch.zeros((0, k), dtype=torch.float32, device=g.device)
            grads = None
        gh_part = self._return(gh_recv, ctx, d)
        gw_part = self._return(gw_recv, ctx, k)
        grad_h = self.ops.combine(gh_part, ctx["pos"], ctx["T"], d)
        grad_w = self.ops.combine_slots(gw_part, ctx["pos"], ctx["idx"], self.E)
        grads = self._allreduce_grads(grads, g.device)
        return grad_h, grad_w, grads

    def _local_count(self) -> int:
        fn = getattr(self.local, "last_launch_count", None)
        return int(fn()) if fn is not None else 0

    def _allreduce_grads(self, grads: Optional[Dict[str, torch.Tensor]], device) -> Dict[str, torch.Tensor]:
        shapes = self.local.lora_shapes()
        flat = torch.zeros(sum(a * b for a, b in shapes.values()), dtype=torch.float32, device=device)
        off = 0
        for name in LORA_GRADS:
            a, b = shapes[name]
            if grads is not None and grads.get(name) is not None:
                flat[off:off + a * b] = grads[name].reshape(-1)
            off += a * b
        dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=self.group)
        out, off = {}, 0
        for name in LORA_GRADS:
            a, b = shapes[name]
            out[name] = flat[off:off + a * b].view(a, b)
            off += a * b
        return out
