"""
Expert-parallel routed-expert layer: one process per GPU, experts split over the ranks.

The reference runs every routed expert in one process (lazy_lora/trainer/lazy_trainer.py
:806-880); this module spreads one layer's experts over n ranks of a torch.distributed
process group (NCCL on GPUs) and keeps the single-GPU layer (`RoutedExpertsLayer`, the
ll_moe_forward / ll_moe_backward calls) unchanged on each rank:

  expert e lives on rank floor(e * n / E)        (ll_ep_experts_of_rank)
  forward   plan (ll_ep_plan) -> exchange row counts (the step's only host
            synchronisation reads them) -> gather this rank's token rows once per destination
            rank (ll_ep_gather_rows) -> all-to-all of the rows and of their k-slot headers
            (local expert id or -1, routing weight) -> local layer forward on the rows
            received -> the partial outputs back as fp16 rows with a power-of-two row scale
            (ll_ep_pack_rows, half the fp32 bytes) -> sum of each token's partials in
            ascending rank order (ll_ep_combine_packed)
  backward  the same exchange for the upstream gradient rows (sizes known from the forward:
            no host synchronisation), local layer backward, grad_h partials back packed the
            same way and summed, grad_w slots gathered from the rank that owns each slot's
            expert (ll_ep_combine_slots), and one all-reduce (sum) of the six LoRA gradients
            (the adapters are shared by all experts)

All data crossing ranks goes through NCCL all-to-all / all-reduce into local HBM before any
kernel reads it. The result equals the single-GPU layer on the concatenated tokens up to the
fp32 summation order of the partial outputs and the fp16 rounding (2^-11 relative) of the
returned partial rows.

The index kernels and the exchange order are separated (`ops`), so the same orchestration
runs with another implementation of the index operations.
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
    """The index operations as this library's CUDA kernels (C ABI)."""

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

    def pack_rows(self, part: torch.Tensor) -> torch.Tensor:
        """fp32 partial rows [R, d] -> packed rows (fp16 + power-of-two row scale), viewed as
        int32 [R, d/2 + 4] for the exchange."""
        R, d = part.shape
        out = torch.empty((R, d // 2 + 4), dtype=torch.int32, device=part.device)
        if R:
            L.check(self.lib.ll_ep_pack_rows(out.data_ptr(), part.contiguous().data_ptr(), R, d, L.stream_ptr()),
                    "ll_ep_pack_rows")
            self.launches += 1
        return out

    def combine_packed(self, part: torch.Tensor, pos: torch.Tensor, T: int, d: int) -> torch.Tensor:
        out = torch.empty((T, d), dtype=torch.float32, device=pos.device)
        n = pos.shape[1]
        L.check(self.lib.ll_ep_combine_packed(out.data_ptr(), part.data_ptr() if part.numel() else None,
                                              pos.data_ptr(), T, n, d, L.stream_ptr()), "ll_ep_combine_packed")
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
        # set to a list to record (name, bytes sent, (start, end) CUDA events) per exchange
        self.profile: Optional[list] = None
        self.local_launches = 0    # kernels the local layer launched in the last forward + backward

    # ---------------------------------------------------------------- exchanges
    def _a2a(self, out: torch.Tensor, inp: torch.Tensor, out_splits: List[int], in_splits: List[int], name: str):
        ev = None
        if self.profile is not None:
            ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            ev[0].record()
        dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)
        if ev is not None:
            ev[1].record()
            self.profile.append((name, inp.numel() * inp.element_size(), ev))
        return out

    def _dispatch(self, rows_src: torch.Tensor, ctx, name: str) -> torch.Tensor:
        send = self.ops.gather_rows(rows_src, ctx["send_tok"], ctx["S"])
        recv = torch.empty((ctx["R"],) + tuple(rows_src.shape[1:]), dtype=rows_src.dtype, device=rows_src.device)
        return self._a2a(recv, send, ctx["recv_counts"], ctx["send_counts"], name)

    def _return(self, rows: torch.Tensor, ctx, name: str) -> torch.Tensor:
        rows = rows.contiguous()
        back = torch.empty((ctx["S"],) + tuple(rows.shape[1:]), dtype=rows.dtype, device=rows.device)
        return self._a2a(back, rows, ctx["send_counts"], ctx["recv_counts"], name)

    def _return_combined(self, part: torch.Tensor, ctx, name: str) -> torch.Tensor:
        """Sends fp32 partial rows back packed (fp16 + row scale) and sums each token's
        partials in ascending rank order."""
        back = self._return(self.ops.pack_rows(part), ctx, name)
        return self.ops.combine_packed(back, ctx["pos"], ctx["T"], ctx["d"])

    # ---------------------------------------------------------------- forward
    def forward(self, x: torch.Tensor, idx: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        """out [T, d] fp32 for this rank's T tokens (all k experts, wherever they live)."""
        idx = idx.to(torch.int64).contiguous()
        w = w.to(torch.float32).contiguous()
        x = x.contiguous()
        T, k = idx.shape
        d = x.shape[1]
        n = self.n
        counts, pos, send_tok, send_idx, send_w = self.ops.plan(idx, w, self.E, n)
        # every rank sends each rank (rows for it, invalid ids here), so a bad id on any rank
        # fails all ranks after the same collective instead of leaving the others waiting
        sc = torch.stack([counts[:n], counts[n].expand(n)], dim=1).contiguous()
        rc = torch.empty_like(sc)
        self._a2a(rc, sc, [1] * n, [1] * n, "counts")
        # the step's one host synchronisation: this rank's counts and the received ones together
        host = torch.cat([counts[:n + 1], rc.reshape(-1)]).tolist()
        send_counts = [int(c) for c in host[:n]]
        own_bad = int(host[n])
        recv_counts = [int(c) for c in host[n + 1::2]]
        bad = [r for r, b in enumerate(host[n + 2::2]) if b]
        if bad:
            raise ValueError(f"routed expert ids outside [0, {self.E}) on rank(s) {bad}")
        S, R = sum(send_counts), sum(recv_counts)
        # routed slots per received row, estimated from this rank's own send side (a row carries
        # 1..k slots); it sizes the local layer's token tiles, forward and backward alike
        per_row = (T * k - own_bad) / S if S else float(k)
        rows_hint = max(R, min(R * k, int(round(R * per_row))))
        ctx = dict(T=T, k=k, d=d, pos=pos, send_tok=send_tok, S=S, R=R, send_counts=send_counts,
                   recv_counts=recv_counts, idx=idx, rows_hint=rows_hint)
        x_recv = self._dispatch(x, ctx, "dispatch x")
        # the k-slot headers (local expert id, routing weight) in one exchange
        hdr = torch.cat([send_idx[:S].view(torch.int32), send_w[:S].view(torch.int32)], dim=1)
        hdr_recv = self._a2a(torch.empty((R, 3 * k), dtype=torch.int32, device=idx.device), hdr, recv_counts,
                             send_counts, "dispatch headers")
        idx_recv = hdr_recv[:, :2 * k].contiguous().view(torch.int64)
        w_recv = hdr_recv[:, 2 * k:].contiguous().view(torch.float32)
        self.local_launches = 0
        if R:
            kw = {"rows_hint": rows_hint} if getattr(self.local, "accepts_rows_hint", False) else {}
            out_recv = self.local.forward(x_recv, idx_recv, w_recv, **kw)
            self.local_launches += self._local_count()
        else:
            out_recv = torch.zeros((0, d), dtype=torch.float32, device=x.device)
        out = self._return_combined(out_recv, ctx, "combine out")
        ctx.update(x_recv=x_recv, idx_recv=idx_recv, w_recv=w_recv)
        self._ctx = ctx
        return out

    # ---------------------------------------------------------------- backward
    def backward(self, g: torch.Tensor):
        """(grad_h [T,d], grad_w [T,k], LoRA grads summed over all ranks) for the last forward.
        No host synchronisation: the exchange sizes are the forward's."""
        ctx = self._ctx
        if ctx is None:
            raise RuntimeError("backward before forward")
        g = g.contiguous()
        d, k = ctx["d"], ctx["k"]
        g_recv = self._dispatch(g, ctx, "dispatch g")
        if ctx["R"]:
            gh_recv, gw_recv, grads = self.local.backward(ctx["x_recv"], ctx["idx_recv"], ctx["w_recv"], g_recv)
            self.local_launches += self._local_count()
        else:
            gh_recv = torch.zeros((0, d), dtype=torch.float32, device=g.device)
            gw_recv = torch.zeros((0, k), dtype=torch.float32, device=g.device)
            grads = None
        grad_h = self._return_combined(gh_recv, ctx, "combine grad_h")
        gw_part = self._return(gw_recv, ctx, "return grad_w")
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
        ev = None
        if self.profile is not None:
            ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            ev[0].record()
        dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=self.group)
        if ev is not None:
            ev[1].record()
            self.profile.append(("all-reduce LoRA grads", flat.numel() * 4, ev))
        out, off = {}, 0
        for name in LORA_GRADS:
            a, b = shapes[name]
            out[name] = flat[off:off + a * b].view(a, b)
            off += a * b
        return out
