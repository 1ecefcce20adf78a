"""
CPU restatement of the expert-parallel index operations. TEST INFRASTRUCTURE ONLY.

The reference has no expert parallelism: lazy_lora/trainer/lazy_trainer.py:806-880 runs all
routed experts in one process. Parity of the expert-parallel layer is therefore anchored on
that single-process result (moe_oracle.experts_forward / experts_backward over all tokens and
all experts): an n-rank run must reproduce it. This module restates, in plain torch CPU
loops, the index operations the CUDA kernels of lazylora_b200/csrc/expert_parallel.cu
implement (plan, row gather, ordered combine, packing of the returned partial rows and the
combine over them, slot combine), so that

  * the CUDA plan can be checked bit-exactly against `plan` on the GPU, and
  * the rank orchestration (lazylora_b200.trainer.expert_parallel.ExpertParallelLayer) can run
    on CPU `gloo` ranks with these operations and the moe_oracle expert loop plugged in.

Only tests/ may import it.
"""
from typing import Tuple

import torch


def owner(e: int, E: int, n: int) -> int:
    return (e * n) // E


def first(r: int, E: int, n: int) -> int:
    return (r * E + n - 1) // n


class OracleEPOps:
    """Same interface as lazylora_b200.trainer.expert_parallel.CudaEPOps, on CPU tensors."""

    def plan(self, idx: torch.Tensor, w: torch.Tensor, E: int, n: int):
        T, k = idx.shape
        counts = [0] * (n + 1)
        pos = torch.full((T, n), -1, dtype=torch.int32)
        rows_tok, rows_idx, rows_w = [[] for _ in range(n)], [[] for _ in range(n)], [[] for _ in range(n)]
        for t in range(T):
            ranks = set()
            for j in range(k):
                e = int(idx[t, j])
                if 0 <= e < E:
                    ranks.add(owner(e, E, n))
                else:
                    counts[n] += 1
            for r in sorted(ranks):
                pos[t, r] = len(rows_tok[r])          # rank-local row, offset below
                rows_tok[r].append(t)
                hdr_i, hdr_w = [], []
                for j in range(k):
                    e = int(idx[t, j])
                    here = 0 <= e < E and owner(e, E, n) == r
                    hdr_i.append(e - first(r, E, n) if here else -1)
                    hdr_w.append(float(w[t, j]) if here else 0.0)
                rows_idx[r].append(hdr_i)
                rows_w[r].append(hdr_w)
        base = 0
        for r in range(n):
            counts[r] = len(rows_tok[r])
            col = pos[:, r]
            col[col >= 0] += base
            base += counts[r]
        send_tok = torch.tensor([t for r in range(n) for t in rows_tok[r]], dtype=torch.int32)
        send_idx = torch.tensor([h for r in range(n) for h in rows_idx[r]], dtype=torch.int64).reshape(-1, k)
        send_w = torch.tensor([h for r in range(n) for h in rows_w[r]], dtype=torch.float32).reshape(-1, k)
        return torch.tensor(counts, dtype=torch.int32), pos, send_tok, send_idx, send_w

    def gather_rows(self, src: torch.Tensor, tok: torch.Tensor, rows: int) -> torch.Tensor:
        return src.index_select(0, tok[:rows].to(torch.int64)).contiguous()

    def combine(self, part: torch.Tensor, pos: torch.Tensor, T: int, d: int) -> torch.Tensor:
        out = torch.zeros((T, d), dtype=torch.float32)
        for t in range(T):
            for r in range(pos.shape[1]):
                p = int(pos[t, r])
                if p >= 0:
                    out[t] += part[p]
        return out

    def pack_rows(self, part: torch.Tensor) -> torch.Tensor:
        """fp32 rows [R, d] -> packed rows [R, 2d + 16] bytes (as int32 [R, d/2 + 4]): d fp16
        values times 2^e, e bringing the row's largest magnitude into [2^14, 2^15), then the fp32
        2^-e and 12 zero bytes (the layout of ll_ep_pack_rows)."""
        R, d = part.shape
        out = torch.zeros((R, 2 * d + 16), dtype=torch.uint8)
        for i in range(R):
            mx = float(part[i].abs().max()) if d else 0.0
            e = 0
            if mx > 0 and mx != float("inf") and mx == mx:
                e = 15 - int(torch.frexp(torch.tensor(mx, dtype=torch.float32)).exponent)
            out[i, :2 * d] = (part[i] * 2.0 ** e).to(torch.float16).view(torch.uint8)
            out[i, 2 * d:2 * d + 4] = torch.tensor([2.0 ** -e], dtype=torch.float32).view(torch.uint8)
        return out.view(torch.int32)

    def combine_packed(self, part: torch.Tensor, pos: torch.Tensor, T: int, d: int) -> torch.Tensor:
        """combine over packed rows: each row unpacked to fp32 (fp16 value x its 2^-e), then the
        sum over ranks in ascending order."""
        b = part.view(torch.uint8).reshape(-1, 2 * d + 16)
        out = torch.zeros((T, d), dtype=torch.float32)
        for t in range(T):
            for r in range(pos.shape[1]):
                p = int(pos[t, r])
                if p >= 0:
                    inv = float(b[p, 2 * d:2 * d + 4].view(torch.float32)[0])
                    out[t] += b[p, :2 * d].view(torch.float16).float() * inv
        return out

    def combine_slots(self, part: torch.Tensor, pos: torch.Tensor, idx: torch.Tensor, E: int) -> torch.Tensor:
        T, k = idx.shape
        n = pos.shape[1]
        out = torch.zeros((T, k), dtype=torch.float32)
        for t in range(T):
            for j in range(k):
                e = int(idx[t, j])
                if 0 <= e < E:
                    p = int(pos[t, owner(e, E, n)])
                    if p >= 0:
                        out[t, j] = part[p, j]
        return out


def split_experts(inp, E: int, n: int, rank: int):
    """The expert-weight slices of `rank` (contiguous block) from a full-layer input dict."""
    lo, hi = first(rank, E, n), first(rank + 1, E, n)
    out = dict(inp)
    for key in ("w1p", "w1s", "w3p", "w3s", "w2p", "w2s"):
        out[key] = inp[key][lo:hi]
    return out, lo, hi


def expected_counts(idx: torch.Tensor, E: int, n: int) -> Tuple[int, ...]:
    """Rows each rank receives from these tokens (one per token and owning rank)."""
    c = [0] * n
    for t in range(idx.shape[0]):
        for r in {owner(int(e), E, n) for e in idx[t].tolist() if 0 <= int(e) < E}:
            c[r] += 1
    return tuple(c)
