"""
Streaming routed-expert weights from pinned host memory into HBM, overlapped with compute.

B200 counterpart of DynamicExpertStreamer.stream_experts (lazy_lora/streaming/
expert_streamer.py:315-369). The reference reads one expert at a time from disk with a
depth-2 read-ahead thread and multiplies it on the CPU; the whole active set of a layer is
known once the router ran (its sort_by_disk_order, :286-304, orders the reads). Here:

  * `HostExpertStore` keeps each layer's MXFP4 stacks (the reference layout: packed
    [E, rows, cols/2] and E8M0 scales [E, rows, cols/32] for w1, w3, w2) in pinned host
    memory, the stage the reference's mmap reader feeds;
  * `ExpertStreamer.stream_layer(layer, expert_ids)` splits the layer's active experts (in
    ascending id order, i.e. disk order for a packed checkpoint) into groups and copies
    group i + 1 host -> HBM on a copy stream (one cudaMemcpyAsync per contiguous run of
    experts per stack, at PCIe speed) while the caller computes on group i; each group is
    handed out as a RoutedExpertsLayer over the staged stacks (the decode bias is computed on
    the compute stream once the copy event fired; the transposed copy the backward reads is
    built only for a group that runs a backward, into buffers each staging slot keeps). Two
    staging slots bound the HBM held.
    `prefetch(next_layer, ids)` lets the copy engine start the next layer's first group
    during the current layer's last group when the next expert set is known (all experts
    when every expert is active, the forward's set during the backward), so the copies
    run back to back across layers;
  * `streamed_forward` / `streamed_backward` run one layer group by group: the routed
    experts of a group see the token slots routed to them, all other slots are -1, and the
    group results add up to the layer's (the same partial-sum algebra as expert parallelism:
    outputs and grad_h summed in group order, each grad_w slot from its expert's group, LoRA
    gradients summed).

`stream_experts(layer, ids, depth)` keeps the reference's generator interface: it yields
(expert_id, bundle) pairs whose tensors are HBM views of the staged groups.
"""
from typing import Dict, Iterator, List, Optional, Sequence, Tuple

import torch

from .routed_experts import RoutedExpertsLayer

STACKS = ("w1p", "w1s", "w3p", "w3s", "w2p", "w2s")


class HostExpertStore:
    """Per-layer MXFP4 expert stacks in pinned host memory (reference layout)."""

    def __init__(self):
        self.layers: Dict[int, Dict[str, torch.Tensor]] = {}

    def add_layer(self, layer_idx: int, stacks: Dict[str, torch.Tensor]) -> None:
        pinned = {}
        for name in STACKS:
            t = stacks[name]
            p = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
            p.copy_(t)
            pinned[name] = p
        e = {pinned[n].shape[0] for n in STACKS}
        if len(e) != 1:
            raise ValueError("all stacks of a layer need the same expert count")
        self.layers[layer_idx] = pinned

    def add_layer_from_checkpoint(self, layer_idx: int, index, num_experts: int, threads: int = 16) -> int:
        """Read layer `layer_idx`'s experts 0..num_experts-1 from a safetensors checkpoint
        (lazylora_b200.streaming.safetensors_reader.SafetensorsIndex) straight into pinned
        stacks, with one parallel batch of reads; returns the bytes read."""
        from ..streaming.safetensors_reader import read_layer_experts
        stacks, nbytes = read_layer_experts(index, layer_idx, range(num_experts), pin=True, threads=threads)
        self.layers[layer_idx] = {n: stacks[n] for n in STACKS}
        return nbytes

    def num_experts(self, layer_idx: int) -> int:
        return self.layers[layer_idx]["w1p"].shape[0]

    def expert_bytes(self, layer_idx: int) -> int:
        L = self.layers[layer_idx]
        return sum(L[n][0].numel() * L[n].element_size() for n in STACKS)


class ExpertBundle:
    """One expert's packed MXFP4 weights in HBM (the reference's ExpertWeightBundle, packed form)."""

    def __init__(self, expert_idx: int, g: Dict[str, torch.Tensor], j: int):
        self.expert_idx = expert_idx
        self.gate_packed, self.gate_scale = g["w1p"][j], g["w1s"][j]
        self.up_packed, self.up_scale = g["w3p"][j], g["w3s"][j]
        self.down_packed, self.down_scale = g["w2p"][j], g["w2s"][j]
        self.packed = True


def _runs(ids: Sequence[int]) -> List[Tuple[int, int, int]]:
    """(first id, position in the group, length) of each run of consecutive ids."""
    out = []
    i = 0
    while i < len(ids):
        j = i
        while j + 1 < len(ids) and ids[j + 1] == ids[j] + 1:
            j += 1
        out.append((ids[i], i, j - i + 1))
        i = j + 1
    return out


class ExpertStreamer:
    """Host -> HBM streaming of a layer's active experts in groups, double-buffered.

    lora: dict with A_g, B_g, A_u, B_u, A_d, B_d (device tensors shared by all experts).
    group_experts: experts per group (the copy / compute granularity).
    """

    def __init__(self, store: HostExpertStore, lora: Dict[str, torch.Tensor], lora_scaling: float,
                 group_experts: int = 224, device=None, slots: int = 2):
        if group_experts <= 0 or slots < 2:
            raise ValueError("group_experts > 0 and at least two staging slots")
        self.store = store
        self.lora = lora
        self.scaling = float(lora_scaling)
        self.group = int(group_experts)
        self.device = torch.device(device if device is not None else "cuda")
        self.copy_stream = torch.cuda.Stream(device=self.device)
        self.n_slots = slots
        self._slots: List[Optional[Dict[str, torch.Tensor]]] = [None] * slots
        self._tslots: List[Optional[Dict[str, torch.Tensor]]] = [None] * slots
        self._slot_free: List[Optional[torch.cuda.Event]] = [None] * slots
        self._rot = 0                 # next staging slot
        self._hint = None             # (layer, ids) streamed next, see prefetch
        self._prefetched = None       # (layer, first group, slot, event) already being copied
        self.bytes_copied = 0

    def _slot(self, i: int, layer_idx: int) -> Dict[str, torch.Tensor]:
        L = self.store.layers[layer_idx]
        shapes = {n: (self.group,) + tuple(L[n].shape[1:]) for n in STACKS}
        s = self._slots[i]
        if s is None or any(s[n].shape != shapes[n] or s[n].dtype != L[n].dtype for n in STACKS):
            s = {n: torch.empty(shapes[n], dtype=L[n].dtype, device=self.device) for n in STACKS}
            self._slots[i] = s
        return s

    def _tslot(self, i: int, layer_idx: int) -> Dict[str, torch.Tensor]:
        """The transposed-copy buffers of staging slot i, sized for a full group: allocated
        the first time a group in that slot runs a backward, reused by every later group."""
        _, f, dh = self.store.layers[layer_idx]["w1p"].shape
        d, G, u8, f16 = 2 * dh, self.group, torch.uint8, torch.float16
        want = {"w1t": ((G, d, f // 2), u8), "w3t": ((G, d, f // 2), u8), "w2t": ((G, f, d // 2), u8),
                "s1t": ((G, d // 32, f), f16), "s3t": ((G, d // 32, f), f16), "s2t": ((G, f // 32, d), f16)}
        t = self._tslots[i]
        if t is None or any(tuple(t[n].shape) != want[n][0] or t[n].dtype != want[n][1] for n in want):
            t = {n: torch.empty(shape, dtype=dt, device=self.device) for n, (shape, dt) in want.items()}
            self._tslots[i] = t
        return t

    def _copy_group(self, layer_idx: int, ids: List[int], slot: int) -> torch.cuda.Event:
        L = self.store.layers[layer_idx]
        dst = self._slot(slot, layer_idx)
        with torch.cuda.stream(self.copy_stream):
            if self._slot_free[slot] is not None:          # the slot's previous group is done
                self.copy_stream.wait_event(self._slot_free[slot])
            for first, pos, n in _runs(ids):
                for name in STACKS:
                    dst[name][pos:pos + n].copy_(L[name][first:first + n], non_blocking=True)
                    self.bytes_copied += n * L[name][0].numel() * L[name].element_size()
            ev = torch.cuda.Event()
            ev.record(self.copy_stream)
        return ev

    def _start(self, layer_idx: int, ids: List[int]):
        """Start copying one group into the next slot of the rotation."""
        slot = self._rot
        self._rot = (self._rot + 1) % self.n_slots
        return layer_idx, tuple(ids), slot, self._copy_group(layer_idx, ids, slot)

    def prefetch(self, layer_idx: int, expert_ids: Sequence[int]) -> None:
        """Name the layer streamed next: its first group is copied while the last group of
        the current layer computes (the caller knows the next expert set, e.g. all experts
        when every expert is active, or the forward's set during the backward)."""
        self._hint = (layer_idx, sorted(int(e) for e in expert_ids))

    def stream_layer(self, layer_idx: int, expert_ids: Sequence[int]) -> Iterator[Tuple[List[int], RoutedExpertsLayer]]:
        """Yield (expert ids, RoutedExpertsLayer over them, local ids 0..n-1) group by group."""
        ids = sorted(int(e) for e in expert_ids)
        groups = [ids[i:i + self.group] for i in range(0, len(ids), self.group)]
        if not groups:
            return
        cur = torch.cuda.current_stream(self.device)
        pf, self._prefetched = self._prefetched, None
        pend = [pf if pf is not None and pf[0] == layer_idx and pf[1] == tuple(groups[0])
                else self._start(layer_idx, groups[0])]
        for gi, g in enumerate(groups):
            if gi + 1 < len(groups):                       # next group's copy overlaps this one
                pend.append(self._start(layer_idx, groups[gi + 1]))
            elif self._hint is not None:                   # last group: start the next layer's first
                hl, hids = self._hint
                self._hint = None
                if hids:
                    self._prefetched = self._start(hl, hids[:self.group])
            _, _, slot, ev = pend[gi]
            cur.wait_event(ev)
            st = self._slots[slot]
            n = len(g)
            lo = self.lora
            # the transposed copy is built only if this group runs a backward, into the slot's
            # persistent buffers (no allocation per group)
            layer = RoutedExpertsLayer(st["w1p"][:n], st["w1s"][:n], st["w3p"][:n], st["w3s"][:n], st["w2p"][:n],
                                       st["w2s"][:n], lo["A_g"], lo["B_g"], lo["A_u"], lo["B_u"], lo["A_d"],
                                       lo["B_d"], self.scaling, prepare_backward=False,
                                       transposed=lambda sl=slot, li=layer_idx: self._tslot(sl, li))
            yield g, layer
            done = torch.cuda.Event()
            done.record(cur)
            self._slot_free[slot] = done

    def stream_experts(self, layer_idx: int, expert_ids: List[int], depth: int = 2):
        """The reference's generator interface: (expert_id, bundle) in ascending id order, the
        bundles' tensors HBM views of the staged groups (valid until the group after next)."""
        del depth   # the group size sets the read-ahead here
        for g, layer in self.stream_layer(layer_idx, expert_ids):
            staged = {"w1p": layer.w1p, "w1s": layer.w1s, "w3p": layer.w3p, "w3s": layer.w3s, "w2p": layer.w2p,
                      "w2s": layer.w2s}
            for j, e in enumerate(g):
                yield e, ExpertBundle(e, staged, j)


def _local_ids(idx: torch.Tensor, group: List[int], num_experts: int) -> torch.Tensor:
    lut = torch.full((num_experts,), -1, dtype=torch.int64, device=idx.device)
    lut[torch.tensor(group, dtype=torch.int64, device=idx.device)] = torch.arange(len(group), device=idx.device)
    safe = idx.clamp(min=0)
    return torch.where(idx >= 0, lut[safe], idx)


def _group_rows_hint(idx: torch.Tensor, group: List[int], ids: Sequence[int]) -> int:
    """Routed slots a group's layer sees, estimated without reading the routing back: the
    layer's T * k slots spread evenly over its active experts (it sets the token-tile width;
    forward and backward compute the same value)."""
    return max(1, round(idx.numel() * len(group) / max(1, len(ids))))


def streamed_forward(streamer: ExpertStreamer, layer_idx: int, x: torch.Tensor, idx: torch.Tensor,
                     w: torch.Tensor, expert_ids: Optional[Sequence[int]] = None):
    """out [T, d] of one layer, its experts streamed group by group. Returns (out, staged)
    where `staged` keeps what streamed_backward needs when it re-streams the layer."""
    E = streamer.store.num_experts(layer_idx)
    ids = expert_ids if expert_ids is not None else torch.unique(idx[idx >= 0]).tolist()
    out = None
    for g, layer in streamer.stream_layer(layer_idx, ids):
        o = layer.forward(x, _local_ids(idx, g, E), w, rows_hint=_group_rows_hint(idx, g, ids))
        out = o if out is None else out.add_(o)
    if out is None:
        out = torch.zeros((x.shape[0], x.shape[1]), dtype=torch.float32, device=x.device)
    return out, ids


def streamed_backward(streamer: ExpertStreamer, layer_idx: int, x: torch.Tensor, idx: torch.Tensor,
                      w: torch.Tensor, g: torch.Tensor, expert_ids: Sequence[int]):
    """(grad_h, grad_w, LoRA grads) of one layer, re-streaming its experts group by group."""
    E = streamer.store.num_experts(layer_idx)
    grad_h = grad_w = grads = None
    for grp, layer in streamer.stream_layer(layer_idx, expert_ids):
        li = _local_ids(idx, grp, E)
        gh, gw, gr = layer.backward(x, li, w, g, rows_hint=_group_rows_hint(idx, grp, expert_ids))
        if grad_h is None:
            grad_h, grad_w, grads = gh, gw, gr
        else:
            grad_h.add_(gh)
            grad_w.add_(gw)             # slots of other groups are 0 in each group's grad_w
            for k2 in grads:
                grads[k2].add_(gr[k2])
    return grad_h, grad_w, grads


class StreamedLocalExperts:
    """One layer's experts held in pinned host memory and streamed into HBM group by group for
    every forward and backward, with the interface of a resident RoutedExpertsLayer that
    ExpertParallelLayer takes as its local layer: under expert parallelism each rank's store
    holds only that rank's block of experts (ids local to the rank), so a rank moves 1/n of the
    layer's bytes over its PCIe link instead of all of them (configs[4] on n GPUs; the
    reference streams every expert to its one GPU, expert_streamer.py:315-369).

    expert_ids: the experts streamed for each call, ascending (None: those the call routes to,
    read back from the routing once, a host synchronisation).
    """

    accepts_rows_hint = False

    def __init__(self, streamer: ExpertStreamer, layer_idx: int, expert_ids: Optional[Sequence[int]] = None):
        self.streamer = streamer
        self.layer_idx = int(layer_idx)
        self.E = streamer.store.num_experts(layer_idx)
        self.expert_ids = list(expert_ids) if expert_ids is not None else None
        self._ids = None

    def forward(self, x: torch.Tensor, idx: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        out, self._ids = streamed_forward(self.streamer, self.layer_idx, x, idx, w, expert_ids=self.expert_ids)
        return out

    def backward(self, x: torch.Tensor, idx: torch.Tensor, w: torch.Tensor, g: torch.Tensor):
        if self._ids is None:
            raise RuntimeError("backward before forward")
        return streamed_backward(self.streamer, self.layer_idx, x, idx, w, g, self._ids)

    def lora_shapes(self) -> Dict[str, tuple]:
        lo = self.streamer.lora
        r, d = lo["A_g"].shape
        f = lo["B_g"].shape[0]
        return {"dA_g": (r, d), "dB_g": (f, r), "dA_u": (r, d), "dB_u": (f, r), "dA_d": (r, f), "dB_d": (d, r)}
