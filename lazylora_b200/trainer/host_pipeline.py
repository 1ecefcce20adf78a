"""
Training steps fed from pinned host memory, with the host<->device copies overlapped with
compute.

A training loop whose batches arrive in host memory pays, per step, the copy of the inputs
to HBM and the copy of the results back (the reference reads and writes host tensors on every
call: lazy_lora/trainer/lazy_trainer.py:806-880 runs entirely on the CPU). On the GPU those
copies run on the copy engines, so they need not stall the SMs: `HostStepPipeline` issues step
i + 1's input copies on an input stream while step i computes, and step i's result copies on
an output stream while step i + 1 computes. Device input buffers are double-buffered; an input
slot is rewritten only after the step that read it finished, and result tensors are kept alive
for the output stream (`record_stream`) until their copies are done.

The step itself is any callable (x_dev, g_dev) -> sequence of device tensors (e.g. route +
forward + backward of one layer); `run` copies the tensors named by `out_index` back.
"""
from typing import Callable, List, Sequence

import torch


class CapturedStep:
    """`step_fn(x, g)` captured once as a CUDA graph over the fixed device tensors x and g;
    replay() reruns the whole step (tens of kernels) as one graph launch and returns the
    same output tensors, overwritten. The step must not synchronise with the host (the
    library's routing, forward and backward calls do not). Work of a replay is ordered after
    the current stream's earlier work and before its later work."""

    def __init__(self, step_fn: Callable, x: torch.Tensor, g: torch.Tensor, warmup: int = 1):
        cur = torch.cuda.current_stream(x.device)
        side = torch.cuda.Stream(device=x.device)
        side.wait_stream(cur)
        with torch.cuda.stream(side):
            for _ in range(warmup):             # lazily allocated workspaces exist before capture
                step_fn(x, g)
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph, stream=side):
                self.outputs = step_fn(x, g)
        cur.wait_stream(side)
        self.x, self.g = x, g

    def replay(self):
        self.graph.replay()
        return self.outputs


class HostStepPipeline:
    """Runs `step_fn` over batches held in pinned host memory, copies overlapped with compute.

    step_fn: (x_dev, g_dev) -> sequence of device tensors (the step's results).
    out_index: which results to copy back to host, in the order of the host buffers.
    graph: run each step as a CUDA graph (one per input slot, captured on first use); a
        graph's outputs are rewritten by its next replay, which therefore waits for their
        copies to the host.
    """

    def __init__(self, step_fn: Callable, out_index: Sequence[int], device=None, graph: bool = False):
        self.step_fn = step_fn
        self.out_index = list(out_index)
        self.device = torch.device(device if device is not None else "cuda")
        self.h2d = torch.cuda.Stream(device=self.device)
        self.d2h = torch.cuda.Stream(device=self.device)
        self.graph = graph
        self._captured = None
        self._slots = None

    def _buffers(self, x_h: torch.Tensor, g_h: torch.Tensor):
        want = (tuple(x_h.shape), x_h.dtype, tuple(g_h.shape), g_h.dtype)
        if self._slots is None or self._slots[0] != want:
            mk = lambda t: torch.empty(t.shape, dtype=t.dtype, device=self.device)
            self._slots = (want, [(mk(x_h), mk(g_h)) for _ in range(2)])
            self._captured = None
        return self._slots[1]

    def _graphs(self, slots, x_h, g_h):
        if self._captured is None:
            for s in range(2):                   # capture on real data so the warm-up is valid
                slots[s][0].copy_(x_h)
                slots[s][1].copy_(g_h)
            self._captured = [CapturedStep(self.step_fn, slots[s][0], slots[s][1]) for s in range(2)]
            torch.cuda.current_stream(self.device).synchronize()
        return self._captured

    def run(self, xs_h: Sequence[torch.Tensor], gs_h: Sequence[torch.Tensor],
            outs_h: Sequence[Sequence[torch.Tensor]]) -> List:
        """Run len(xs_h) steps. xs_h[i], gs_h[i]: pinned host inputs of step i; outs_h[i]: pinned
        host tensors receiving step i's results out_index (the same buffers may serve several
        steps: copies into them are ordered). Returns the device results of the last step.
        Work is enqueued on the current stream and the two copy streams; nothing waits on the
        host. The current stream is ordered after every copy when `run` returns."""
        n = len(xs_h)
        if n == 0:
            return []
        if len(gs_h) != n or len(outs_h) != n:
            raise ValueError("one input pair and one output set per step")
        for t in list(xs_h) + list(gs_h) + [o for os in outs_h for o in os]:
            if t.device.type != "cpu" or not t.is_pinned():
                raise ValueError("host buffers must be pinned CPU tensors")
        comp = torch.cuda.current_stream(self.device)
        slots = self._buffers(xs_h[0], gs_h[0])
        graphs = self._graphs(slots, xs_h[0], gs_h[0]) if self.graph else None
        copied = [None, None]     # event: the outputs of slot s's graph reached the host
        start = torch.cuda.Event()
        start.record(comp)
        self.h2d.wait_event(start)
        self.d2h.wait_event(start)
        loaded = [None, None]     # event: slot's inputs landed
        freed = [None, None]      # event: the step reading the slot finished

        def load(i):
            s = i % 2
            with torch.cuda.stream(self.h2d):
                if freed[s] is not None:
                    self.h2d.wait_event(freed[s])
                slots[s][0].copy_(xs_h[i], non_blocking=True)
                slots[s][1].copy_(gs_h[i], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(self.h2d)
            loaded[s] = ev

        load(0)
        if n > 1:
            load(1)
        res = []
        for i in range(n):
            s = i % 2
            comp.wait_event(loaded[s])
            if graphs is not None:
                if copied[s] is not None:
                    comp.wait_event(copied[s])
                res = graphs[s].replay()
            else:
                res = self.step_fn(slots[s][0], slots[s][1])
            done = torch.cuda.Event()
            done.record(comp)
            freed[s] = done
            with torch.cuda.stream(self.d2h):
                self.d2h.wait_event(done)
                for j, o in zip(self.out_index, outs_h[i]):
                    o.copy_(res[j], non_blocking=True)
                    if graphs is None:
                        res[j].record_stream(self.d2h)
                ev = torch.cuda.Event()
                ev.record(self.d2h)
                copied[s] = ev
            if i + 2 < n:
                load(i + 2)
        end = torch.cuda.Event()
        end.record(self.d2h)
        comp.wait_event(end)
        return res
