"""
Benchmark of the routed-expert MoE layer (router + forward + manual backward with LoRA) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = route the tokens (KimiK3MoERouter), run the routed-expert forward (gate/up with
SiTU-GLU, down, weighted combine, LoRA fused) and the full backward (grad_h, grad_w and the
six LoRA gradients) of one 896-expert MXFP4 layer, d=7168, f=2048, top-8. Expert weights
(~21 GB) are resident in HBM, far larger than the 126 MB L2, so every step streams them from
DRAM. Inputs are seeded synthetic tensors with the distributions of BASELINE.json (the Kimi
K3 checkpoint is not available).

  N = 1   BASELINE configs[1]: T = 1024 tokens on one GPU.
  N > 1   BASELINE configs[2]: T = 8192 tokens in total, 8192 / N per rank, the experts split
          expert-parallel over the N ranks (896 / N each) with NCCL all-to-all dispatch and
          combine: "scaling": "strong". Rank 0 also times the same 8192-token layer on its own
          GPU in the same job, and the line reports strong_efficiency = t(1 GPU) / (N t(N)).
Timing is device time (CUDA events on the launching stream), barrier + synchronize on both
sides, max over ranks.

--impl reference times the reference's own CPU implementation of the path on this box's
host cores: the reference's C kernel (lazy_lora/native/mxfp4_gemm.c, compiled from source into
oracle/_ref) driven by the restated expert loop of oracle/moe_oracle.py, with the router on
the CPU. At N = 1 each timed step is the whole configs[1] layer; at N > 1 (configs[2], 8192
tokens, too long for a bounded run) each step is a sample of the layer's experts with all
their routed tokens, scaled to the layer.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from typing import Optional

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

METRIC = "MoE-layer fwd+bwd tokens/s (d=7168, f=2048, E=896, top-8, LoRA r=16)"
UNIT = "tokens/s"


# DRAM bytes (read + write) per touched expert of each grouped-GEMM launch (F1, F2, B1, B2),
# from one ncu capture of the same kernels at d=7168, f=2048, 64 experts, 9 tokens per expert.
# Weight reads dominate, so a launch's traffic scales with the number of experts it touches.
NCU_DRAM_BYTES_PER_EXPERT = {
    (7168, 2048): [(1015.426e6 + 13.455616e6) / 64, (502.113e6 + 16.451584e6) / 64,
                   (548.347e6 + 9.062400e6) / 64, (1061.752e6 + 18.494720e6) / 64],
}


def _peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as fh:
            p = json.load(fh)
        return float(p["hbm_gbs"]), float(p.get("bf16_tflops", 1639.8)), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """SM clock and clock-event (throttle) reasons polled through NVML (read-only queries)
    every 20 ms by one background thread, started before the warm-up; a `with` block marks
    the timed region and summary() reports the samples taken inside it (or, for a region
    shorter than five samples, those of the 0.25 s before it too: the warm-up of the same
    work). Reports nothing when NVML is absent."""
    REASONS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40), ("sw_thermal_slowdown", 0x20),
               ("sw_power_cap", 0x4), ("hw_power_brake_slowdown", 0x80))
    _samples = []          # (time, sm MHz, reason bits)
    _mx = None
    _thread = None

    @classmethod
    def start(cls, gpu_index: int):
        if cls._thread is not None:
            return
        try:
            import pynvml as nv
            nv.nvmlInit()
            try:   # the CUDA device's PCI address (CUDA and NVML may number GPUs differently)
                p = torch.cuda.get_device_properties(gpu_index)
                h = nv.nvmlDeviceGetHandleByPciBusId("%08x:%02x:%02x.0" % (p.pci_domain_id, p.pci_bus_id,
                                                                          p.pci_device_id))
            except Exception:
                h = nv.nvmlDeviceGetHandleByIndex(gpu_index)
            cls._mx = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
        except Exception:
            cls._thread = False
            return

        def run():
            while True:
                try:
                    cls._samples.append((time.time(), float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)),
                                         int(nv.nvmlDeviceGetCurrentClocksEventReasons(h))))
                except Exception:
                    return
                time.sleep(0.02)

        cls._thread = threading.Thread(target=run, daemon=True)
        cls._thread.start()

    def __init__(self, gpu_index: int):
        ClockSampler.start(gpu_index)

    def __enter__(self):
        self.t0 = time.time()
        return self

    def __exit__(self, *exc):
        self.t1 = time.time()

    def summary(self):
        win = [x for x in list(self._samples) if self.t0 <= x[0] <= self.t1]
        extended = len(win) < 5
        if extended:
            win = [x for x in list(self._samples) if self.t0 - 0.25 <= x[0] <= self.t1]
        reasons = sorted({name for _, _, r in win for name, bit in self.REASONS if r & bit})
        return {"sm_mhz": statistics.median(x[1] for x in win) if win else None, "sm_max_mhz": self._mx,
                "reasons": reasons, "samples": len(win), "source": "nvml every 20 ms" +
                (", window includes the 0.25 s warm-up before the timed region" if extended else "")}


def dist_setup(args):
    if args.gpus > 1 or int(os.environ.get("WORLD_SIZE", "1")) > 1:
        import datetime
        import torch.distributed as dist
        rank = int(os.environ.get("RANK", "0"))
        local = int(os.environ.get("LOCAL_RANK", "0"))
        world = int(os.environ.get("WORLD_SIZE", "1"))
        backend = "nccl" if torch.cuda.is_available() else "gloo"
        os.environ.setdefault("NCCL_DEBUG", "WARN")   # no version banner on stdout: one JSON line only
        if torch.cuda.is_available():
            torch.cuda.set_device(local)
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=300))
        return rank, local, world, dist
    if torch.cuda.is_available():
        torch.cuda.set_device(0)
    return 0, 0, 1, None


def expert_bytes(cfg):
    return 3 * cfg.f * cfg.d // 2 + 3 * cfg.f * cfg.d // 32


# --------------------------------------------------------------------- reference arm
def cpu_reference_sample(cfg, inp_dev, idx, w, n_experts: Optional[int], kind: str = "ref"):
    """Time the reference CPU path (fwd + bwd sweep) over the layer's active experts, or over a
    seeded sample of n_experts of them with all their routed tokens; returns (seconds, fraction
    of the layer's active experts covered, threads)."""
    from oracle import moe_oracle as O
    nthreads = os.cpu_count() or 1
    torch.set_num_threads(nthreads)
    os.environ.setdefault("OMP_NUM_THREADS", str(nthreads))
    kern = O.MXFP4Checker(kind)
    active = torch.unique(idx[idx >= 0]).tolist()
    if n_experts is None or n_experts >= len(active):
        pick = active
    else:
        g = torch.Generator().manual_seed(123)
        pick = sorted(active[i] for i in torch.randperm(len(active), generator=g)[:n_experts].tolist())
    ev = torch.tensor(pick, device=idx.device)
    cpu = {key: inp_dev[key][ev].cpu() for key in ("w1p", "w1s", "w3p", "w3s", "w2p", "w2s")}
    cpu.update({key: inp_dev[key].float().cpu() for key in ("A_g", "B_g", "A_u", "B_u", "A_d", "B_d")})
    remap = torch.full((cfg.E,), -1, dtype=torch.int64)
    remap[torch.tensor(pick)] = torch.arange(len(pick))
    idx_c = idx.cpu()
    idx_r = torch.where(idx_c >= 0, remap[idx_c.clamp(min=0)], idx_c)
    layer = O.Layer.from_inputs(cpu, cfg.scaling)
    x = inp_dev["x"].float().cpu()
    gr = inp_dev["g"].float().cpu()
    wc = w.cpu()
    experts = list(range(len(pick)))
    t0 = time.perf_counter()
    O.experts_forward(kern, layer, x, idx_r, wc, experts)
    O.experts_backward(kern, layer, x, idx_r, wc, gr, experts)
    dt = time.perf_counter() - t0
    return dt, len(pick) / max(1, len(active)), kern.threads()


def workload_config(cfg, world, U=None):
    """The `config` object both arms print for the same workload."""
    if world == 1:
        wl = (("configs[1]" if cfg.T == 1024 else f"configs[2]'s {cfg.T} tokens on one GPU") +
              f": {cfg.E}-expert MXFP4 MoE layer, route + fwd + full LoRA bwd")
        par = "single GPU"
    else:
        wl = (f"configs[2]: 896-expert MXFP4 MoE layer, {cfg.T * world} tokens, route + fwd + full LoRA bwd, "
              f"expert parallel over {world} GPUs ({cfg.E // world} experts and {cfg.T} tokens each, NCCL "
              f"all-to-all dispatch + combine)")
        par = f"ep{world}"
    c = {"workload": wl, "d": cfg.d, "f": cfg.f, "E": cfg.E, "k": cfg.k, "T_total": cfg.T * world,
         "T_per_gpu": cfg.T, "r": cfg.r, "parallelism": par,
         "l2": "weights >> 126 MB L2: every step streams them from HBM"}
    if U is not None:
        c["active_experts_rank0"] = U
    return c


REF_SAMPLE_EXPERTS_EP = 64     # configs[2] reference steps: experts sampled, all their tokens


def run_reference(args, cfg, rank, world, dist):
    """The reference's CPU path on the box's host cores, on the same workload as our arm (cfg
    is the per-rank config; the workload is its T times world tokens): rank 0 only (the other
    ranks of a torchrun launch exit without work). Each timed step routes every token on the
    CPU (KimiK3MoERouter arithmetic: fp32 logits, torch.topk) and runs the reference expert loop
    forward + backward; warm-up steps run a 16-expert sample (they only warm the code paths)."""
    from dataclasses import replace
    from lazylora_b200.synthetic import make_layer_device
    if rank != 0:
        return
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    if dev == "cpu":
        print(json.dumps({"impl": "reference", "unavailable": "no CUDA device to generate the layer inputs on"}))
        return
    total = replace(cfg, T=cfg.T * world)
    inp = make_layer_device(total, device=dev)
    from oracle import moe_oracle as O
    kind = "ref" if os.path.exists(O.REF_SO) else "oracle"
    x_cpu, wr, br = inp["x"].float().cpu(), inp["router_w"].cpu(), inp["router_b"].cpu()
    sample = None if world == 1 else REF_SAMPLE_EXPERTS_EP
    times = []
    threads = os.cpu_count() or 1
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        idx, w = O.route(x_cpu, wr, br, total.k)
        t_route = time.perf_counter() - t0
        dt, frac, threads = cpu_reference_sample(total, inp, idx.to(dev), w.to(dev),
                                                 16 if i < args.warmup else sample, kind)
        if i >= args.warmup:
            times.append(t_route + dt / frac)            # seconds for the whole layer
    step_s = statistics.median(times)
    value = total.T / step_s
    if sample is None:
        desc = ("the whole layer each step: CPU router over all tokens, then the reference expert loop "
                "fwd+bwd over every active expert")
    else:
        desc = (f"CPU router over all {total.T} tokens, then the reference expert loop fwd+bwd over {sample} of "
                f"the active experts with all their routed tokens, scaled by active/{sample}")
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": step_s * 1e3, "higher_is_better": True,
            "scaling": "weak" if world == 1 else "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": workload_config(cfg, world), "impl": "reference",
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads,
                             "kind": "reference" if kind == "ref" else "port", "sample": desc},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------- our arm
def run_ours(args, cfg, rank, local, world, dist):
    from lazylora_b200 import _lib as L
    from lazylora_b200.core.moe_router import KimiK3MoERouter
    from lazylora_b200.synthetic import make_layer_device
    from lazylora_b200.trainer.routed_experts import RoutedExpertsLayer
    from lazylora_b200.trainer.host_pipeline import HostStepPipeline

    dev = torch.device("cuda", local)
    lib = L.load()
    ep = None
    single_ms = None
    if world > 1:
        # the same total workload on one GPU, timed by rank 0 in this job (the denominator of
        # strong_efficiency); the other ranks wait at the barrier
        if rank == 0:
            single_ms = time_single_gpu(args, cfg, world, dev)
        dist.barrier()
        # expert parallel: this rank's block of experts and its own cfg.T tokens
        from lazylora_b200.synthetic import make_ep_rank_device
        from lazylora_b200.trainer.expert_parallel import ExpertParallelLayer
        inp = make_ep_rank_device(cfg, rank, world, device=dev)
        layer = RoutedExpertsLayer.from_inputs(inp, cfg.scaling, device=dev)
        ep = ExpertParallelLayer(layer, cfg.E)
    else:
        inp = make_layer_device(cfg, device=dev)
        layer = RoutedExpertsLayer.from_inputs(inp, cfg.scaling, device=dev)
    router = KimiK3MoERouter(hidden_size=cfg.d, num_experts=cfg.E, top_k=cfg.k, device=dev)
    x = inp["x"].to(torch.bfloat16).contiguous()
    g = inp["g"].to(torch.bfloat16).contiguous()
    Wr, br = inp["router_w"], inp["router_b"]
    del inp["w1p"], inp["w3p"], inp["w2p"]   # the layer holds the weights

    launches = [0]

    def step(xx, gg):
        idx, w = router.forward(xx, weight=Wr, bias=br)
        n = lib.ll_last_launch_count()          # router kernels
        if ep is not None:
            l0 = ep.ops.launches
            out = ep.forward(xx, idx, w)
            gh, gw, grads = ep.backward(gg)
            n += ep.ops.launches - l0 + ep.local_launches
        else:
            out = layer.forward(xx, idx, w)
            n += lib.ll_last_launch_count()
            gh, gw, grads = layer.backward(xx, idx, w, gg)
            n += lib.ll_last_launch_count()
        launches[0] += n
        return out, gh, gw, grads, idx, w

    # ---- warm-up + correctness status
    ClockSampler.start(local)
    for _ in range(args.warmup):
        res = step(x, g)
    if ep is not None:
        if ep._ctx["R"]:
            layer.check_status(ep._ctx["R"], cfg.k)
        local_idx = ep._ctx["idx_recv"]
        U = int(torch.unique(local_idx[local_idx >= 0]).numel())
    else:
        layer.check_status(cfg.T, cfg.k)
        U = int(torch.unique(res[4]).numel())
    idx = res[4]
    torch.cuda.synchronize()

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    # ---- timed region (device time), with per-GEMM events for the roofline
    stream = torch.cuda.current_stream()
    n_gemm_ev = 8
    gemm_events = [[torch.cuda.Event(enable_timing=True) for _ in range(n_gemm_ev)] for _ in range(args.steps)]
    for evs in gemm_events:          # torch creates the CUDA event on first record
        for e in evs:
            e.record(stream)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches[0] = 0
    barrier()
    with ClockSampler(local) as clk:
        start.record(stream)
        for i in range(args.steps):
            ev = gemm_events[i]
            arr = (L.c_void_p * n_gemm_ev)(*[e.cuda_event for e in ev])
            lib.ll_profile_gemm_events(arr, n_gemm_ev)
            step(x, g)
        end.record(stream)
        barrier()
    lib.ll_profile_gemm_events(None, 0)
    if ep is None:
        layer.check_status(cfg.T, cfg.k)
    elif ep._ctx["R"]:
        layer.check_status(ep._ctx["R"], cfg.k)
    total_ms = start.elapsed_time(end)
    gemm_ms = [[gemm_events[i][2 * j].elapsed_time(gemm_events[i][2 * j + 1]) for j in range(4)]
               for i in range(args.steps)]
    clocks = clk.summary()

    # ---- per-kernel breakdown (untimed pass): an event after every launch of the library
    breakdown = {}
    nb_steps = min(args.steps, 5)
    for _ in range(nb_steps):
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(128)]
        for e in evs:
            e.record(stream)
        t0 = torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        lib.ll_profile_launch_events((L.c_void_p * 128)(*[e.cuda_event for e in evs]), 128)
        step(x, g)
        nrec = lib.ll_profile_launch_recorded()
        names_rec = [lib.ll_profile_launch_name(i).decode() for i in range(nrec)]
        lib.ll_profile_launch_events(None, 0)
        torch.cuda.synchronize()
        prev = t0
        for i, nm in enumerate(names_rec):
            breakdown[nm] = breakdown.get(nm, 0.0) + prev.elapsed_time(evs[i]) * 1e3 / nb_steps
            prev = evs[i]

    # ---- all-to-all time per exchange (untimed pass, CUDA events around each collective)
    a2a = None
    if ep is not None:
        ep.profile = []
        step(x, g)
        torch.cuda.synchronize()
        prof, ep.profile = ep.profile, None
        names = [nm for nm, _, _ in prof]
        ms = torch.tensor([e[0].elapsed_time(e[1]) for _, _, e in prof], device=dev, dtype=torch.float64)
        byts = torch.tensor([b for _, b, _ in prof], device=dev, dtype=torch.float64)
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        dist.all_reduce(byts, op=dist.ReduceOp.MAX)
        a2a = {"source": "CUDA events around each collective in one untimed step, max over ranks",
               "total_ms": round(float(ms.sum()), 4),
               **{nm: {"ms": round(float(m), 4), "bytes_sent_max_rank": int(b)}
                  for nm, m, b in zip(names, ms.tolist(), byts.tolist())}}

    # ---- end to end through the public API, host buffers, copies inside the timed region
    x_h = x.cpu().pin_memory()
    g_h = g.cpu().pin_memory()
    out_h = torch.empty((cfg.T, cfg.d), dtype=torch.float32).pin_memory()
    gh_h = torch.empty((cfg.T, cfg.d), dtype=torch.float32).pin_memory()
    gw_h = torch.empty((cfg.T, cfg.k), dtype=torch.float32).pin_memory()
    e_steps = max(1, min(args.steps, 10))
    # the library's host pipeline: step i + 1's inputs are copied in, and step i's results out,
    # on copy streams while the SMs compute; every copy lies inside the timed region
    pipe = HostStepPipeline(step, out_index=[0, 1, 2], device=dev)
    pipe.run([x_h] * 2, [g_h] * 2, [(out_h, gh_h, gw_h)] * 2)      # warm-up of the streams
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    pipe.run([x_h] * e_steps, [g_h] * e_steps, [(out_h, gh_h, gw_h)] * e_steps)
    e1.record(stream)
    barrier()
    e2e_ms = e0.elapsed_time(e1) / e_steps
    h2d = x_h.numel() * 2 + g_h.numel() * 2
    d2h = (out_h.numel() + gh_h.numel() + gw_h.numel()) * 4

    # ---- max over ranks
    ms_step = total_ms / args.steps
    vals = torch.tensor([ms_step, e2e_ms], device=dev, dtype=torch.float64)
    if dist is not None:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    ms_step, e2e_ms = float(vals[0]), float(vals[1])
    if rank != 0:
        return

    hbm_peak, tf_peak, peak_kind = _peaks()
    eb = expert_bytes(cfg)
    names = ["F1 gate/up (W1,W3 . x)", "F2 down (W2 . h)", "B1 (g . W2)", "B2 dX (dg . W1 + du . W3)"]
    per_kernel_bytes = [U * 2 * cfg.f * cfg.d * 17 // 32, U * cfg.f * cfg.d * 17 // 32,
                        U * cfg.f * cfg.d * 17 // 32, U * 2 * cfg.f * cfg.d * 17 // 32]
    traffic_pe = NCU_DRAM_BYTES_PER_EXPERT.get((cfg.d, cfg.f))
    avg_ms = [statistics.mean(s[j] for s in gemm_ms) for j in range(4)]
    shares = [a / ms_step for a in avg_ms]
    dom = max(range(4), key=lambda j: avg_ms[j])
    achieved = per_kernel_bytes[dom] / (avg_ms[dom] * 1e-3) / 1e9
    weight_tbs = 2 * U * eb / (ms_step * 1e-3) / 1e12
    value = world * cfg.T / (ms_step * 1e-3)

    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "weak" if world == 1 else "strong",
        "vs_baseline": None, "dtype": "fp16 operands / fp32 accumulate (MXFP4 weights decoded exactly)",
        "data": "synthetic",
        "config": workload_config(cfg, world, U) if args.config in ("c1", "c2") else
        {**workload_config(cfg, world, U), "workload": f"{args.config}: {cfg.E}-expert MXFP4 MoE layer, "
                                                       f"route + fwd + full LoRA bwd"},
        "weight_TBps": weight_tbs,
        "hbm_roofline_ms": 2 * U * eb / (hbm_peak * 1e9) * 1e3,
        "roofline": {"bound": "hbm", "kernel": names[dom], "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                     "frac": achieved / hbm_peak, "peak_kind": peak_kind,
                     "traffic": None if traffic_pe is None else round(U * traffic_pe[dom]),
                     "traffic_source": None if traffic_pe is None else
                     "ncu dram__bytes_read.sum + dram__bytes_write.sum of the same kernel at d=7168, f=2048, "
                     "64 experts x 9 tokens, per touched expert, times the experts this launch touches",
                     "algorithmic_bytes_per_launch": per_kernel_bytes[dom], "avg_launch_ms": avg_ms[dom]},
        "kernel_ms": {n: round(a, 4) for n, a in zip(names, avg_ms)},
        "kernel_share": {n: round(s, 4) for n, s in zip(names, shares)},
        "kernel_breakdown_us": {"source": f"CUDA events after every launch of the library, mean of {nb_steps} "
                                          "untimed steps (includes the launch gaps on the stream)",
                                **{k: round(v, 1) for k, v in sorted(breakdown.items(), key=lambda kv: -kv[1])}},
        "e2e": {"value": world * cfg.T / (e2e_ms * 1e-3), "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "steps": e_steps,
                "api": "lazylora_b200.trainer.host_pipeline.HostStepPipeline over router + layer fwd + bwd: "
                       "pinned host x, g in; out, grad_h, grad_w back to pinned host; copies on copy streams "
                       "overlapped with the neighbouring steps' compute, all inside the timed region"},
        "gpu_launches": launches[0],
        "clocks": clocks,
    }
    if world > 1:
        line["layer_ms_max_over_ranks"] = ms_step
        line["single_gpu_same_workload_ms"] = single_ms
        line["strong_efficiency"] = single_ms / (world * ms_step) if single_ms else None
        line["all_to_all"] = a2a
    if args.cpu_baseline and world == 1:
        weights = {"w1p": layer.w1p, "w3p": layer.w3p, "w2p": layer.w2p, "w1s": layer.w1s[..., :cfg.d // 32],
                   "w3s": layer.w3s[..., :cfg.d // 32], "w2s": layer.w2s[..., :cfg.f // 32]}
        dt, frac, threads = cpu_reference_sample(cfg, {**inp, **weights}, idx, res[5], None)
        line["cpu_baseline"] = {"value": cfg.T / dt, "unit": UNIT, "cores": threads, "kind": "reference",
                                "sample": f"one whole-layer step: the reference C kernel (oracle/_ref) driven by the "
                                          f"restated expert loop, fwd+bwd over all {U} active experts with the GPU "
                                          f"step's routing"}
    print(json.dumps(line), flush=True)


def time_single_gpu(args, cfg, world, dev):
    """ms per step of the N-rank run's whole workload (world * cfg.T tokens, all experts) on this
    GPU alone: route + forward + full backward, CUDA events, after warm-up. Frees its memory."""
    from dataclasses import replace
    from lazylora_b200.core.moe_router import KimiK3MoERouter
    from lazylora_b200.synthetic import make_layer_device
    from lazylora_b200.trainer.routed_experts import RoutedExpertsLayer
    total = replace(cfg, T=cfg.T * world)
    inp = make_layer_device(total, device=dev)
    layer = RoutedExpertsLayer.from_inputs(inp, total.scaling, device=dev)
    router = KimiK3MoERouter(hidden_size=total.d, num_experts=total.E, top_k=total.k, device=dev)
    x = inp["x"].to(torch.bfloat16).contiguous()
    g = inp["g"].to(torch.bfloat16).contiguous()
    Wr, br = inp["router_w"], inp["router_b"]
    del inp

    def step():
        idx, w = router.forward(x, weight=Wr, bias=br)
        layer.forward(x, idx, w)
        layer.backward(x, idx, w, g)

    for _ in range(max(3, args.warmup)):
        step()
    layer.check_status(total.T, total.k)
    stream = torch.cuda.current_stream()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n = max(3, min(args.steps, 10))
    torch.cuda.synchronize()
    a.record(stream)
    for _ in range(n):
        step()
    b.record(stream)
    torch.cuda.synchronize()
    layer.check_status(total.T, total.k)
    ms = a.elapsed_time(b) / n
    del layer, router, x, g
    torch.cuda.empty_cache()
    return ms


# ----------------------------------------------------------------------- decode
def run_decode(args, cfg, rank, local, world, dist):
    ClockSampler.start(local)
    """Forward-only decode steps (router + routed experts) at T in {1, 4, 16} with Zipf-skewed
    routing. The HBM bound is the MXFP4 bytes of the U experts the step touches; L2 is flushed
    before every timed step (a 256 MB write, then a 256 MB read of another buffer so that the
    write's dirty lines are written back before the step starts, not during it), so those bytes
    come from HBM. Each step is timed
    by its own CUDA events; --graph replays the step as one CUDA graph."""
    from lazylora_b200 import _lib as L
    from lazylora_b200.core.moe_router import KimiK3MoERouter
    from lazylora_b200.synthetic import make_layer_device
    from lazylora_b200.trainer.routed_experts import RoutedExpertsLayer
    dev = torch.device("cuda", local)
    lib = L.load()
    inp = make_layer_device(cfg, device=dev, with_grad=False)
    layer = RoutedExpertsLayer.from_inputs(inp, cfg.scaling, device=dev, prepare_backward=False)
    router = KimiK3MoERouter(hidden_size=cfg.d, num_experts=cfg.E, top_k=cfg.k, device=dev)
    x = inp["x"].to(torch.bfloat16).contiguous()
    Wr, br = inp["router_w"], inp["router_b"]
    zipf_fit = {"method": "scalar: bias = gamma ln(p / p_max)", "gamma": cfg.zipf_gamma}
    if cfg.zipf_s is not None and args.zipf_fit == "expert":
        # a per-expert bias fit to the Zipf target on seeded tokens (the scalar fit reaches L1
        # 0.81 only; frequencies above 1/k are out of reach for any bias)
        from lazylora_b200.synthetic import fit_zipf_bias, zipf_target
        p_t = zipf_target(cfg.E, cfg.zipf_s, torch.Generator().manual_seed(cfg.seed + 1))
        br, l1 = fit_zipf_bias(Wr, p_t, cfg.k)
        zipf_fit = {"method": "per-expert bias, 1000 damped steps of bias += 0.01 (ln p - ln f) on 65,536 "
                              "seeded tokens", "L1": round(l1, 4),
                    "L1_floor": round(2 * float((p_t - 1.0 / cfg.k).clamp(min=0).sum()), 4)}
    del inp["w1p"], inp["w3p"], inp["w2p"]
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    flush_rd = torch.ones(64 << 20, dtype=torch.float32, device=dev)

    def flush_l2():
        flush.fill_(1)
        flush_rd.sum()
    stream = torch.cuda.current_stream()
    state = {}

    def step():
        idx, w = router.forward(x, weight=Wr, bias=br)
        n = lib.ll_last_launch_count()
        state["idx"] = idx
        state["out"] = layer.forward(x, idx, w)
        state["n"] = n + lib.ll_last_launch_count()

    for _ in range(args.warmup):
        step()
    layer.check_status(cfg.T, cfg.k)
    # per-kernel breakdown (untimed, L2 flushed first): an event after every launch of the library.
    # With --graph the step is captured once more with those events as event-record nodes and
    # replayed, so the times are those of kernels inside a graph (each event node adds a little);
    # otherwise the launches are eager. Reported per kernel: the time from the latest earlier
    # event that had completed to this one's, and the timeline of completion times.
    breakdown, timeline = {}, []
    nb = 5
    evs = [torch.cuda.Event(enable_timing=True, external=bool(args.graph)) for _ in range(64)]
    t0 = torch.cuda.Event(enable_timing=True, external=bool(args.graph))
    for e in evs + [t0]:
        e.record(stream)
    torch.cuda.synchronize()
    names_rec, ends = [], None
    if args.graph:
        pg = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream()
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            step()
            with torch.cuda.graph(pg, stream=side):
                t0.record(side)
                lib.ll_profile_launch_events((L.c_void_p * 64)(*[e.cuda_event for e in evs]), 64)
                step()
                nrec = lib.ll_profile_launch_recorded()
                names_rec = [lib.ll_profile_launch_name(i).decode() for i in range(nrec)]
                lib.ll_profile_launch_events(None, 0)
        stream.wait_stream(side)
    for _ in range(nb):
        flush_l2()
        if args.graph:
            pg.replay()
        else:
            t0.record(stream)
            lib.ll_profile_launch_events((L.c_void_p * 64)(*[e.cuda_event for e in evs]), 64)
            step()
            nrec = lib.ll_profile_launch_recorded()
            names_rec = [lib.ll_profile_launch_name(i).decode() for i in range(nrec)]
            lib.ll_profile_launch_events(None, 0)
        torch.cuda.synchronize()
        e_us = [t0.elapsed_time(evs[i]) * 1e3 for i in range(len(names_rec))]
        ends = e_us if ends is None else [a + b for a, b in zip(ends, e_us)]
    ends = [v / nb for v in ends]
    for i, nm in enumerate(names_rec):
        before = [v for v in ends[:i] if v <= ends[i]]
        breakdown[nm] = breakdown.get(nm, 0.0) + ends[i] - (max(before) if before else 0.0)
        timeline.append([nm, round(ends[i], 1)])
    if args.graph:
        del pg
    run = step
    if args.graph:
        gr = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream()
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            step()                                  # allocations happen outside the capture
            with torch.cuda.graph(gr, stream=side):
                step()
        stream.wait_stream(side)
        run = gr.replay
    torch.cuda.synchronize()
    times, us = [], []
    with ClockSampler(local) as clk:
        for _ in range(args.steps):
            flush_l2()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            run()
            b.record(stream)
            times.append((a, b))
        torch.cuda.synchronize()
    layer.check_status(cfg.T, cfg.k)
    us = sorted(a.elapsed_time(b) * 1e3 for a, b in times)
    med = statistics.median(us)
    U = int(torch.unique(state["idx"]).numel())
    wbytes = U * expert_bytes(cfg)
    hbm_peak, _, peak_kind = _peaks()
    gbs = wbytes / (med * 1e-6) / 1e9
    line = {"metric": f"decode forward weight GB/s (T={cfg.T}, Zipf s={cfg.zipf_s} routing)", "value": gbs,
            "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "us_per_step": med,
            "us_min": us[0], "higher_is_better": True, "dtype": "fp16 operands / fp32 accumulate", "data": "synthetic",
            "config": {"workload": f"configs[3]: decode T={cfg.T}, router + routed experts forward",
                       "d": cfg.d, "f": cfg.f, "E": cfg.E, "k": cfg.k, "T": cfg.T, "r": cfg.r,
                       "zipf_s": cfg.zipf_s, "zipf_fit": zipf_fit, "active_experts": U,
                       "graph": bool(args.graph),
                       "l2": "256 MB written, then another 256 MB read, before every timed step"},
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm_peak, "unit": "GB/s", "frac": gbs / hbm_peak,
                         "peak_kind": peak_kind, "algorithmic_bytes_per_step": wbytes,
                         "roofline_us": wbytes / (hbm_peak * 1e9) * 1e6},
            "gpu_launches": state["n"] * args.steps, "clocks": clk.summary(),
            "kernel_breakdown_us": {"source": f"CUDA events after every launch of the library "
                                              f"({'event nodes in a replayed graph' if args.graph else 'eager launches'}"
                                              f"), L2 flushed before each step, mean of {nb} untimed steps; per "
                                              f"kernel: from the latest earlier completion",
                                    **{k: round(v, 1) for k, v in sorted(breakdown.items(), key=lambda kv: -kv[1])}},
            "kernel_timeline_us": timeline}
    print(json.dumps(line), flush=True)


# ------------------------------------------- real routing (recorded K3 traces, top-16)
def run_traces(args, cfg, rank, local, world, dist):
    """fwd + bwd of the configs[1]-width layer (E = 896) with the twenty real top-16 routings
    of tests/golden/routing_traces.npz (Kimi K3 on five prompts, four layers each, 111..264
    tokens): prefill-sized steps with real expert concentration instead of synthetic routing.
    HBM bound per step: twice the MXFP4 bytes of the experts that routing touches."""
    ClockSampler.start(local)
    import numpy as np
    from dataclasses import replace
    from lazylora_b200.synthetic import make_layer_device
    from lazylora_b200.trainer.routed_experts import RoutedExpertsLayer
    z = np.load(os.path.join(ROOT, "tests", "golden", "routing_traces.npz"))
    keys = sorted({k.rsplit("/", 1)[0] for k in z.files})
    dev = torch.device("cuda", local)
    nmax = max(z[k + "/idx"].shape[0] for k in keys)
    kk = z[keys[0] + "/idx"].shape[1]
    cfg = replace(cfg, k=kk, T=nmax)
    inp = make_layer_device(cfg, device=dev)
    layer = RoutedExpertsLayer.from_inputs(inp, cfg.scaling, device=dev)
    del inp["w1p"], inp["w3p"], inp["w2p"]
    x_all = inp["x"].to(torch.bfloat16)
    g_all = inp["g"].to(torch.bfloat16)
    cases = []
    for k_ in keys:
        idx = torch.from_numpy(z[k_ + "/idx"].astype(np.int64)).to(dev)
        w = torch.from_numpy(z[k_ + "/w"].astype(np.float32)).to(dev)
        cases.append((k_, idx, w, x_all[:idx.shape[0]].contiguous(), g_all[:idx.shape[0]].contiguous()))
    stream = torch.cuda.current_stream()

    def step(c):
        _, idx, w, x, g = c
        layer.forward(x, idx, w)
        layer.backward(x, idx, w, g)

    for _ in range(args.warmup):
        for c in cases:
            step(c)
    torch.cuda.synchronize()
    hbm_peak, _, peak_kind = _peaks()
    per, tot_ms, tot_tok, tot_bytes = {}, 0.0, 0, 0
    with ClockSampler(local) as clk:
        for c in cases:
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            for _ in range(args.steps):
                step(c)
            b.record(stream)
            torch.cuda.synchronize()
            ms = a.elapsed_time(b) / args.steps
            U = int(torch.unique(c[1]).numel())
            byts = 2 * U * expert_bytes(cfg)
            per[c[0]] = {"tokens": int(c[1].shape[0]), "experts_touched": U, "ms": round(ms, 3),
                         "hbm_frac": round(byts / (ms * 1e-3) / 1e9 / hbm_peak, 3)}
            tot_ms += ms
            tot_tok += int(c[1].shape[0])
            tot_bytes += byts
    layer.check_status(nmax, kk)
    line = {"metric": "MoE-layer fwd+bwd tokens/s on real routing (Kimi K3 traces, top-16 of 896)",
            "value": tot_tok / (tot_ms * 1e-3), "unit": UNIT, "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": tot_ms / len(cases), "higher_is_better": True,
            "dtype": "fp16 operands / fp32 accumulate (MXFP4 weights decoded exactly)",
            "data": "synthetic weights and activations; routing recorded from the reference's K3 runs",
            "config": {"workload": "20 recorded routings (5 prompts x 4 layers), one fwd+bwd step each",
                       "d": cfg.d, "f": cfg.f, "E": cfg.E, "k": kk, "r": cfg.r},
            "roofline": {"bound": "hbm", "achieved": tot_bytes / (tot_ms * 1e-3) / 1e9, "peak": hbm_peak,
                         "unit": "GB/s", "frac": tot_bytes / (tot_ms * 1e-3) / 1e9 / hbm_peak,
                         "peak_kind": peak_kind},
            "per_routing": per, "clocks": clk.summary()}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------- shared expert (Kimi K3 shape)
def run_shared(args, cfg, rank, local, world, dist):
    """fwd + bwd of the shared expert (dense SiTU-GLU 7168 -> 6144 -> 7168 with LoRA on its
    three projections) at T = cfg.T tokens. Tensor-bound: the three bf16 projections forward and
    the three input-gradient GEMMs backward (the base weights are frozen)."""
    ClockSampler.start(local)
    from lazylora_b200.trainer.shared_expert import SharedExpert
    dev = torch.device("cuda", local)
    d, F, r, N = args.shared_hidden, args.shared_inter, cfg.r, cfg.T
    gen = torch.Generator(device=dev).manual_seed(cfg.seed + 11)
    W = lambda o, i: (torch.randn(o, i, generator=gen, device=dev) / i ** 0.5).to(torch.bfloat16)
    rnd = lambda *sh: torch.randn(*sh, generator=gen, device=dev) * 0.05
    se = SharedExpert(W(F, d), W(F, d), W(d, F), rnd(r, d), rnd(F, r), rnd(r, d), rnd(F, r), rnd(r, F), rnd(d, r),
                      cfg.scaling)
    x = torch.randn(N, d, generator=gen, device=dev).to(torch.bfloat16)
    g = torch.randn(N, d, generator=gen, device=dev).to(torch.bfloat16)
    stream = torch.cuda.current_stream()

    def step():
        se.forward(x)
        se.backward(g)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        a.record(stream)
        for _ in range(args.steps):
            step()
        b.record(stream)
        torch.cuda.synchronize()
    ms = a.elapsed_time(b) / args.steps
    flops = 2 * 3 * 2 * N * d * F
    _, tf_peak, peak_kind = _peaks()
    tfs = flops / (ms * 1e-3) / 1e12
    # the projections alone, on this library's tcgen05 GEMM and, for context, on cuBLAS
    from lazylora_b200.core import dense

    def timed(fn, n=20):
        for _ in range(3):
            fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(n):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / n
    h_ = torch.randn(N, F, generator=gen, device=dev).to(torch.bfloat16)
    gemms = {
        "gate+up x.W^T (2 outputs)": (lambda: dense.linear_two(x, se.W_g, se.W_u), 2 * 2 * N * d * F),
        "down h.W_d^T": (lambda: dense.linear(h_, se.W_d), 2 * N * d * F),
        "dh = g.W_d": (lambda: dense.matmul(g, se.W_d), 2 * N * d * F),
        "dx = dG.W_g + dU.W_u": (lambda: dense.matmul_sum2(h_, se.W_g, h_, se.W_u), 2 * 2 * N * d * F),
        "cuBLAS gate+up (torch.matmul)": (lambda: (torch.matmul(x, se.W_g.t()), torch.matmul(x, se.W_u.t())),
                                          2 * 2 * N * d * F),
        "cuBLAS dx (torch.matmul + addmm_)": (lambda: torch.matmul(h_, se.W_g).addmm_(h_, se.W_u),
                                              2 * 2 * N * d * F),
    }
    gemm_rep = {}
    for name, (fn, fl) in gemms.items():
        gms = timed(fn)
        gemm_rep[name] = {"ms": round(gms, 4), "tflops": round(fl / (gms * 1e-3) / 1e12, 1)}
    dense.check_status()
    line = {"metric": f"shared expert fwd+bwd tokens/s (d={d}, F={F}, LoRA r={r})", "value": N / (ms * 1e-3),
            "unit": UNIT, "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16 operands / fp32 accumulate", "data": "synthetic",
            "config": {"workload": "shared expert of the K3 MoE layer: 3 bf16 projections + LoRA, forward and "
                                   "input-gradient backward", "d": d, "F": F, "r": r, "T": N},
            "roofline": {"bound": "tensor", "achieved": tfs, "peak": tf_peak, "unit": "TFLOP/s",
                         "frac": tfs / tf_peak, "peak_kind": peak_kind, "flops_per_step": flops},
            "projections": {"source": "CUDA events around 20 calls of each, inputs resident", **gemm_rep},
            "clocks": clk.summary()}
    print(json.dumps(line), flush=True)


# ------------------------------------------------ latent routed block (Kimi K3 shape)
def run_latent(args, cfg, rank, local, world, dist):
    """Route + forward + backward of the latent routed block: down-projection 7168 -> d_l
    (cfg.d), the routed experts at width d_l, RMSNorm of their fp32 sum, up-projection back
    (lazy_trainer.py:722-735). HBM bound: twice the touched experts' MXFP4 bytes plus the two
    projections' bf16 weights read in the forward and again in the backward."""
    ClockSampler.start(local)
    from lazylora_b200 import _lib as L
    from lazylora_b200.core.moe_router import KimiK3MoERouter
    from lazylora_b200.synthetic import make_layer_device
    from lazylora_b200.trainer.latent_moe import LatentRoutedMoE
    from lazylora_b200.trainer.routed_experts import RoutedExpertsLayer
    d_h = args.latent_hidden
    dev = torch.device("cuda", local)
    lib = L.load()
    inp = make_layer_device(cfg, device=dev)
    layer = RoutedExpertsLayer.from_inputs(inp, cfg.scaling, device=dev)
    del inp["w1p"], inp["w3p"], inp["w2p"]
    gen = torch.Generator(device=dev).manual_seed(cfg.seed + 7)
    down_w = (torch.randn(cfg.d, d_h, generator=gen, device=dev) / d_h ** 0.5).to(torch.bfloat16)
    up_w = (torch.randn(d_h, cfg.d, generator=gen, device=dev) / cfg.d ** 0.5).to(torch.bfloat16)
    norm_w = torch.ones(cfg.d, device=dev)
    blk = LatentRoutedMoE(layer, down_w, up_w, norm_w)
    router = KimiK3MoERouter(hidden_size=d_h, num_experts=cfg.E, top_k=cfg.k, device=dev)
    Wr = torch.randn(cfg.E, d_h, generator=gen, device=dev) * 0.02
    br = torch.zeros(cfg.E, device=dev)
    x = torch.randn(cfg.T, d_h, generator=gen, device=dev).to(torch.bfloat16)
    g = torch.randn(cfg.T, d_h, generator=gen, device=dev).to(torch.bfloat16)
    stream = torch.cuda.current_stream()
    state = {}

    def step(xx, gg):
        idx, w = router.forward(xx, weight=Wr, bias=br)
        out = blk.forward(xx, idx, w)
        gx, gw, grads = blk.backward(gg)
        state["idx"] = idx
        return out, gx, gw, grads

    for _ in range(args.warmup):
        step(x, g)
    layer.check_status(cfg.T, cfg.k)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        a.record(stream)
        for _ in range(args.steps):
            step(x, g)
        b.record(stream)
        torch.cuda.synchronize()
    layer.check_status(cfg.T, cfg.k)
    ms = a.elapsed_time(b) / args.steps
    U = int(torch.unique(state["idx"]).numel())
    proj_bytes = 2 * cfg.d * d_h * 2
    wbytes = 2 * U * expert_bytes(cfg) + 2 * proj_bytes
    hbm_peak, _, peak_kind = _peaks()
    roof_ms = wbytes / (hbm_peak * 1e9) * 1e3
    line = {"metric": f"latent MoE block fwd+bwd tokens/s (d_h={d_h}, d_l={cfg.d}, f={cfg.f}, E={cfg.E}, "
                      f"top-{cfg.k}, LoRA r={cfg.r})",
            "value": cfg.T / (ms * 1e-3), "unit": UNIT, "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16 projections / fp16 expert operands, fp32 accumulate", "data": "synthetic",
            "config": {"workload": "latent routed block of the K3 MoE layer: route + down-proj + experts + RMSNorm + "
                                   "up-proj, forward and backward", "d_h": d_h, "d_l": cfg.d, "f": cfg.f,
                       "E": cfg.E, "k": cfg.k, "T": cfg.T, "r": cfg.r, "active_experts": U},
            "roofline": {"bound": "hbm", "achieved": wbytes / (ms * 1e-3) / 1e9, "peak": hbm_peak, "unit": "GB/s",
                         "frac": roof_ms / ms, "peak_kind": peak_kind, "algorithmic_bytes_per_step": wbytes,
                         "roofline_ms": roof_ms},
            "clocks": clk.summary()}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------ streaming
def run_stream_ep(args, cfg, rank, local, world, dist):
    """configs[4] expert-parallel over `world` GPUs: each rank holds only its block of every
    layer's experts in pinned host memory (1/world of the layer) and streams it into HBM for
    every use, inside ExpertParallelLayer (StreamedLocalExperts as the local layer); each rank
    routes its own cfg.T tokens (weak scaling). An 8-layer fwd + bwd a step; the step time is
    the max over ranks."""
    ClockSampler.start(local)
    from lazylora_b200.core.moe_router import KimiK3MoERouter
    from lazylora_b200.synthetic import make_layer_device
    from lazylora_b200.trainer.expert_parallel import ExpertParallelLayer, experts_of_rank
    from lazylora_b200.trainer.expert_streamer import ExpertStreamer, HostExpertStore, StreamedLocalExperts
    dev = torch.device("cuda", local)
    n_layers, D = 8, max(1, args.stream_distinct)
    first, count = experts_of_rank(cfg.E, world, rank)
    store = HostExpertStore()
    inp = None
    for l in range(D):
        inp = make_layer_device(cfg if l == 0 else cfg.__class__(**{**cfg.__dict__, "seed": cfg.seed + 100 * l}),
                                device=dev)
        store.add_layer(l, {n: inp[n][first:first + count] for n in ("w1p", "w1s", "w3p", "w3s", "w2p", "w2s")})
        if l + 1 < D:
            del inp
            torch.cuda.empty_cache()
    lora = {n: inp[n] for n in ("A_g", "B_g", "A_u", "B_u", "A_d", "B_d")}
    gen = torch.Generator(device=dev).manual_seed(cfg.seed + 1000 + rank)      # this rank's tokens
    x = torch.randn(cfg.T, cfg.d, generator=gen, device=dev).to(torch.bfloat16)
    g = torch.randn(cfg.T, cfg.d, generator=gen, device=dev).to(torch.bfloat16)
    Wr, br = inp["router_w"], inp["router_b"]
    del inp
    torch.cuda.empty_cache()
    router = KimiK3MoERouter(hidden_size=cfg.d, num_experts=cfg.E, top_k=cfg.k, device=dev)
    streamer = ExpertStreamer(store, lora, cfg.scaling, group_experts=min(args.stream_group, count), device=dev)
    local_ids = list(range(count))
    eps = [ExpertParallelLayer(StreamedLocalExperts(streamer, l % D, expert_ids=local_ids), cfg.E)
           for l in range(n_layers)]
    stream = torch.cuda.current_stream()

    def step():
        for l in range(n_layers):
            i, ww = router.forward(x, weight=Wr, bias=br)
            if l + 1 < n_layers:
                streamer.prefetch((l + 1) % D, local_ids)
            eps[l].forward(x, i, ww)
        for l in reversed(range(n_layers)):
            if l > 0:
                streamer.prefetch((l - 1) % D, local_ids)
            eps[l].backward(g)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    dist.barrier()
    b0 = streamer.bytes_copied
    with ClockSampler(local) as clk:
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(args.steps):
            step()
        b.record(stream)
        torch.cuda.synchronize()
    t = torch.tensor([a.elapsed_time(b) / args.steps], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    step_ms = float(t.item())
    bytes_step = (streamer.bytes_copied - b0) / args.steps
    h2d = bytes_step / (step_ms * 1e-3) / 1e9
    dist.barrier()
    if rank != 0:
        return
    line = {"metric": "streamed 8-layer MoE fwd+bwd tokens/s (configs[4], weights in pinned host memory, "
                      "expert parallel)",
            "value": world * cfg.T / (step_ms * 1e-3), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": True, "scaling": "weak",
            "dtype": "fp16 operands / fp32 accumulate", "data": "synthetic",
            "config": {"workload": f"configs[4]: 8 layers, T={cfg.T} per GPU, r={cfg.r}; each of {world} ranks holds "
                                   f"{count} of {cfg.E} experts per layer in pinned host memory and streams them "
                                   "host->HBM for the forward and again for the backward; NCCL all-to-all dispatch "
                                   "+ combine", "d": cfg.d, "f": cfg.f, "E": cfg.E, "k": cfg.k, "T_per_gpu": cfg.T,
                       "r": cfg.r, "experts_per_rank": count, "distinct_pinned_layers": D,
                       "group_experts": streamer.group, "parallelism": f"ep{world}"},
            "h2d_rank0": {"bytes_per_step": bytes_step, "achieved_GBps": h2d, "peak_GBps": args.h2d_peak,
                          "frac": h2d / args.h2d_peak, "peak_kind": "measured pinned cudaMemcpyAsync on this box"},
            "clocks": clk.summary()}
    print(json.dumps(line), flush=True)


def run_stream(args, cfg, rank, local, world, dist):
    ClockSampler.start(local)
    """configs[4]: an 8-layer fwd + bwd whose expert weights live in pinned host memory and
    are streamed into HBM for every use (2 x 8 layer loads a step), group by group on a copy
    stream while the previous group computes. --stream-distinct N keeps N distinct layers
    pinned (the host RAM bound); layer l uses distinct layer l % N, so the bytes moved per
    step are those of 8 layers either way. Reports tokens/s, the achieved host->device GB/s,
    and the share of the compute hidden under the copies."""
    from lazylora_b200.core.moe_router import KimiK3MoERouter
    from lazylora_b200.synthetic import make_layer_device
    from lazylora_b200.trainer.expert_streamer import (ExpertStreamer, HostExpertStore, streamed_backward,
                                                       streamed_forward)
    from lazylora_b200.trainer.routed_experts import RoutedExpertsLayer
    dev = torch.device("cuda", local)
    n_layers, D = 8, max(1, args.stream_distinct)
    store = HostExpertStore()
    inp = None
    for l in range(D):
        inp = make_layer_device(cfg if l == 0 else cfg.__class__(**{**cfg.__dict__, "seed": cfg.seed + 100 * l}),
                                device=dev)
        store.add_layer(l, {n: inp[n] for n in ("w1p", "w1s", "w3p", "w3s", "w2p", "w2s")})
        if l + 1 < D:
            del inp
            torch.cuda.empty_cache()
    lora = {n: inp[n] for n in ("A_g", "B_g", "A_u", "B_u", "A_d", "B_d")}
    x = inp["x"].to(torch.bfloat16).contiguous()
    g = inp["g"].to(torch.bfloat16).contiguous()
    Wr, br = inp["router_w"], inp["router_b"]
    router = KimiK3MoERouter(hidden_size=cfg.d, num_experts=cfg.E, top_k=cfg.k, device=dev)
    stream = torch.cuda.current_stream()

    # compute alone: one layer fwd + bwd with its weights resident
    res = RoutedExpertsLayer(*(inp[n] for n in ("w1p", "w1s", "w3p", "w3s", "w2p", "w2s")), *(lora[n] for n in (
        "A_g", "B_g", "A_u", "B_u", "A_d", "B_d")), cfg.scaling)
    idx, w = router.forward(x, weight=Wr, bias=br)
    for _ in range(2):
        res.forward(x, idx, w); res.backward(x, idx, w, g)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(3):
        res.forward(x, idx, w); res.backward(x, idx, w, g)
    b.record(stream)
    torch.cuda.synchronize()
    compute_layer_ms = a.elapsed_time(b) / 3
    del res, inp
    torch.cuda.empty_cache()

    streamer = ExpertStreamer(store, lora, cfg.scaling, group_experts=args.stream_group, device=dev)

    every = list(range(cfg.E))   # T * k = 16384 slots over 896 experts: every expert is active

    def step():
        saved = []
        for l in range(n_layers):
            i, ww = router.forward(x, weight=Wr, bias=br)
            streamer.prefetch((l + 1) % D if l + 1 < n_layers else (n_layers - 1) % D, every)
            out, ids = streamed_forward(streamer, l % D, x, i, ww, expert_ids=every)
            saved.append((i, ww, ids))
        for l in reversed(range(n_layers)):
            i, ww, ids = saved[l]
            if l > 0:
                streamer.prefetch((l - 1) % D, saved[l - 1][2])
            streamed_backward(streamer, l % D, x, i, ww, g, ids)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    b0 = streamer.bytes_copied
    with ClockSampler(local) as clk:
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(args.steps):
            step()
        b.record(stream)
        torch.cuda.synchronize()
    step_ms = a.elapsed_time(b) / args.steps
    bytes_step = (streamer.bytes_copied - b0) / args.steps
    h2d = bytes_step / (step_ms * 1e-3) / 1e9
    compute_ms = 2 * n_layers * compute_layer_ms / 2       # fwd+bwd of 8 layers (resident-weight time)
    copy_ms = bytes_step / (args.h2d_peak * 1e9) * 1e3
    hidden = max(0.0, min(1.0, (copy_ms + compute_ms - step_ms) / compute_ms)) if compute_ms > 0 else None
    line = {"metric": "streamed 8-layer MoE fwd+bwd tokens/s (configs[4], weights in pinned host memory)",
            "value": cfg.T / (step_ms * 1e-3), "unit": "tokens/s", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": True, "dtype": "fp16 operands / fp32 "
            "accumulate", "data": "synthetic",
            "config": {"workload": "configs[4]: 8 layers, T=2048, r=64, every layer's experts streamed host->HBM "
                                   "for the forward and again for the backward",
                       "d": cfg.d, "f": cfg.f, "E": cfg.E, "k": cfg.k, "T": cfg.T, "r": cfg.r,
                       "distinct_pinned_layers": D, "group_experts": args.stream_group},
            "h2d": {"bytes_per_step": bytes_step, "achieved_GBps": h2d, "peak_GBps": args.h2d_peak,
                    "frac": h2d / args.h2d_peak, "peak_kind": "measured pinned cudaMemcpyAsync on this box"},
            "compute_ms_resident": compute_ms, "copy_ms_at_peak": copy_ms, "compute_hidden_frac": hidden,
            "clocks": clk.summary()}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="c1")
    ap.add_argument("--no-cpu-baseline", dest="cpu_baseline", action="store_false")
    ap.add_argument("--decode", action="store_true", help="forward-only decode steps (configs[3]: c3_t1/4/16)")
    ap.add_argument("--graph", action="store_true", help="with --decode: replay each step as a CUDA graph")
    ap.add_argument("--zipf-gamma", type=float, default=None, help="override the config's Zipf bias scale")
    ap.add_argument("--zipf-fit", default="expert", choices=["expert", "gamma"],
                    help="decode routing skew: a per-expert bias fit (default) or the scalar gamma")
    ap.add_argument("--experts", type=int, default=None,
                    help="override the config's expert count (profiler captures on a smaller weight stack)")
    ap.add_argument("--tokens", type=int, default=None,
                    help="override the config's token count (profiler captures of other tile widths)")
    ap.add_argument("--stream", action="store_true", help="configs[4]: experts streamed from pinned host memory")
    ap.add_argument("--latent", action="store_true", help="the latent routed block (use --config c1_latent)")
    ap.add_argument("--traces", action="store_true", help="fwd+bwd steps on the recorded K3 routings (top-16)")
    ap.add_argument("--shared", action="store_true", help="the shared expert (dense SiTU-GLU with LoRA)")
    ap.add_argument("--shared-hidden", type=int, default=7168)
    ap.add_argument("--shared-inter", type=int, default=6144)
    ap.add_argument("--latent-hidden", type=int, default=7168, help="hidden width around the latent block")
    ap.add_argument("--stream-distinct", type=int, default=1, help="distinct layers kept in pinned host memory")
    ap.add_argument("--stream-group", type=int, default=224, help="experts per streamed group")
    ap.add_argument("--h2d-peak", type=float, default=55.6, help="measured pinned H2D GB/s of the box")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    from dataclasses import replace
    from lazylora_b200.synthetic import CONFIGS
    cfg = CONFIGS[args.config]
    if args.zipf_gamma is not None:
        cfg = replace(cfg, zipf_gamma=args.zipf_gamma)
    if args.experts is not None:
        cfg = replace(cfg, E=args.experts)
    if args.tokens is not None:
        cfg = replace(cfg, T=args.tokens)
    rank, local, world, dist = dist_setup(args)
    if world > 1 and args.config in ("c1", "c2") and not (args.decode or args.stream or args.latent or
                                                          args.traces or args.shared):
        # 8192 tokens in total over the N ranks (strong scaling)
        total = CONFIGS["c2"]
        if total.T % world:
            raise SystemExit(f"--gpus {world} does not divide configs[2]'s {total.T} tokens")
        cfg = replace(total, T=total.T // world)
        args.config = "c2"
    try:
        if args.impl == "reference":
            run_reference(args, cfg, rank, world, dist)   # rank 0 only; no collective
        elif args.decode:
            run_decode(args, cfg, rank, local, world, dist)
        elif args.stream:
            if world > 1:
                run_stream_ep(args, cfg, rank, local, world, dist)
            else:
                run_stream(args, cfg, rank, local, world, dist)
        elif args.latent:
            run_latent(args, cfg, rank, local, world, dist)
        elif args.traces:
            run_traces(args, cfg, rank, local, world, dist)
        elif args.shared:
            run_shared(args, cfg, rank, local, world, dist)
        else:
            run_ours(args, cfg, rank, local, world, dist)
            if dist is not None:
                dist.barrier()
    finally:
        if dist is not None:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
