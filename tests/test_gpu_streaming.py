"""
GPU checks of expert streaming (pinned host memory -> HBM, group by group):

  * the streamed layer against the reference's own outputs (tests/golden/ref_<case>.npz,
    made by LazyLoRATrainer._routed_experts_forward / _backward, whose expert loop is fed by
    DynamicExpertStreamer.stream_experts, lazy_lora/streaming/expert_streamer.py:315-369):
    out, grad_h, grad_w and the six LoRA gradients within relative L2 2e-3, for group sizes
    that split the active set evenly, raggedly and one expert at a time;
  * the streamed layer against the resident layer (the same kernels; only the fp32 order in
    which the groups' partial sums are added differs), including an active set with gaps;
  * the reference-interface generator yields the right bytes; forward-only streaming never
    builds the backward's transposed copy, and backward groups reuse one set of transposed
    buffers per staging slot.
"""
import os

import numpy as np
import pytest
import torch

from lazylora_b200.synthetic import CONFIGS, make_layer
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu


def _setup(case):
    from lazylora_b200.trainer.expert_streamer import ExpertStreamer, HostExpertStore
    from lazylora_b200.trainer.routed_experts import RoutedExpertsLayer
    cfg = CONFIGS[case]
    inp = make_layer(cfg)
    store = HostExpertStore()
    store.add_layer(0, {n: inp[n] for n in ("w1p", "w1s", "w3p", "w3s", "w2p", "w2s")})
    lora = {n: inp[n].cuda() for n in ("A_g", "B_g", "A_u", "B_u", "A_d", "B_d")}
    resident = RoutedExpertsLayer.from_inputs(inp, cfg.scaling)
    x = inp["x"].cuda()
    g = inp["g"].cuda()
    if cfg.x_dtype == "bf16":
        x, g = x.to(torch.bfloat16), g.to(torch.bfloat16)
    idx, w = O.route(inp["x"].float(), inp["router_w"], inp["router_b"], cfg.k)
    return cfg, inp, store, lora, resident, x, g, idx.cuda(), w.cuda(), ExpertStreamer


KEYS = ("out", "grad_h", "grad_w", "dA_g", "dB_g", "dA_u", "dB_u", "dA_d", "dB_d")


@pytest.mark.parametrize("case,group", [("small", 16), ("small", 5), ("small", 1), ("c0", 6), ("k3", 7)])
def test_streamed_layer_matches_reference_goldens(golden_dir, case, group):
    from lazylora_b200.trainer.expert_streamer import streamed_backward, streamed_forward
    fx = np.load(os.path.join(golden_dir, f"ref_{case}.npz"))
    cfg, inp, store, lora, resident, x, g, _idx, _w, ES = _setup(case)
    idx = torch.from_numpy(fx["idx"]).cuda()
    w = torch.from_numpy(fx["w"]).cuda()
    streamer = ES(store, lora, cfg.scaling, group_experts=group)
    out, ids = streamed_forward(streamer, 0, x, idx, w)
    assert all(t is None for t in streamer._tslots), "forward-only streaming built a transposed copy"
    gh, gw, grads = streamed_backward(streamer, 0, x, idx, w, g, ids)
    got = {"out": out, "grad_h": gh, "grad_w": gw, **grads}
    for key in KEYS:
        err = O.rel_l2(got[key].float().cpu(), torch.from_numpy(fx[key]))
        assert err <= 2e-3, f"{case} group {group}: {key} rel-L2 {err:.3e}"
    # later backward passes re-stream into the same two slots and reuse their transposed buffers
    # (the slot rotation continues across passes, so both slots have run a backward after two)
    gh2, _, _ = streamed_backward(streamer, 0, x, idx, w, g, ids)
    assert torch.equal(gh2, gh)
    bufs = [None if t is None else {n: v.data_ptr() for n, v in t.items()} for t in streamer._tslots]
    streamed_backward(streamer, 0, x, idx, w, g, ids)
    assert bufs == [None if t is None else {n: v.data_ptr() for n, v in t.items()} for t in streamer._tslots]


@pytest.mark.parametrize("case,group", [("small", 16), ("small", 5), ("small", 3), ("c0", 6)])
def test_streamed_layer_matches_resident(case, group):
    from lazylora_b200.trainer.expert_streamer import streamed_backward, streamed_forward
    cfg, inp, store, lora, resident, x, g, idx, w, ES = _setup(case)
    streamer = ES(store, lora, cfg.scaling, group_experts=group)
    out, ids = streamed_forward(streamer, 0, x, idx, w)
    gh, gw, grads = streamed_backward(streamer, 0, x, idx, w, g, ids)
    torch.cuda.synchronize()
    want_out = resident.forward(x, idx, w)
    want_gh, want_gw, want_grads = resident.backward(x, idx, w, g)
    assert O.rel_l2(out.cpu(), want_out.cpu()) < 1e-5
    assert O.rel_l2(gh.cpu(), want_gh.cpu()) < 1e-5
    assert O.rel_l2(gw.cpu(), want_gw.cpu()) < 1e-5
    for k2 in want_grads:
        assert O.rel_l2(grads[k2].cpu(), want_grads[k2].cpu()) < 1e-5, k2
    per_expert = store.expert_bytes(0)
    assert streamer.bytes_copied == 2 * len(ids) * per_expert       # forward + backward


def test_streamed_subset_and_generator():
    from lazylora_b200.trainer.expert_streamer import streamed_forward
    cfg, inp, store, lora, resident, x, g, idx, w, ES = _setup("small")
    # route every token away from experts 3..6: the active set has a gap
    keep = (idx < 3) | (idx > 6)
    idx2 = torch.where(keep, idx, torch.full_like(idx, -1))
    w2 = torch.where(keep, w, torch.zeros_like(w))
    streamer = ES(store, lora, cfg.scaling, group_experts=4)
    out, ids = streamed_forward(streamer, 0, x, idx2, w2)
    assert all(not (3 <= e <= 6) for e in ids)
    want = resident.forward(x, idx2, w2)
    assert O.rel_l2(out.cpu(), want.cpu()) < 1e-5
    seen = []
    for e, b in streamer.stream_experts(0, [9, 1, 2, 12]):
        seen.append(e)
        assert b.packed and torch.equal(b.gate_packed.cpu(), inp["w1p"][e])
        assert torch.equal(b.down_scale.cpu(), inp["w2s"][e])
    assert seen == [1, 2, 9, 12]


def test_prefetch_across_layers():
    """With prefetch naming the next layer, its first group is copied during the current
    layer's last group; results equal the resident layers'."""
    import dataclasses
    from lazylora_b200.trainer.expert_streamer import ExpertStreamer, HostExpertStore, streamed_forward
    from lazylora_b200.trainer.routed_experts import RoutedExpertsLayer
    cfg = CONFIGS["small"]
    inps = [make_layer(cfg), make_layer(dataclasses.replace(cfg, seed=5))]
    store = HostExpertStore()
    for l, inp in enumerate(inps):
        store.add_layer(l, {n: inp[n] for n in ("w1p", "w1s", "w3p", "w3s", "w2p", "w2s")})
    lora = {n: inps[0][n].cuda() for n in ("A_g", "B_g", "A_u", "B_u", "A_d", "B_d")}
    streamer = ExpertStreamer(store, lora, cfg.scaling, group_experts=5)
    x = inps[0]["x"].cuda().to(torch.bfloat16)
    idx, w = O.route(inps[0]["x"].float(), inps[0]["router_w"], inps[0]["router_b"], cfg.k)
    idx, w = idx.cuda(), w.cuda()
    every = list(range(cfg.E))
    outs = []
    for l in (0, 1, 0):
        streamer.prefetch((l + 1) % 2, every)
        out, _ = streamed_forward(streamer, l, x, idx, w, expert_ids=every)
        outs.append(out)
    for l, out in zip((0, 1, 0), outs):
        src = dict(inps[l], A_g=inps[0]["A_g"], B_g=inps[0]["B_g"], A_u=inps[0]["A_u"], B_u=inps[0]["B_u"],
                   A_d=inps[0]["A_d"], B_d=inps[0]["B_d"])
        want = RoutedExpertsLayer.from_inputs(src, cfg.scaling).forward(x, idx, w)
        assert O.rel_l2(out.cpu(), want.cpu()) < 1e-5, l


def test_checkpoint_to_pinned_stage_to_streamed_layer(tmp_path):
    """A layer written as a safetensors checkpoint with the reference's tensor names, read by
    the parallel reader straight into the pinned stage, streams to the resident layer's result."""
    from lazylora_b200.streaming.safetensors_reader import SafetensorsIndex, write_layer_experts
    from lazylora_b200.trainer.expert_streamer import ExpertStreamer, HostExpertStore, streamed_forward
    cfg, inp, _store, lora, resident, x, g, idx, w, _ES = _setup("small")
    stacks = {n: inp[n] for n in ("w1p", "w1s", "w3p", "w3s", "w2p", "w2s")}
    write_layer_experts(str(tmp_path / "experts.safetensors"), 5, stacks, range(cfg.E))
    store = HostExpertStore()
    nbytes = store.add_layer_from_checkpoint(5, SafetensorsIndex(str(tmp_path)), cfg.E, threads=4)
    assert nbytes == cfg.E * store.expert_bytes(5)
    assert all(store.layers[5][n].is_pinned() for n in stacks)
    streamer = ExpertStreamer(store, lora, cfg.scaling, group_experts=5)
    out, _ = streamed_forward(streamer, 5, x, idx, w)
    assert O.rel_l2(out.cpu(), resident.forward(x, idx, w).cpu()) < 1e-5
