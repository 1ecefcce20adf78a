"""
GPU check of HostStepPipeline: steps fed from pinned host memory with the copies on their own
streams give, step by step, exactly the results of the same steps run on device tensors
(the kernels are deterministic, so the comparison is bitwise), including when one host
output buffer serves several steps.
"""
import pytest
import torch

from lazylora_b200.synthetic import CONFIGS, make_layer

pytestmark = pytest.mark.gpu


def _setup():
    from lazylora_b200.core.moe_router import KimiK3MoERouter
    from lazylora_b200.trainer.routed_experts import RoutedExpertsLayer
    cfg = CONFIGS["small"]
    inp = make_layer(cfg)
    layer = RoutedExpertsLayer.from_inputs(inp, cfg.scaling)
    router = KimiK3MoERouter(hidden_size=cfg.d, num_experts=cfg.E, top_k=cfg.k)
    Wr, br = inp["router_w"].cuda(), inp["router_b"].cuda()

    def step(x, g):
        idx, w = router.forward(x, weight=Wr, bias=br)
        out = layer.forward(x, idx, w)
        gh, gw, grads = layer.backward(x, idx, w, g)
        return out, gh, gw, grads

    return cfg, step


def test_pipeline_matches_plain_steps():
    from lazylora_b200.trainer.host_pipeline import HostStepPipeline
    cfg, step = _setup()
    gen = torch.Generator().manual_seed(3)
    n = 4
    xs = [torch.randn(cfg.T, cfg.d, generator=gen).to(torch.bfloat16).pin_memory() for _ in range(n)]
    gs = [torch.randn(cfg.T, cfg.d, generator=gen).to(torch.bfloat16).pin_memory() for _ in range(n)]
    pinned = lambda *shape: torch.empty(shape, dtype=torch.float32).pin_memory()
    outs = [(pinned(cfg.T, cfg.d), pinned(cfg.T, cfg.d), pinned(cfg.T, cfg.k)) for _ in range(n)]
    pipe = HostStepPipeline(step, out_index=[0, 1, 2])
    pipe.run(xs, gs, outs)
    torch.cuda.synchronize()
    for i in range(n):
        want = step(xs[i].cuda(), gs[i].cuda())
        for j in range(3):
            assert torch.equal(outs[i][j], want[j].cpu()), (i, j)
    # one shared set of host buffers: it ends up holding the last step's results
    shared = (pinned(cfg.T, cfg.d), pinned(cfg.T, cfg.d), pinned(cfg.T, cfg.k))
    pipe.run(xs, gs, [shared] * n)
    torch.cuda.synchronize()
    for j in range(3):
        assert torch.equal(shared[j], outs[n - 1][j]), j


def test_pipeline_rejects_pageable_buffers():
    from lazylora_b200.trainer.host_pipeline import HostStepPipeline
    cfg, step = _setup()
    x = torch.zeros(cfg.T, cfg.d, dtype=torch.bfloat16)
    pipe = HostStepPipeline(step, out_index=[0])
    with pytest.raises(ValueError):
        pipe.run([x], [x], [(torch.zeros(cfg.T, cfg.d),)])


def test_captured_step_and_graph_pipeline_match_eager():
    from lazylora_b200.trainer.host_pipeline import CapturedStep, HostStepPipeline
    cfg, step = _setup()
    gen = torch.Generator().manual_seed(5)
    x = torch.randn(cfg.T, cfg.d, generator=gen).to(torch.bfloat16).cuda()
    g = torch.randn(cfg.T, cfg.d, generator=gen).to(torch.bfloat16).cuda()
    want = step(x, g)
    cap = CapturedStep(step, x, g)
    got = cap.replay()
    torch.cuda.synchronize()
    for j in range(3):
        assert torch.equal(got[j], want[j]), j
    n = 3
    xs = [torch.randn(cfg.T, cfg.d, generator=gen).to(torch.bfloat16).pin_memory() for _ in range(n)]
    gs = [torch.randn(cfg.T, cfg.d, generator=gen).to(torch.bfloat16).pin_memory() for _ in range(n)]
    pinned = lambda *shape: torch.empty(shape, dtype=torch.float32).pin_memory()
    outs = [(pinned(cfg.T, cfg.d), pinned(cfg.T, cfg.d), pinned(cfg.T, cfg.k)) for _ in range(n)]
    HostStepPipeline(step, out_index=[0, 1, 2], graph=True).run(xs, gs, outs)
    torch.cuda.synchronize()
    for i in range(n):
        ref = step(xs[i].cuda(), gs[i].cuda())
        for j in range(3):
            assert torch.equal(outs[i][j], ref[j].cpu()), (i, j)
