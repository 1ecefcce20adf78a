"""
GPU parity of the drop-in autograd node and its gradient accumulation, against the
reference's own outputs (tests/golden/ref_<case>.npz).

The reference trainer calls `RoutedExpertsFunction.apply(h_latent, topk_weights,
topk_indices, trainer, layer_idx, bundle, active_experts, cached)`
(lazy_lora/trainer/lazy_trainer.py:45-77, 729-731); its backward returns dL/dh_latent and
dL/dtopk_weights to autograd and accumulates the six LoRA gradients into
bundle.{gate,up,down}_lora.lora_{A,B}.grad (LazyLoRALinear.accumulate_grad,
lazy_lora/core/lora_layer.py:258-290). Here the same node runs with a B200ExpertEngine as
the `trainer`:

  * torch.autograd.grad through the node: grad_h and grad_w within relative L2 2e-3 of the
    reference, the LoRA .grad tensors likewise;
  * a second forward + backward adds the same gradients again (.grad = 2x the reference), as
    accumulate_grad does across micro-batches;
  * the `cached` replay (the trainer's backward pass re-running the layer with the forward's
    saved output): the node returns the cached tensor unchanged, skips the expert sweep, and
    its backward still produces the reference gradients (.grad = 3x);
  * the replay after another forward overwrote the layer's workspace (the backward recomputes
    the forward), and bf16 activations (the gradients take the input dtypes, as in the
    reference).
"""
import os
import types

import numpy as np
import pytest
import torch

from lazylora_b200.synthetic import CONFIGS, make_layer
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu

TOL = 2e-3
LORA = (("gate_lora", "dA_g", "dB_g"), ("up_lora", "dA_u", "dB_u"), ("down_lora", "dA_d", "dB_d"))


def _bundle(inp, dev):
    """A stand-in for the reference's LoRALayerBundle: three modules with lora_A / lora_B
    parameters (fp32, as LazyLoRALinear holds them)."""
    mods = {}
    for name, a, b in (("gate_lora", "A_g", "B_g"), ("up_lora", "A_u", "B_u"), ("down_lora", "A_d", "B_d")):
        mods[name] = types.SimpleNamespace(lora_A=torch.nn.Parameter(inp[a].to(dev).clone()),
                                           lora_B=torch.nn.Parameter(inp[b].to(dev).clone()))
    return types.SimpleNamespace(**mods)


def _setup(golden_dir, case):
    from lazylora_b200.trainer.routed_experts import B200ExpertEngine, RoutedExpertsLayer
    fx = np.load(os.path.join(golden_dir, f"ref_{case}.npz"))
    cfg = CONFIGS[case]
    inp = make_layer(cfg)
    dev = torch.device("cuda")
    layer = RoutedExpertsLayer.from_inputs(inp, cfg.scaling)
    engine = B200ExpertEngine({3: layer})
    bundle = _bundle(inp, dev)
    idx = torch.from_numpy(fx["idx"]).to(dev)
    w = torch.from_numpy(fx["w"]).to(dev)
    active = sorted(set(fx["idx"].reshape(-1).tolist()))
    return fx, cfg, inp, engine, bundle, idx, w, active


def _check_grads(bundle, fx, times, case):
    for mod, ka, kb in LORA:
        m = getattr(bundle, mod)
        for p, key in ((m.lora_A, ka), (m.lora_B, kb)):
            assert p.grad is not None, f"{case}: {mod} {key} has no .grad"
            want = torch.from_numpy(fx[key]) * times
            err = O.rel_l2(p.grad.detach().cpu(), want)
            assert err <= TOL, f"{case}: {mod}.{key} after {times} backward(s): rel-L2 {err:.3e}"


@pytest.mark.parametrize("case", ["c0", "k3", "small"])
def test_autograd_node_matches_reference(golden_dir, case):
    from lazylora_b200.trainer.routed_experts import RoutedExpertsFunction
    fx, cfg, inp, engine, bundle, idx, w, active = _setup(golden_dir, case)
    dev = idx.device
    h = inp["x"].to(dev).float().requires_grad_(True)      # bf16-valued cases fed as fp32: same values
    tw = w.clone().requires_grad_(True)
    g = inp["g"].to(dev).float()

    # 1. forward + autograd backward through the node
    out = RoutedExpertsFunction.apply(h, tw, idx, engine, 3, bundle, active, None)
    assert out.dtype == torch.float32 and out.shape == (cfg.T, cfg.d)
    assert O.rel_l2(out.detach().cpu(), torch.from_numpy(fx["out"])) <= TOL
    gh, gw = torch.autograd.grad(out, (h, tw), grad_outputs=g)
    assert gh.dtype == h.dtype and gw.dtype == tw.dtype
    assert O.rel_l2(gh.cpu(), torch.from_numpy(fx["grad_h"])) <= TOL, "grad_h"
    assert O.rel_l2(gw.cpu(), torch.from_numpy(fx["grad_w"])) <= TOL, "grad_w"
    _check_grads(bundle, fx, 1, case)

    # 2. a second micro-batch on the same inputs: .grad accumulates
    out2 = RoutedExpertsFunction.apply(h, tw, idx, engine, 3, bundle, active, None)
    torch.autograd.grad(out2, (h, tw), grad_outputs=g)
    assert torch.equal(out2, out), "same inputs, same bits"
    _check_grads(bundle, fx, 2, case)

    # 3. the cached replay: output is the cached tensor, backward still streams the experts
    cached = out.detach().clone()
    out3 = RoutedExpertsFunction.apply(h, tw, idx, engine, 3, bundle, active, cached)
    assert torch.equal(out3.detach(), cached)
    gh3, gw3 = torch.autograd.grad(out3, (h, tw), grad_outputs=g)
    assert torch.equal(gh3, gh) and torch.equal(gw3, gw), "replay gradients equal the first pass's"
    _check_grads(bundle, fx, 3, case)


def test_autograd_node_cached_replay_after_other_forward(golden_dir):
    """The replay after another forward went through the same device layer (the workspace no
    longer holds this forward): the backward recomputes it and the gradients are unchanged."""
    from lazylora_b200.trainer.routed_experts import RoutedExpertsFunction
    fx, cfg, inp, engine, bundle, idx, w, active = _setup(golden_dir, "c0")
    dev = idx.device
    h = inp["x"].to(dev).float().requires_grad_(True)
    tw = w.clone().requires_grad_(True)
    g = inp["g"].to(dev).float()
    out = RoutedExpertsFunction.apply(h, tw, idx, engine, 3, bundle, active, None).detach()
    hx, ix, wx = h.detach().flip(0).contiguous(), torch.roll(idx, 1, dims=0).contiguous(), w.flip(0).contiguous()
    engine.layers[3].forward(hx, ix, wx)        # other routing overwrites the shared workspace
    out_r = RoutedExpertsFunction.apply(h, tw, idx, engine, 3, bundle, active, out)
    gh, gw = torch.autograd.grad(out_r, (h, tw), grad_outputs=g)
    assert O.rel_l2(gh.cpu(), torch.from_numpy(fx["grad_h"])) <= TOL
    assert O.rel_l2(gw.cpu(), torch.from_numpy(fx["grad_w"])) <= TOL
    _check_grads(bundle, fx, 1, "c0 replay")


def test_autograd_node_bf16_dtypes(golden_dir):
    """bf16 activations in, gradients returned in the inputs' dtypes (the reference returns
    grad_h.to(h_latent.dtype), grad_w.to(topk_weights.dtype))."""
    from lazylora_b200.trainer.routed_experts import RoutedExpertsFunction
    fx, cfg, inp, engine, bundle, idx, w, active = _setup(golden_dir, "small")
    dev = idx.device
    h = inp["x"].to(dev).to(torch.bfloat16).requires_grad_(True)
    tw = w.clone().requires_grad_(True)
    g = inp["g"].to(dev).float()
    out = RoutedExpertsFunction.apply(h, tw, idx, engine, 3, bundle, active, None)
    gh, gw = torch.autograd.grad(out, (h, tw), grad_outputs=g)
    assert gh.dtype == torch.bfloat16 and gw.dtype == torch.float32
    # rounding grad_h to bf16 alone is ~1e-3 relative; the fp32 result is within 2e-3
    assert O.rel_l2(gh.float().cpu(), torch.from_numpy(fx["grad_h"])) <= 4e-3
    assert O.rel_l2(gw.cpu(), torch.from_numpy(fx["grad_w"])) <= TOL
    _check_grads(bundle, fx, 1, "small bf16")
