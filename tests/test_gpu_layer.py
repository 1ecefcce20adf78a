"""
GPU parity of the routed-expert layer (forward + manual backward) through the C ABI.

  * against the reference's own outputs (tests/golden/ref_<case>.npz, made by running
    LazyLoRATrainer._routed_experts_forward/_backward): out, grad_h, grad_w and the six LoRA
    gradients within relative L2 2e-3 (the bar BASELINE.json's north_star states); the
    stable (expert, token) permutation bit-exact;
  * edge cases the reference's loop handles: experts with no tokens, an expert with more
    tokens than one MMA tile takes, slots routed elsewhere (-1), a single token;
  * the full-width configurations (d=7168, f=2048, E=896, k=8; T=1024 for configs[1] and
    T=8192 for configs[2]'s single-GPU shape) through size-independent properties: token
    independence (outputs of a token subset against the oracle run on that subset alone),
    and bitwise determinism across runs.
"""
import dataclasses
import os

import numpy as np
import pytest
import torch

from lazylora_b200.synthetic import CONFIGS, make_layer, make_layer_device
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu

TOL = 2e-3
KEYS = ("out", "grad_h", "grad_w", "dA_g", "dB_g", "dA_u", "dB_u", "dA_d", "dB_d")


def _run(layer, x, idx, w, g):
    out = layer.forward(x, idx, w)
    gh, gw, grads = layer.backward(x, idx, w, g)
    layer.check_status(idx.shape[0], idx.shape[1])
    return {"out": out, "grad_h": gh, "grad_w": gw, **grads}


@pytest.mark.parametrize("case", ["tiny", "small", "k3", "c0"])
def test_layer_matches_reference_goldens(golden_dir, case):
    from lazylora_b200.trainer.routed_experts import RoutedExpertsLayer
    fx = np.load(os.path.join(golden_dir, f"ref_{case}.npz"))
    cfg = CONFIGS[case]
    inp = make_layer(cfg)
    layer = RoutedExpertsLayer.from_inputs(inp, cfg.scaling)
    x = inp["x"].cuda()
    if cfg.x_dtype == "bf16":
        x = x.to(torch.bfloat16)           # the values are bf16 already; feed them as such
    idx = torch.from_numpy(fx["idx"]).cuda()
    w = torch.from_numpy(fx["w"]).cuda()
    g = inp["g"].cuda()
    got = _run(layer, x, idx, w, g.to(x.dtype))
    for key in KEYS:
        err = O.rel_l2(got[key].cpu(), torch.from_numpy(fx[key]))
        assert err <= TOL, f"{case}.{key}: rel-L2 {err:.3e}"
    off, tok, slot = layer.permutation(cfg.T, cfg.k)
    assert np.array_equal(off.cpu().numpy(), fx["offsets"].astype(np.int32))
    assert np.array_equal(tok.cpu().numpy(), fx["perm_token"].astype(np.int32))
    assert np.array_equal(slot.cpu().numpy(), fx["perm_slot"].astype(np.int32))


def _oracle(inp, idx, w, g, scaling, tokens=None):
    layer = O.Layer.from_inputs(inp, scaling)
    k = O.MXFP4Checker("oracle")
    x = inp["x"].float()
    if tokens is not None:
        x, idx, w, g = x[tokens], idx[tokens], w[tokens], g[tokens]
    experts = [e for e in O.active_experts(idx) if e >= 0]     # -1: slot routed to another rank
    out = O.experts_forward(k, layer, x, idx, w, experts)
    gh, gw = O.experts_backward(k, layer, x, idx, w, g, experts)
    return {"out": out, "grad_h": gh, "grad_w": gw, "dA_g": layer.gate.grad_A, "dB_g": layer.gate.grad_B,
            "dA_u": layer.up.grad_A, "dB_u": layer.up.grad_B, "dA_d": layer.down.grad_A, "dB_d": layer.down.grad_B}


def _masked_routing(idx, w, keep):
    idx = idx.clone()
    w = w.clone()
    idx[~keep] = -1
    w[~keep] = 0
    return idx, w


def test_edge_cases_vs_oracle():
    """Empty experts, one expert over the N tile, slots routed elsewhere, one token."""
    from lazylora_b200.trainer.routed_experts import RoutedExpertsLayer
    cfg = CONFIGS["small"]
    inp = make_layer(cfg)
    layer = RoutedExpertsLayer.from_inputs(inp, cfg.scaling)
    T, k, E = cfg.T, cfg.k, cfg.E
    gen = torch.Generator().manual_seed(9)
    # every token picks expert 3 plus k-1 of experts 5..8 (experts 0-2, 4, 9.. get nothing)
    idx = torch.stack([torch.cat([torch.tensor([3]), torch.randperm(4, generator=gen)[:k - 1] + 5]) for _ in range(T)])
    w = torch.softmax(torch.randn(T, k, generator=gen), -1)
    # half the tokens have their last slot routed to another rank
    keep = torch.ones(T, k, dtype=torch.bool)
    keep[::2, -1] = False
    idx_m, w_m = _masked_routing(idx, w, keep)
    for (ii, ww) in [(idx, w), (idx_m, w_m)]:
        want = _oracle(inp, ii, ww, inp["g"].float(), cfg.scaling)
        got = _run(layer, inp["x"].cuda(), ii.cuda(), ww.cuda(), inp["g"].cuda())
        for key in KEYS:
            gk, wk = got[key].cpu(), want[key]
            if key == "grad_w":
                gk, wk = gk[ii >= 0], wk[ii >= 0]
            assert O.rel_l2(gk, wk) <= TOL, key
    # a single token
    x1 = inp["x"][:1]
    inp1 = dict(inp, x=x1)
    want = _oracle(inp1, idx[:1], w[:1], inp["g"][:1].float(), cfg.scaling)
    got = _run(layer, x1.cuda(), idx[:1].cuda(), w[:1].cuda(), inp["g"][:1].cuda())
    for key in KEYS:
        assert O.rel_l2(got[key].cpu(), want[key]) <= TOL, key


@pytest.mark.parametrize("T", [1, 2, 3, 4, 5])
def test_few_tokens_vs_oracle(T):
    """Up to four tokens the forward GEMMs use four-row activation tiles (MMA N = 16) and the
    backward's fp16 GEMMs 16-row tiles; five tokens are back on 16-row tiles. Forward and
    backward against the oracle."""
    from lazylora_b200.trainer.routed_experts import RoutedExpertsLayer
    cfg = dataclasses.replace(CONFIGS["small"], T=T)
    inp = make_layer(cfg)
    layer = RoutedExpertsLayer.from_inputs(inp, cfg.scaling)
    gen = torch.Generator().manual_seed(40 + T)
    idx = torch.stack([torch.randperm(cfg.E, generator=gen)[:cfg.k] for _ in range(T)])
    w = torch.softmax(torch.randn(T, cfg.k, generator=gen), -1)
    x = inp["x"][:T]
    g = inp["g"][:T]
    want = _oracle(dict(inp, x=x), idx, w, g.float(), cfg.scaling)
    got = _run(layer, x.cuda(), idx.cuda(), w.cuda(), g.cuda())
    for key in KEYS:
        assert O.rel_l2(got[key].cpu(), want[key]) <= TOL, (T, key)


def test_expert_over_tile_width():
    """An expert with more rows than N_MAX (128) is split into chunks; results unchanged."""
    from lazylora_b200.trainer.routed_experts import RoutedExpertsLayer
    cfg = CONFIGS["tiny"]
    inp = make_layer(dataclasses.replace(cfg, T=300))
    layer = RoutedExpertsLayer.from_inputs(inp, cfg.scaling)
    T, k = 300, cfg.k
    idx = torch.stack([torch.tensor([0, 1 + (t % 7)]) for t in range(T)])
    w = torch.full((T, k), 0.5)
    want = _oracle(inp, idx, w, inp["g"].float(), cfg.scaling)
    got = _run(layer, inp["x"].cuda(), idx.cuda(), w.cuda(), inp["g"].cuda())
    for key in KEYS:
        assert O.rel_l2(got[key].cpu(), want[key]) <= TOL, key


def _full_width_layer(name):
    from lazylora_b200.trainer.routed_experts import RoutedExpertsLayer
    from lazylora_b200.core.moe_router import KimiK3MoERouter
    cfg = CONFIGS[name]
    inp = make_layer_device(cfg)
    layer = RoutedExpertsLayer.from_inputs(inp, cfg.scaling)
    router = KimiK3MoERouter(hidden_size=cfg.d, num_experts=cfg.E, top_k=cfg.k)
    x = inp["x"].to(torch.bfloat16)
    idx, w = router.forward(x, weight=inp["router_w"], bias=inp["router_b"])
    return cfg, inp, layer, x, idx, w


@pytest.fixture(scope="module")
def c1_layer():
    return _full_width_layer("c1")


def _token_subset_vs_oracle(cfg, inp, layer, x, idx, w, tokens):
    """Token independence: the layer's outputs for `tokens` (run inside the full batch) against
    the oracle run on those tokens alone, over only the experts they touch; the LoRA gradients
    of the full-batch run with the upstream gradient zeroed outside `tokens`. Returns the
    number of experts the tokens touch."""
    g = inp["g"].to(torch.bfloat16)
    got = _run(layer, x, idx, w, g)
    tk = tokens.to(idx.device)
    sub = idx[tk].cpu()
    experts = sorted(set(sub.flatten().tolist()))
    remap = {e: i for i, e in enumerate(experts)}
    ev = torch.tensor(experts, device=idx.device)
    cpu = {key: inp[key][ev].cpu() for key in ("w1p", "w1s", "w3p", "w3s", "w2p", "w2s")}
    cpu.update({key: inp[key].cpu() for key in ("A_g", "B_g", "A_u", "B_u", "A_d", "B_d")})
    cpu["x"] = x[tk].float().cpu()
    sub_idx = sub.clone().apply_(lambda e: remap[e])
    g_sub = torch.zeros_like(g)
    g_sub[tk] = g[tk]
    got_sub = _run(layer, x, idx, w, g_sub)
    want = _oracle(cpu, sub_idx, w[tk].cpu(), g[tk].float().cpu(), cfg.scaling)
    for key in ("out", "grad_h", "grad_w"):
        err = O.rel_l2(got[key][tk].cpu(), want[key])
        assert err <= TOL, f"{key}: rel-L2 {err:.3e}"
    for key in ("dA_g", "dB_g", "dA_u", "dB_u", "dA_d", "dB_d"):
        err = O.rel_l2(got_sub[key].cpu(), want[key])
        assert err <= TOL, f"{key}: rel-L2 {err:.3e}"
    return len(experts)


def test_full_width_token_subset(c1_layer):
    """configs[1] (896 experts, 16-row token tiles): 64 tokens spread over the batch, which
    touch a few hundred experts, against the oracle."""
    cfg, inp, layer, x, idx, w = c1_layer
    tokens = torch.linspace(0, cfg.T - 1, 64).round().long()
    n_exp = _token_subset_vs_oracle(cfg, inp, layer, x, idx, w, tokens)
    assert n_exp >= 200, n_exp


@pytest.mark.parametrize("T", [1, 4, 16])
def test_full_width_decode_batches(c1_layer, T):
    """Decode-sized batches of the 896-expert layer (configs[3]'s T = 1, 4, 16: the one-launch
    sort with the x terms, and the GEMMs' K stages shared out evenly over the CTAs, a unit cut
    between CTAs finished from fp32 partials) against the oracle, and bitwise repeatable."""
    cfg, inp, layer, x, idx, w = c1_layer
    sub = dict(inp, g=inp["g"][:T])
    tokens = torch.arange(T)
    _token_subset_vs_oracle(cfg, sub, layer, x[:T].contiguous(), idx[:T].contiguous(), w[:T].contiguous(), tokens)
    a = layer.forward(x[:T].contiguous(), idx[:T].contiguous(), w[:T].contiguous())
    b = layer.forward(x[:T].contiguous(), idx[:T].contiguous(), w[:T].contiguous())
    layer.check_status(T, cfg.k)
    assert torch.equal(a, b)


def test_split_thresholds_raised_subprocess():
    """The balanced split on every launch it can take (F1 and F2 up to 1280 units, env read once
    per process, so in a child pytest): the c0 / k3 goldens and the decode batches."""
    import os
    import subprocess
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    env = dict(os.environ, LL_BS_SPLIT_F1="1280", LL_BS_SPLIT_F2="1280")
    r = subprocess.run([sys.executable, "-m", "pytest", "-x", "-q", "-p", "no:cacheprovider",
                        os.path.join(here, "test_gpu_layer.py"), "-k",
                        "(goldens and (c0 or k3)) or decode_batches"],
                       env=env, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert " passed" in r.stdout and "5 passed" in r.stdout, r.stdout[-2000:]


def test_configs2_shape_token_subset():
    """configs[2]'s single-GPU shape (T = 8192, about 73 rows per expert: the 128-row token
    tiles, experts split over two chunks): 24 tokens spread over the batch against the oracle."""
    cfg, inp, layer, x, idx, w = _full_width_layer("c2")
    tokens = torch.linspace(0, cfg.T - 1, 24).round().long()
    _token_subset_vs_oracle(cfg, inp, layer, x, idx, w, tokens)
    del layer, inp
    torch.cuda.empty_cache()


def test_full_width_deterministic(c1_layer):
    cfg, inp, layer, x, idx, w = c1_layer
    g = inp["g"].to(torch.bfloat16)
    a = _run(layer, x, idx, w, g)
    b = _run(layer, x, idx, w, g)
    for key in KEYS:
        assert torch.equal(a[key], b[key]), key


@pytest.mark.parametrize("r,T", [(64, 48), (48, 40), (8, 600), (16, 120)])
def test_lora_rank_and_many_tokens_vs_oracle(r, T):
    """LoRA ranks above 32 (configs[4] uses r = 64; the rank-r kernels work 32 ranks at a
    time) and token counts that take the 64- and 128-row tile paths, against the oracle."""
    from lazylora_b200.trainer.routed_experts import RoutedExpertsLayer
    cfg = dataclasses.replace(CONFIGS["small"], r=r, T=T)
    inp = make_layer(cfg)
    layer = RoutedExpertsLayer.from_inputs(inp, cfg.scaling)
    idx, w = O.route(inp["x"].float(), inp["router_w"], inp["router_b"], cfg.k)
    want = _oracle(inp, idx, w, inp["g"].float(), cfg.scaling)
    x = inp["x"].cuda().to(torch.bfloat16)
    got = _run(layer, x, idx.cuda(), w.cuda(), inp["g"].cuda().to(torch.bfloat16))
    for key in KEYS:
        assert O.rel_l2(got[key].cpu(), want[key]) <= TOL, f"r={r} T={T} {key}"
