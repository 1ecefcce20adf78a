"""
Real routing decisions (tests/golden/routing_traces.npz: Kimi K3's top-16 of 896 experts on
five prompts, four layers each, from the reference's recorded expert traces; made by
tests/golden/make_trace_fixture.py) as inputs:

  * CPU: the fixture is well formed; the expert-parallel send plan's per-rank load on real
    routing (the imbalance an EP deployment sees) from the oracle;
  * GPU: the CUDA send plan bit-exact against the oracle on every real routing, n = 2, 4, 8;
    the routed-expert layer with real top-16 routing (ids reduced mod E to a small layer)
    against the CPU oracle, forward and backward.
"""
import os

import numpy as np
import pytest
import torch

from oracle import ep_oracle as EPO
from oracle import moe_oracle as O

E_FULL = 896


def _traces(golden_dir):
    z = np.load(os.path.join(golden_dir, "routing_traces.npz"))
    keys = sorted({k.rsplit("/", 1)[0] for k in z.files})
    return [(k, torch.from_numpy(z[k + "/idx"].astype(np.int64)), torch.from_numpy(z[k + "/w"].astype(np.float32)))
            for k in keys]


def test_fixture_well_formed(golden_dir):
    tr = _traces(golden_dir)
    assert len(tr) == 20
    for name, idx, w in tr:
        N, K = idx.shape
        assert K == 16 and 100 <= N <= 300, name
        assert int(idx.min()) >= 0 and int(idx.max()) < E_FULL, name
        assert all(len(set(r.tolist())) == K for r in idx), name          # distinct experts per token
        assert torch.allclose(w.sum(1), torch.ones(N), atol=2e-3), name    # renormalised weights


def test_ep_load_on_real_routing(golden_dir):
    """Rows each rank receives under contiguous expert blocks: real routing is uneven (the
    busiest rank gets more than the mean) but every rank gets work."""
    worst = {}
    for n in (2, 4, 8):
        ratios = []
        for name, idx, w in _traces(golden_dir):
            counts = torch.tensor(EPO.expected_counts(idx, E_FULL, n)[:n], dtype=torch.float64)
            assert int(counts.min()) > 0, (name, n)
            ratios.append(float(counts.max() / counts.mean()))
        worst[n] = max(ratios)
    assert 1.0 <= worst[2] <= worst[8] < 3.0, worst


@pytest.mark.gpu
@pytest.mark.parametrize("n", [2, 4, 8])
def test_cuda_plan_bit_exact_on_real_routing(golden_dir, n):
    from lazylora_b200.trainer.expert_parallel import CudaEPOps
    ref, got = EPO.OracleEPOps(), CudaEPOps()
    for name, idx, w in _traces(golden_dir):
        k = idx.shape[1]
        rc, rpos, rtok, ridx, rw = ref.plan(idx, w, E_FULL, n)
        gc, gpos, gtok, gidx, gw = got.plan(idx.cuda(), w.cuda(), E_FULL, n)
        S = int(rc[:n].sum())
        assert gc.cpu().tolist() == rc.tolist(), name
        assert torch.equal(gpos.cpu(), rpos), name
        assert torch.equal(gtok[:S].cpu(), rtok[:S]), name
        assert torch.equal(gidx[:S].cpu(), ridx.reshape(-1, k)[:S]), name
        assert torch.equal(gw[:S].cpu(), rw.reshape(-1, k)[:S]), name


@pytest.mark.gpu
def test_layer_with_real_top16_routing_matches_oracle(golden_dir):
    """Real top-16 decisions on a small layer (E = 64: ids mod 64, duplicates within a token
    dropped to -1 so each token keeps distinct experts), fwd + bwd against the oracle."""
    from lazylora_b200.synthetic import LayerConfig, make_layer
    from lazylora_b200.trainer.routed_experts import RoutedExpertsLayer
    name, idx, w = _traces(golden_dir)[0]
    E = 64
    idx = idx % E
    for r in range(idx.shape[0]):                          # keep the first of repeated experts
        seen = set()
        for j in range(idx.shape[1]):
            e = int(idx[r, j])
            if e in seen:
                idx[r, j] = -1
                w[r, j] = 0.0
            seen.add(e)
    cfg = LayerConfig(d=512, f=256, E=E, k=16, T=idx.shape[0], r=16, x_dtype="bf16")
    inp = make_layer(cfg)
    k = O.MXFP4Checker()
    lay = O.Layer.from_inputs(inp, cfg.scaling)
    x = inp["x"]
    valid = idx >= 0
    experts = [e for e in O.active_experts(idx) if e >= 0]
    want_out = O.experts_forward(k, lay, x, idx, w, experts=experts)
    want_gh, want_gw = O.experts_backward(k, lay, x, idx, w, inp["g"], experts=experts)
    layer = RoutedExpertsLayer.from_inputs(inp, cfg.scaling)
    xd = x.cuda().to(torch.bfloat16)
    out = layer.forward(xd, idx.cuda(), w.cuda())
    gh, gw, grads = layer.backward(xd, idx.cuda(), w.cuda(), inp["g"].cuda().to(torch.bfloat16))
    layer.check_status(cfg.T, cfg.k)
    assert O.rel_l2(out.cpu(), want_out) < 2e-3
    assert O.rel_l2(gh.cpu(), want_gh.float()) < 2e-3
    assert O.rel_l2(gw.cpu()[valid], want_gw[valid]) < 2e-3
    for key, lo in (("dA_g", lay.gate.grad_A), ("dB_g", lay.gate.grad_B), ("dA_u", lay.up.grad_A),
                    ("dB_u", lay.up.grad_B), ("dA_d", lay.down.grad_A), ("dB_d", lay.down.grad_B)):
        assert O.rel_l2(grads[key].cpu(), lo) < 2e-3, key
