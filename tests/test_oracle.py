"""
Pins the CPU oracle before anything is checked against it.

  * the C restatement (oracle/mxfp4_oracle.c) against the reference's own C kernel
    (oracle/_ref, built from lazy_lora/native/mxfp4_gemm.c): dequant bit-exact, GEMMs to fp32
    rounding, and the reference's dequant of an edge block (scale bytes 0..255, >= 253 zero);
  * the Python restatement (oracle/moe_oracle.py) against the reference's vendored fixtures
    for this path (router, SiTU-GLU, the latent MoE block, tolerances of
    lazy_lora/tests/test_reference_ops.py:52-53, 309) and against the goldens made by running
    the reference's trainer methods (tests/golden/make_golden.py): bit-exact routing and row
    order, outputs and gradients bit-exact when the oracle drives the reference kernel.
"""
import os

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from lazylora_b200.synthetic import CONFIGS, make_layer
from oracle import moe_oracle as O

HAVE_REF = os.path.exists(O.REF_SO)


def _npz(golden_dir, name):
    return np.load(os.path.join(golden_dir, name))


def _matches(got, want, abs_tol=1e-5, rel_tol=1e-4):
    got = np.asarray(got, dtype=np.float32).reshape(-1)
    want = np.asarray(want, dtype=np.float32).reshape(-1)
    assert got.shape == want.shape
    assert np.all(np.abs(got - want) <= abs_tol + rel_tol * np.abs(want)), np.abs(got - want).max()


@pytest.fixture(scope="module")
def oracle_k():
    return O.MXFP4Checker("oracle")


@pytest.fixture(scope="module")
def ref_k():
    if not HAVE_REF:
        pytest.skip("reference C kernel not built")
    return O.MXFP4Checker("ref")


def test_dequant_edges_match_reference(golden_dir, oracle_k):
    fx = _npz(golden_dir, "dequant_edges.npz")
    got = oracle_k.dequant(torch.from_numpy(fx["packed"]), torch.from_numpy(fx["scales"]))
    want = fx["out"]
    assert np.array_equal(got.numpy().view(np.uint32), want.view(np.uint32))
    # bytes >= 253 decode to zero (mxfp4_gemm.c:41), and the first group carries every code
    sc = fx["scales"]
    assert np.all(want.reshape(len(sc), 2, 32)[sc >= 253] == 0)


def test_oracle_gemms_match_reference_kernel(oracle_k, ref_k):
    g = torch.Generator().manual_seed(5)
    for (M, K, R) in [(1, 32, 8), (5, 256, 40), (17, 1024, 96), (3, 4096, 64)]:
        packed = torch.randint(0, 256, (R, K // 2), dtype=torch.uint8, generator=g)
        scales = torch.randint(110, 130, (R, K // 32), dtype=torch.uint8, generator=g)
        scales[0, 0] = 255
        x = torch.randn(M, K, generator=g)
        dy = torch.randn(M, R, generator=g)
        assert torch.equal(oracle_k.dequant(packed, scales), ref_k.dequant(packed, scales))
        y0, y1 = oracle_k.gemm(x, packed, scales), ref_k.gemm(x, packed, scales)
        assert O.rel_l2(y1, y0) < 2e-6
        t0, t1 = oracle_k.gemm_t(dy, packed, scales), ref_k.gemm_t(dy, packed, scales)
        assert O.rel_l2(t1, t0) < 2e-6


def test_reference_k_chunking(oracle_k, ref_k):
    """At K = 7168 the reference kernel runs in K chunks of 3584 (its stack tile ends at 4096)."""
    g = torch.Generator().manual_seed(6)
    M, K, R = 4, 7168, 24
    packed = torch.randint(0, 256, (R, K // 2), dtype=torch.uint8, generator=g)
    scales = torch.randint(117, 122, (R, K // 32), dtype=torch.uint8, generator=g)
    x = torch.randn(M, K, generator=g)
    assert O.rel_l2(ref_k.gemm(x, packed, scales), oracle_k.gemm(x, packed, scales)) < 2e-6


def test_router_fixture(golden_dir):
    """lazy_lora/tests/test_reference_ops.py:197-221 on the vendored router.json."""
    fx = _npz(golden_dir, "fx_router.npz")
    idx, w = O.route(torch.from_numpy(fx["in"]), torch.from_numpy(fx["gate_weight"]),
                     torch.from_numpy(fx["bias"]), int(fx["top_k"]))
    got = {(r, int(i)): float(v) for r, (ii, ww) in enumerate(zip(idx.tolist(), w.tolist())) for i, v in zip(ii, ww)}
    want_idx = fx["topk_idx"].astype(np.int64)
    want = {(r, int(i)): float(v) for r, (ii, ww) in enumerate(zip(want_idx.tolist(), fx["topk_weight"].tolist()))
            for i, v in zip(ii, ww)}
    assert sorted(got) == sorted(want)
    _matches([got[k] for k in sorted(got)], [want[k] for k in sorted(want)])


def test_situ_glu_fixture(golden_dir):
    fx = _npz(golden_dir, "fx_situ_glu.npz")
    x = torch.from_numpy(fx["in"])
    d = x.shape[-1] // 2
    got = O.situ_glu_forward(x[..., :d], x[..., d:], beta=float(fx["beta"]), linear_beta=float(fx["linear_beta"]))
    _matches(got.numpy(), fx["out"])


def _fx_moe_parts(fx):
    t = lambda k: torch.from_numpy(fx[k])
    E = int(fx["n_experts"])
    experts = {e: (t(f"experts_{e}_w1_weight"), t(f"experts_{e}_w3_weight"), t(f"experts_{e}_w2_weight"))
               for e in range(E)}
    return t, experts


def test_moe_block_fixture(golden_dir):
    """The MoE block of test_reference_ops.py:259-309 through the oracles' own compositions:
    shared_oracle.shared_expert (no LoRA) plus latent_oracle.latent_block_with (down-projection,
    the fixture's fp32 experts, RMSNorm of their sum, up-projection), routed by moe_oracle.route."""
    from oracle import latent_oracle as LO
    from oracle import shared_oracle as SO
    fx = _npz(golden_dir, "fx_moe.npz")
    t, experts = _fx_moe_parts(fx)
    hidden = int(fx["hidden"])
    x = t("in").reshape(-1, hidden)
    b1, b2 = float(fx["situ_b1"]), float(fx["situ_b2"])
    assert (b1, b2) == (O.SITU_BETA, O.SITU_LINEAR_BETA)      # shared_oracle's SiTU-GLU constants
    F_s = t("shared_w1_weight").shape[0]
    zero_lora = {"A_g": torch.zeros(1, hidden), "B_g": torch.zeros(F_s, 1), "A_u": torch.zeros(1, hidden),
                 "B_u": torch.zeros(F_s, 1), "A_d": torch.zeros(1, F_s), "B_d": torch.zeros(hidden, 1)}
    shared = SO.shared_expert(x, t("shared_w1_weight"), t("shared_w3_weight"), t("shared_w2_weight"), zero_lora,
                              1.0)["out"]
    idx, w = O.route(x, t("gate_weight"), t("e_score_correction_bias"), int(fx["top_k"]),
                     routed_scaling_factor=float(fx["routed_scale"]))
    blk = LO.latent_block_with(lambda h, i, ww: LO.dense_experts_forward(h, i, ww, experts, b1, b2), None,
                               x, t("down_weight"), t("up_weight"), t("norm_weight"), idx, w,
                               eps=float(fx["rms_eps"]))
    got = shared + blk["out"]
    _matches(got.numpy(), fx["out"].reshape(got.shape), abs_tol=2e-4)


def test_latent_block_backward_composition(golden_dir):
    """latent_oracle's manual backward chain (up-projection grad, RMSNorm and cast by autograd,
    the experts' own backward, down-projection grad) equals autograd of its forward, on the
    fixture's block with a seeded upstream gradient: pins the composition the GPU latent block
    is checked against."""
    from oracle import latent_oracle as LO
    fx = _npz(golden_dir, "fx_moe.npz")
    t, experts = _fx_moe_parts(fx)
    hidden = int(fx["hidden"])
    gen = torch.Generator().manual_seed(3)
    x = torch.randn(16, hidden, generator=gen)
    g = torch.randn(16, hidden, generator=gen)
    idx, w = O.route(x, t("gate_weight"), t("e_score_correction_bias"), int(fx["top_k"]))
    down_w, up_w, norm_w, eps = t("down_weight"), t("up_weight"), t("norm_weight"), float(fx["rms_eps"])
    res = LO.latent_block_with(lambda h, i, ww: LO.dense_experts_forward(h, i, ww, experts),
                               lambda h, i, ww, gg: LO.dense_experts_backward(h, i, ww, gg, experts),
                               x, down_w, up_w, norm_w, idx, w, grad_out=g, eps=eps)
    xr = x.clone().requires_grad_(True)
    wr = w.clone().requires_grad_(True)
    h = F.linear(xr, down_w)
    routed = LO.dense_experts_forward(h, idx, wr, experts)
    out = F.linear(routed * torch.rsqrt(routed.pow(2).mean(-1, keepdim=True) + eps) * norm_w, up_w)
    assert O.rel_l2(res["out"], out.detach()) < 1e-6
    gx, gw = torch.autograd.grad(out, (xr, wr), g)
    assert O.rel_l2(res["grad_x"], gx) < 1e-5
    assert O.rel_l2(res["grad_w"], gw) < 1e-5


GOLDEN_KEYS = ("out", "grad_h", "grad_w", "dA_g", "dB_g", "dA_u", "dB_u", "dA_d", "dB_d")


@pytest.mark.parametrize("case", ["tiny", "small", "k3", "c0"])
def test_layer_goldens(golden_dir, case, oracle_k, ref_k):
    if case in ("k3", "c0") and os.environ.get("LAZYLORA_FAST_CPU_TESTS"):
        pytest.skip("large golden skipped in fast mode")
    fx = _npz(golden_dir, f"ref_{case}.npz")
    cfg = CONFIGS[case]
    inp = make_layer(cfg)
    # routing, permutation: bit-exact
    res_ref = O.run_layer(ref_k, inp, cfg.k, cfg.scaling)
    assert np.array_equal(res_ref["idx"].numpy(), fx["idx"])
    assert np.array_equal(res_ref["w"].numpy().view(np.uint32), fx["w"].view(np.uint32))
    for key in ("offsets", "perm_token", "perm_slot"):
        assert np.array_equal(res_ref[key].numpy(), fx[key]), key
    # driving the reference kernel, the restated loop reproduces the reference bit for bit
    for key in GOLDEN_KEYS:
        assert np.array_equal(res_ref[key].numpy(), fx[key]), key
    # the C restatement agrees to fp32 rounding
    res = O.run_layer(oracle_k, inp, cfg.k, cfg.scaling)
    for key in GOLDEN_KEYS:
        assert O.rel_l2(res[key], torch.from_numpy(fx[key])) < 1e-5, key
