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

HAVE_REF = os.path.exists(O.REF_SO) or os.path.isdir("/root/reference/lazy_lora")


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


def test_moe_block_fixture(golden_dir):
    """The latent MoE block (test_reference_ops.py:259-309): router + per-expert SiTU-GLU + combine."""
    fx = _npz(golden_dir, "fx_moe.npz")
    t = lambda k: torch.from_numpy(fx[k])
    x = t("in")
    hidden = int(fx["hidden"])
    s_act = O.situ_glu_forward(F.linear(x, t("shared_w1_weight")), F.linear(x, t("shared_w3_weight")),
                               float(fx["situ_b1"]), float(fx["situ_b2"]))
    shared = F.linear(s_act, t("shared_w2_weight"))
    idx, w = O.route(x, t("gate_weight"), t("e_score_correction_bias"), int(fx["top_k"]),
                     routed_scaling_factor=float(fx["routed_scale"]))
    h = F.linear(x.reshape(-1, hidden), t("down_weight"))
    routed = torch.zeros_like(h)
    for e in O.active_experts(idx):
        mask = idx == e
        rows = mask.any(-1).nonzero().squeeze(-1)
        xe = h.index_select(0, rows)
        act = O.situ_glu_forward(F.linear(xe, t(f"experts_{e}_w1_weight")), F.linear(xe, t(f"experts_{e}_w3_weight")),
                                 float(fx["situ_b1"]), float(fx["situ_b2"]))
        tw = (w.index_select(0, rows) * mask.index_select(0, rows).float()).sum(-1, keepdim=True)
        routed.index_add_(0, rows, F.linear(act, t(f"experts_{e}_w2_weight")) * tw)
    routed = routed * torch.rsqrt(routed.pow(2).mean(-1, keepdim=True) + float(fx["rms_eps"])) * t("norm_weight")
    got = shared + F.linear(routed, t("up_weight")).view_as(shared)
    _matches(got.numpy(), fx["out"], abs_tol=2e-4)


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
