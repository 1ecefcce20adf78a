"""
GPU parity of the shared expert (dense SiTU-GLU MLP with LoRA on its three projections,
lazy_lora/trainer/lazy_trainer.py:702-707) against the CPU restatement in
oracle/shared_oracle.py (the reference's blocks, backward by autograd).

Tolerances: the block's intermediates are bf16 as in the reference (the projections' outputs,
the LoRA-corrected gate and up, the activation, the input gradient), and a different fp32
summation order can round an element to the neighbouring bf16 value, one ulp = 2^-8 = 3.9e-3
relative. The bf16 output and input gradient, and the fp32 LoRA gradients (contractions of
those bf16 intermediates), are held to 5e-3 relative L2.
"""
import pytest
import torch

from oracle import moe_oracle as O
from oracle import shared_oracle as SO

pytestmark = pytest.mark.gpu
TOL_BF16 = 5e-3


def _case(N, d, F, r, seed=3):
    g = torch.Generator().manual_seed(seed)
    W = lambda o, i: (torch.randn(o, i, generator=g) / i ** 0.5).to(torch.bfloat16)
    ad = {"A_g": torch.randn(r, d, generator=g) / d ** 0.5, "B_g": torch.randn(F, r, generator=g) * 0.05,
          "A_u": torch.randn(r, d, generator=g) / d ** 0.5, "B_u": torch.randn(F, r, generator=g) * 0.05,
          "A_d": torch.randn(r, F, generator=g) / F ** 0.5, "B_d": torch.randn(d, r, generator=g) * 0.05}
    x = torch.randn(N, d, generator=g).to(torch.bfloat16)
    go = torch.randn(N, d, generator=g).to(torch.bfloat16)
    return W(F, d), W(F, d), W(d, F), ad, x, go


@pytest.mark.parametrize("N,d,F,r", [(16, 256, 384, 8), (64, 1024, 768, 16), (5, 512, 1536, 32)])
def test_shared_expert_matches_oracle(N, d, F, r):
    from lazylora_b200.trainer.shared_expert import SharedExpert
    Wg, Wu, Wd, ad, x, go = _case(N, d, F, r)
    scaling = 32.0 / r
    want = SO.shared_expert(x, Wg, Wu, Wd, ad, scaling, grad_out=go)
    se = SharedExpert(Wg.cuda(), Wu.cuda(), Wd.cuda(), *(ad[k].cuda() for k in ("A_g", "B_g", "A_u", "B_u", "A_d",
                                                                              "B_d")), scaling)
    out = se.forward(x.cuda())
    gx, grads = se.backward(go.cuda())
    assert out.dtype == torch.bfloat16 and gx.dtype == torch.bfloat16
    assert O.rel_l2(out.cpu(), want["out"]) < TOL_BF16
    assert O.rel_l2(gx.cpu(), want["grad_x"]) < TOL_BF16
    for k in ("dA_g", "dB_g", "dA_u", "dB_u", "dA_d", "dB_d"):
        assert O.rel_l2(grads[k].cpu(), want[k]) < TOL_BF16, k
