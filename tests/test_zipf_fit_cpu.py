"""
The decode bench's routing skew (configs[3]: expert popularity Zipf(s = 1.1)) comes from a
per-expert router bias fitted by lazylora_b200.synthetic.fit_zipf_bias. On a small CPU case:
the fit brings the selection frequencies much closer to the target than no bias does, the
frequencies it reports are the ones the router arithmetic (sigmoid(x Wr^T) + bias, top-k) gives,
and the L1 cannot go below the floor set by an expert being chosen at most once per token.
"""
import torch

from lazylora_b200.synthetic import fit_zipf_bias


def _zipf(E, s):
    p = torch.arange(1, E + 1, dtype=torch.float64) ** -s
    return p / p.sum()


def _freq(w, bias, tokens, k, seed, chunk):
    E, d = w.shape
    gx = torch.Generator().manual_seed(seed)
    counts = torch.zeros(E, dtype=torch.float64)
    for t0 in range(0, tokens, chunk):
        n = min(chunk, tokens - t0)
        x = torch.randn(n, d, generator=gx).to(torch.bfloat16).float()
        sc = torch.sigmoid(x @ w.float().t()) + bias.float()
        counts += torch.bincount(torch.topk(sc, k, dim=-1).indices.reshape(-1), minlength=E).double()
    return counts / (tokens * k)


def test_fit_brings_frequencies_to_the_zipf_target():
    E, d, k, tokens, chunk = 64, 256, 4, 4096, 1024
    w = torch.randn(E, d, generator=torch.Generator().manual_seed(0)) * 0.02
    p = _zipf(E, 1.1)
    bias, l1 = fit_zipf_bias(w, p, k, tokens=tokens, chunk=chunk, iters=400, lr=0.05, step_max=0.02)
    f0 = _freq(w, torch.zeros(E), tokens, k, 7, chunk)
    f1 = _freq(w, bias, tokens, k, 7, chunk)
    l1_none = float((f0 - p).abs().sum())
    assert abs(float((f1 - p).abs().sum()) - l1) < 1e-9, "the reported L1 is the router's own"
    floor = 2 * float((p - 1.0 / k).clamp(min=0).sum())
    assert l1 >= floor - 1e-9
    assert l1 < 0.5 * l1_none, (l1, l1_none)
