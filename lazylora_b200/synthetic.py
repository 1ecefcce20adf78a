"""
Seeded synthetic inputs for the routed-expert layer.

The reference measures on the Kimi K3 checkpoint, which is not available here, so every
input is drawn from the distributions the benchmark configurations name:

  router weight  Wr [E, d]   ~ N(0, 0.02^2); bias [E] = 0 unless a Zipf skew is asked for
  per expert e, in id order:
     gate W1 / up W3: packed [f, d/2] u8 uniform 0..255 (two uniform E2M1 codes a byte),
                      scales [f, d/32] = 127 + U{-10..-6}  (bytes 117..121)
     down W2:         packed [d, f/2], scales [d, f/32], same distributions
  LoRA gate/up/down: A ~ N(0, 1/fan_in), B ~ N(0, 1e-4); alpha = 32
  x [T, d] ~ N(0, 1)   fp32 for the CPU-sized case, bf16-rounded otherwise
  g [T, d] ~ N(0, 1)   upstream gradient, same dtype rule

`make_layer(cfg)` draws them on the CPU with a torch.Generator seeded `cfg.seed`, in the
order above, so the oracle and the CUDA path read identical bytes. `make_layer_device`
draws the same distributions directly in HBM (a different random stream) for the
full-width benchmark, where 21 GB of weights would not be worth a host round trip.
"""
from dataclasses import dataclass, replace
from typing import Dict, Optional

import math
import torch


@dataclass(frozen=True)
class LayerConfig:
    d: int            # expert input width (K of gate/up)
    f: int            # expert intermediate width
    E: int            # routed experts
    k: int            # top-k
    T: int            # tokens
    r: int = 16       # LoRA rank
    alpha: int = 32   # LoRA alpha (scaling = alpha / r)
    x_dtype: str = "bf16"   # "f32" or "bf16" (values rounded to bf16, held as fp32 for the oracle)
    zipf_s: Optional[float] = None   # router-bias skew, None = uniform-ish routing
    zipf_gamma: float = 0.05         # bias_e = gamma * ln(p_e / p_max) (fit_zipf_gamma picks it)
    seed: int = 0

    @property
    def scaling(self) -> float:
        return self.alpha / self.r

    @property
    def pairs(self) -> int:
        return self.T * self.k

    def expert_bytes(self) -> int:
        """MXFP4 bytes of one expert (gate + up + down, packed codes + scale bytes)."""
        return 3 * self.f * self.d // 2 + 3 * self.f * self.d // 32


# The benchmark configurations (BASELINE configs[0..4]) plus small parity cases.
CONFIGS: Dict[str, LayerConfig] = {
    "c0": LayerConfig(d=7168, f=2048, E=16, k=8, T=32, x_dtype="f32"),
    "c1": LayerConfig(d=7168, f=2048, E=896, k=8, T=1024),
    "c2": LayerConfig(d=7168, f=2048, E=896, k=8, T=8192),
    "c3_t1": LayerConfig(d=7168, f=2048, E=896, k=8, T=1, zipf_s=1.1),
    "c3_t4": LayerConfig(d=7168, f=2048, E=896, k=8, T=4, zipf_s=1.1),
    "c3_t16": LayerConfig(d=7168, f=2048, E=896, k=8, T=16, zipf_s=1.1),
    "c4": LayerConfig(d=7168, f=2048, E=896, k=8, T=2048, r=64),
    # configs[1]'s per-expert load (9 tokens per expert) on 64 experts: 1.5 GB of weights,
    # larger than L2 but small enough for multi-pass ncu captures
    "prof": LayerConfig(d=7168, f=2048, E=64, k=8, T=72),
    # configs[1] with the routed experts at Kimi K3's latent width (routed_expert_hidden_size
    # 3584; the block projects 7168 -> 3584 -> experts -> RMSNorm -> 7168)
    "c1_latent": LayerConfig(d=3584, f=2048, E=896, k=8, T=1024),
    # configs[1]'s token count (the LoRA products, combines and router see T = 1024, 8192 pairs)
    # on 64 experts, for captures of the small kernels around the GEMMs
    "prof_aux": LayerConfig(d=7168, f=2048, E=64, k=8, T=1024),
    # small parity cases (K <= 4096 so the reference C kernel runs unchunked)
    "tiny": LayerConfig(d=256, f=128, E=8, k=2, T=16, r=4, alpha=8, x_dtype="f32"),
    "small": LayerConfig(d=1024, f=512, E=16, k=4, T=48, r=16, x_dtype="bf16"),
    "k3": LayerConfig(d=3584, f=3072, E=32, k=16, T=24, r=16, x_dtype="bf16"),
}


def _round_bf16(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.bfloat16).to(torch.float32)


def zipf_bias(E: int, s: float, gamma: float, gen: torch.Generator) -> torch.Tensor:
    """bias_e = gamma * ln(p_e / p_max) with p_e proportional to rank_e^-s, ranks a seeded permutation."""
    p = zipf_target(E, s, gen)
    return (gamma * torch.log(p / p.max())).to(torch.float32)


def zipf_target(E: int, s: float, gen: torch.Generator) -> torch.Tensor:
    """p_e proportional to rank_e^-s over a seeded permutation of ranks (same draw as zipf_bias)."""
    perm = torch.randperm(E, generator=gen)
    rank = torch.empty(E, dtype=torch.float64)
    rank[perm] = torch.arange(1, E + 1, dtype=torch.float64)
    p = rank.pow(-s)
    return p / p.sum()


def fit_zipf_bias(router_w: torch.Tensor, p: torch.Tensor, k: int, tokens: int = 65536, chunk: int = 8192,
                  iters: int = 1000, lr: float = 0.01, step_max: float = 0.005, seed: int = 7):
    """A per-expert router bias whose top-k selection frequencies over `tokens` seeded N(0,1)
    (bf16) tokens approach the target p (iterative: bias_e += clip(lr * (ln p_e - ln f_e),
    +-step_max); the scores' spread is a few tenths, so steps stay small). An expert
    is chosen at most once per token, so frequencies above 1/k are out of reach; those targets
    are capped at 1/k for the iteration. Returns (bias [E] fp32, L1 of the achieved frequencies
    against the uncapped p). The router arithmetic is the reference's: sigmoid(x Wr^T) + bias,
    top-k of that (lazy_lora/core/moe_router.py:80-100)."""
    dev = router_w.device
    E, d = router_w.shape
    gx = torch.Generator(device=dev).manual_seed(seed)
    scores = torch.empty((tokens, E), dtype=torch.float32, device=dev)
    for t0 in range(0, tokens, chunk):
        n = min(chunk, tokens - t0)
        x = torch.randn(n, d, generator=gx, device=dev).to(torch.bfloat16).float()
        scores[t0:t0 + n] = torch.sigmoid(x @ router_w.float().t())
    p = p.to(dev).double()
    target = torch.log(p.clamp(max=1.0 / k))
    bias = torch.zeros(E, dtype=torch.float64, device=dev)

    def freq(b):
        idx = torch.topk(scores + b.float(), k, dim=-1).indices
        return torch.bincount(idx.reshape(-1), minlength=E).double() / (tokens * k)

    for _ in range(iters):
        f = freq(bias)
        bias += (lr * (target - torch.log(f + 0.5 / (tokens * k)))).clamp(-step_max, step_max)
        bias -= bias.max()
    f = freq(bias)
    return bias.float(), float((f - p).abs().sum())


def fit_zipf_gamma(cfg: LayerConfig, device="cuda", tokens: int = 65536, chunk: int = 8192):
    """The router-bias scale gamma whose top-k selection frequencies over `tokens` seeded
    N(0,1) tokens best match the Zipf target p in L1 (1-D search, log grid then refinement).
    Returns (gamma, L1). The router arithmetic is the reference's: sigmoid(x Wr^T) + bias,
    top-k of that (lazy_lora/core/moe_router.py:80-100); ties do not matter for frequencies."""
    dev = torch.device(device)
    E, d, k = cfg.E, cfg.d, cfg.k
    g = torch.Generator(device=device).manual_seed(cfg.seed)
    Wr = torch.randn(E, d, generator=g, device=dev) * 0.02
    gx = torch.Generator(device=device).manual_seed(cfg.seed + 7)
    scores = torch.empty((tokens, E), dtype=torch.float32, device=dev)
    for t0 in range(0, tokens, chunk):
        n = min(chunk, tokens - t0)
        x = torch.randn(n, d, generator=gx, device=dev).to(torch.bfloat16).float()
        scores[t0:t0 + n] = torch.sigmoid(x @ Wr.t())
    p = zipf_target(E, cfg.zipf_s, torch.Generator(device="cpu").manual_seed(cfg.seed + 1)).to(dev)
    lnp = torch.log(p / p.max()).float()

    def l1(gamma: float) -> float:
        idx = torch.topk(scores + gamma * lnp, k, dim=-1).indices
        freq = torch.bincount(idx.reshape(-1), minlength=E).double() / (tokens * k)
        return float((freq - p).abs().sum())

    grid = [10 ** (-3 + 4 * i / 80) for i in range(81)]
    vals = [l1(x) for x in grid]
    i = min(range(len(grid)), key=vals.__getitem__)
    lo, hi = grid[max(i - 1, 0)], grid[min(i + 1, len(grid) - 1)]
    for _ in range(30):                       # golden-section refinement on [lo, hi]
        a = hi - (hi - lo) / 1.618034
        b = lo + (hi - lo) / 1.618034
        if l1(a) < l1(b):
            hi = b
        else:
            lo = a
    gamma = (lo + hi) / 2
    return gamma, l1(gamma)


def make_layer(cfg: LayerConfig, with_grad: bool = True) -> Dict[str, torch.Tensor]:
    """All inputs of one layer on the CPU, drawn in the documented order."""
    d, f, E, r = cfg.d, cfg.f, cfg.E, cfg.r
    assert d % 32 == 0 and f % 32 == 0, "MXFP4 needs K a multiple of 32"
    g = torch.Generator(device="cpu").manual_seed(cfg.seed)
    out: Dict[str, torch.Tensor] = {}
    out["router_w"] = torch.randn(E, d, generator=g) * 0.02
    out["router_b"] = torch.zeros(E)
    w1p = torch.empty(E, f, d // 2, dtype=torch.uint8)
    w1s = torch.empty(E, f, d // 32, dtype=torch.uint8)
    w3p = torch.empty_like(w1p)
    w3s = torch.empty_like(w1s)
    w2p = torch.empty(E, d, f // 2, dtype=torch.uint8)
    w2s = torch.empty(E, d, f // 32, dtype=torch.uint8)
    for e in range(E):
        w1p[e] = torch.randint(0, 256, (f, d // 2), dtype=torch.uint8, generator=g)
        w1s[e] = (torch.randint(-10, -5, (f, d // 32), generator=g) + 127).to(torch.uint8)
        w3p[e] = torch.randint(0, 256, (f, d // 2), dtype=torch.uint8, generator=g)
        w3s[e] = (torch.randint(-10, -5, (f, d // 32), generator=g) + 127).to(torch.uint8)
        w2p[e] = torch.randint(0, 256, (d, f // 2), dtype=torch.uint8, generator=g)
        w2s[e] = (torch.randint(-10, -5, (d, f // 32), generator=g) + 127).to(torch.uint8)
    out.update(w1p=w1p, w1s=w1s, w3p=w3p, w3s=w3s, w2p=w2p, w2s=w2s)
    out["A_g"] = torch.randn(r, d, generator=g) / math.sqrt(d)
    out["B_g"] = torch.randn(f, r, generator=g) * 0.01
    out["A_u"] = torch.randn(r, d, generator=g) / math.sqrt(d)
    out["B_u"] = torch.randn(f, r, generator=g) * 0.01
    out["A_d"] = torch.randn(r, f, generator=g) / math.sqrt(f)
    out["B_d"] = torch.randn(d, r, generator=g) * 0.01
    x = torch.randn(cfg.T, d, generator=g)
    out["x"] = x if cfg.x_dtype == "f32" else _round_bf16(x)
    if with_grad:
        gr = torch.randn(cfg.T, d, generator=g)
        out["g"] = gr if cfg.x_dtype == "f32" else _round_bf16(gr)
    if cfg.zipf_s is not None:
        out["router_b"] = zipf_bias(E, cfg.zipf_s, gamma=cfg.zipf_gamma, gen=g)
    return out


def make_layer_device(cfg: LayerConfig, device="cuda", with_grad: bool = True) -> Dict[str, torch.Tensor]:
    """Same distributions as make_layer, drawn directly on `device` (different stream)."""
    d, f, E, r = cfg.d, cfg.f, cfg.E, cfg.r
    g = torch.Generator(device=device).manual_seed(cfg.seed)
    dev = torch.device(device)
    out: Dict[str, torch.Tensor] = {}
    out["router_w"] = torch.randn(E, d, generator=g, device=dev) * 0.02
    out["router_b"] = torch.zeros(E, device=dev)

    def packed(rows, cols):
        return torch.randint(0, 256, (E, rows, cols // 2), dtype=torch.uint8, generator=g, device=dev)

    def scales(rows, cols):
        return (torch.randint(-10, -5, (E, rows, cols // 32), generator=g, device=dev,
                              dtype=torch.int32) + 127).to(torch.uint8)

    out["w1p"], out["w1s"] = packed(f, d), scales(f, d)
    out["w3p"], out["w3s"] = packed(f, d), scales(f, d)
    out["w2p"], out["w2s"] = packed(d, f), scales(d, f)
    out["A_g"] = torch.randn(r, d, generator=g, device=dev) / math.sqrt(d)
    out["B_g"] = torch.randn(f, r, generator=g, device=dev) * 0.01
    out["A_u"] = torch.randn(r, d, generator=g, device=dev) / math.sqrt(d)
    out["B_u"] = torch.randn(f, r, generator=g, device=dev) * 0.01
    out["A_d"] = torch.randn(r, f, generator=g, device=dev) / math.sqrt(f)
    out["B_d"] = torch.randn(d, r, generator=g, device=dev) * 0.01
    x = torch.randn(cfg.T, d, generator=g, device=dev)
    out["x"] = x if cfg.x_dtype == "f32" else _round_bf16(x)
    if with_grad:
        gr = torch.randn(cfg.T, d, generator=g, device=dev)
        out["g"] = gr if cfg.x_dtype == "f32" else _round_bf16(gr)
    if cfg.zipf_s is not None:
        gc = torch.Generator(device="cpu").manual_seed(cfg.seed + 1)
        out["router_b"] = zipf_bias(E, cfg.zipf_s, gamma=cfg.zipf_gamma, gen=gc).to(dev)
    return out


def make_ep_rank_device(cfg: LayerConfig, rank: int, world: int, device="cuda",
                        with_grad: bool = True) -> Dict[str, torch.Tensor]:
    """One rank's inputs for an expert-parallel layer of `world` ranks, drawn on `device`.

    Replicated on every rank (stream seeded `cfg.seed`): the router weight and bias and the
    three LoRA adapters. Rank-local (stream seeded `cfg.seed + 1 + rank`): the MXFP4 weights
    of the rank's experts (the contiguous block of expert e = floor(e * world / E)) and its
    cfg.T tokens x and upstream gradient g. Same distributions as make_layer.
    """
    d, f, E, r = cfg.d, cfg.f, cfg.E, cfg.r
    lo = (rank * E + world - 1) // world
    n_loc = ((rank + 1) * E + world - 1) // world - lo
    dev = torch.device(device)
    gs = torch.Generator(device=device).manual_seed(cfg.seed)
    gl = torch.Generator(device=device).manual_seed(cfg.seed + 1 + rank)
    out: Dict[str, torch.Tensor] = {"first_expert": torch.tensor(lo), "n_local": torch.tensor(n_loc)}
    out["router_w"] = torch.randn(E, d, generator=gs, device=dev) * 0.02
    out["router_b"] = torch.zeros(E, device=dev)
    if cfg.zipf_s is not None:
        gc = torch.Generator(device="cpu").manual_seed(cfg.seed + 1)
        out["router_b"] = zipf_bias(E, cfg.zipf_s, gamma=cfg.zipf_gamma, gen=gc).to(dev)
    out["A_g"] = torch.randn(r, d, generator=gs, device=dev) / math.sqrt(d)
    out["B_g"] = torch.randn(f, r, generator=gs, device=dev) * 0.01
    out["A_u"] = torch.randn(r, d, generator=gs, device=dev) / math.sqrt(d)
    out["B_u"] = torch.randn(f, r, generator=gs, device=dev) * 0.01
    out["A_d"] = torch.randn(r, f, generator=gs, device=dev) / math.sqrt(f)
    out["B_d"] = torch.randn(d, r, generator=gs, device=dev) * 0.01

    def packed(rows, cols):
        return torch.randint(0, 256, (n_loc, rows, cols // 2), dtype=torch.uint8, generator=gl, device=dev)

    def scales(rows, cols):
        return (torch.randint(-10, -5, (n_loc, rows, cols // 32), generator=gl, device=dev,
                              dtype=torch.int32) + 127).to(torch.uint8)

    out["w1p"], out["w1s"] = packed(f, d), scales(f, d)
    out["w3p"], out["w3s"] = packed(f, d), scales(f, d)
    out["w2p"], out["w2s"] = packed(d, f), scales(d, f)
    x = torch.randn(cfg.T, d, generator=gl, device=dev)
    out["x"] = x if cfg.x_dtype == "f32" else _round_bf16(x)
    if with_grad:
        gr = torch.randn(cfg.T, d, generator=gl, device=dev)
        out["g"] = gr if cfg.x_dtype == "f32" else _round_bf16(gr)
    return out


def with_config(name: str, **kw) -> LayerConfig:
    return replace(CONFIGS[name], **kw)
