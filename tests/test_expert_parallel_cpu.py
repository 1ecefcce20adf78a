"""
Expert-parallel layer on CPU `gloo` ranks (no GPU): the rank orchestration of
lazylora_b200.trainer.expert_parallel.ExpertParallelLayer (plan, count exchange, row
dispatch, packed partial return, ordered combine, slot combine, LoRA all-reduce), driven with the
CPU restatement of the index operations (oracle/ep_oracle.py) and the reference-algorithm
expert loop (oracle/moe_oracle.py) as each rank's local layer. An n-rank run must give the
single-process result over all tokens (to the fp16 rounding of the returned partial rows).
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from lazylora_b200.synthetic import LayerConfig, make_layer
from lazylora_b200.trainer.expert_parallel import ExpertParallelLayer, experts_of_rank
from oracle import ep_oracle as EPO
from oracle import moe_oracle as O


class OracleLocalLayer:
    """One rank's experts through the reference-algorithm loop (local ids 0..E-1, -1 skipped)."""

    def __init__(self, inp, E_local, scaling):
        self.E = E_local
        self.inp = inp
        self.scaling = scaling
        self.k = O.MXFP4Checker("oracle")
        self.d = inp["w1p"].shape[2] * 2
        self.f = inp["w1p"].shape[1]
        self.r = inp["A_g"].shape[0]

    def lora_shapes(self):
        d, f, r = self.d, self.f, self.r
        return {"dA_g": (r, d), "dB_g": (f, r), "dA_u": (r, d), "dB_u": (f, r), "dA_d": (r, f), "dB_d": (d, r)}

    def forward(self, x, idx, w):
        layer = O.Layer.from_inputs(self.inp, self.scaling)
        return O.experts_forward(self.k, layer, x.float(), idx, w, experts=list(range(self.E)))

    def backward(self, x, idx, w, g):
        layer = O.Layer.from_inputs(self.inp, self.scaling)
        gh, gw = O.experts_backward(self.k, layer, x.float(), idx, w, g.float(), experts=list(range(self.E)))
        z = lambda t, like: torch.zeros_like(like) if t is None else t
        grads = {"dA_g": z(layer.gate.grad_A, layer.gate.A), "dB_g": z(layer.gate.grad_B, layer.gate.B),
                 "dA_u": z(layer.up.grad_A, layer.up.A), "dB_u": z(layer.up.grad_B, layer.up.B),
                 "dA_d": z(layer.down.grad_A, layer.down.A), "dB_d": z(layer.down.grad_B, layer.down.B)}
        return gh, gw, grads


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, cfg, bias_hot):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.set_num_threads(1)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        inp = make_layer(cfg)
        if bias_hot is not None:                       # steer every token to the first experts
            inp["router_b"] = torch.where(torch.arange(cfg.E) < bias_hot, 10.0, 0.0)
        x, g = inp["x"].float(), inp["g"].float()
        idx, w = O.route(x, inp["router_w"], inp["router_b"], cfg.k)
        want = {}
        k = O.MXFP4Checker("oracle")
        layer = O.Layer.from_inputs(inp, cfg.scaling)
        want["out"] = O.experts_forward(k, layer, x, idx, w)
        want["grad_h"], want["grad_w"] = O.experts_backward(k, layer, x, idx, w, g)
        want_grads = {"dA_g": layer.gate.grad_A, "dB_g": layer.gate.grad_B, "dA_u": layer.up.grad_A,
                      "dB_u": layer.up.grad_B, "dA_d": layer.down.grad_A, "dB_d": layer.down.grad_B}

        local_inp, lo, hi = EPO.split_experts(inp, cfg.E, world, rank)
        assert (lo, hi - lo) == experts_of_rank(cfg.E, world, rank)
        ep = ExpertParallelLayer(OracleLocalLayer(local_inp, hi - lo, cfg.scaling), cfg.E, ops=EPO.OracleEPOps())
        # tokens are data-parallel: contiguous, possibly uneven, slices
        bounds = [(cfg.T * r) // world for r in range(world + 1)]
        t0, t1 = bounds[rank], bounds[rank + 1]
        out = ep.forward(x[t0:t1], idx[t0:t1], w[t0:t1])
        grad_h, grad_w, grads = ep.backward(g[t0:t1])

        # out and grad_h come back as fp16 rows with a power-of-two row scale (2^-11 relative
        # rounding of each rank's partial); grad_w and the LoRA gradients stay fp32
        assert O.rel_l2(out, want["out"][t0:t1]) < 1e-3
        assert O.rel_l2(grad_h, want["grad_h"][t0:t1]) < 1e-3
        assert O.rel_l2(grad_w, want["grad_w"][t0:t1]) < 1e-6
        for name, t in want_grads.items():
            assert O.rel_l2(grads[name], t) < 1e-5, name
        # the rows this rank received: one per (token anywhere, owning rank) pair
        assert ep._ctx["R"] == EPO.expected_counts(idx, cfg.E, world)[rank]
        if bias_hot is not None and rank == world - 1:
            assert ep._ctx["R"] == 0                    # nothing routed here: the empty path ran
    finally:
        dist.destroy_process_group()


CFG = LayerConfig(d=256, f=128, E=8, k=2, T=21, r=4, alpha=8, x_dtype="f32")


@pytest.mark.parametrize("world,cfg,bias_hot", [
    (2, CFG, None),
    (3, CFG, None),                                                   # 3/3/2 experts, 7 tokens each
    (2, LayerConfig(d=256, f=128, E=6, k=3, T=10, r=4, alpha=8, x_dtype="f32"), None),
    (2, CFG, 3),                                                      # rank 1 receives no rows
])
def test_expert_parallel_matches_single_process(world, cfg, bias_hot):
    O.build()
    mp.start_processes(_rank_main, args=(world, _free_port(), cfg, bias_hot), nprocs=world, start_method="spawn")


def test_oracle_plan_layout():
    idx = torch.tensor([[0, 5], [3, 1], [7, 6], [2, 4], [6, 7]])
    w = torch.rand(5, 2)
    counts, pos, tok, sidx, sw = EPO.OracleEPOps().plan(idx, w, E=8, n=2)
    # rank 0 owns 0..3, rank 1 owns 4..7
    assert counts.tolist() == [3, 4, 0]
    assert tok.tolist() == [0, 1, 3, 0, 2, 3, 4]
    assert pos.tolist() == [[0, 3], [1, -1], [-1, 4], [2, 5], [-1, 6]]
    assert sidx.tolist() == [[0, -1], [3, 1], [2, -1], [-1, 1], [3, 2], [-1, 0], [2, 3]]
    assert float(sw[1, 0]) == float(w[1, 0]) and float(sw[0, 1]) == 0.0
    bad = torch.tensor([[0, 8]])
    assert EPO.OracleEPOps().plan(bad, torch.ones(1, 2), E=8, n=2)[0].tolist() == [1, 0, 1]


def test_experts_of_rank_blocks():
    for E, n in [(896, 8), (896, 2), (10, 4), (8, 3), (5, 5)]:
        blocks = [experts_of_rank(E, n, r) for r in range(n)]
        assert blocks[0][0] == 0 and sum(c for _, c in blocks) == E
        for r, (lo, c) in enumerate(blocks):
            assert all((e * n) // E == r for e in range(lo, lo + c))


def test_c_abi_expert_blocks_match():
    import ctypes
    from lazylora_b200 import _lib as L
    lib = L.load()
    lo, cnt = ctypes.c_int(), ctypes.c_int()
    for E, n in [(896, 8), (10, 4), (8, 3)]:
        for r in range(n):
            assert lib.ll_ep_experts_of_rank(E, n, r, ctypes.byref(lo), ctypes.byref(cnt)) == 0
            assert (lo.value, cnt.value) == experts_of_rank(E, n, r)
    assert lib.ll_ep_experts_of_rank(8, 2, 2, ctypes.byref(lo), ctypes.byref(cnt)) != 0


def _bad_id_main(rank, world, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        cfg = CFG
        inp = make_layer(cfg)
        local_inp, lo, hi = EPO.split_experts(inp, cfg.E, world, rank)
        ep = ExpertParallelLayer(OracleLocalLayer(local_inp, hi - lo, cfg.scaling), cfg.E, ops=EPO.OracleEPOps())
        idx = torch.tensor([[0, 5], [1, 6]])
        if rank == 1:
            idx[1, 1] = cfg.E                    # one bad id, on one rank only
        with pytest.raises(ValueError, match="outside"):
            ep.forward(inp["x"][:2].float(), idx, torch.ones(2, 2))
    finally:
        dist.destroy_process_group()


def test_bad_expert_id_fails_every_rank():
    mp.start_processes(_bad_id_main, args=(2, _free_port()), nprocs=2, start_method="spawn")


def test_packed_rows_round_trip():
    """The packed return rows: fp16 with a power-of-two row scale, exact for values fp16 holds,
    2^-11 relative otherwise; zero rows and rows of very small or large values survive."""
    ops = EPO.OracleEPOps()
    g = torch.Generator().manual_seed(2)
    part = torch.randn(5, 64, generator=g) * torch.tensor([1e-6, 1.0, 3e4, 1e9, 0.0]).unsqueeze(1)
    packed = ops.pack_rows(part)
    assert packed.shape == (5, 64 // 2 + 4) and packed.dtype == torch.int32
    pos = torch.tensor([[0, 3], [1, -1], [2, 4]], dtype=torch.int32)
    got = ops.combine_packed(packed, pos, 3, 64)
    want = torch.stack([part[0] + part[3], part[1], part[2] + part[4]])
    assert O.rel_l2(got, want) < 1e-3
    exact = torch.tensor([[1.0, -2.0, 0.5, 0.0] * 16])
    assert torch.equal(ops.combine_packed(ops.pack_rows(exact), torch.tensor([[0]], dtype=torch.int32), 1, 64), exact)
