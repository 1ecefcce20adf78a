"""
GPU checks of the expert-parallel path.

  * one GPU: the CUDA index kernels (ll_ep_plan, ll_ep_gather_rows, ll_ep_combine,
    ll_ep_pack_rows, ll_ep_combine_packed, ll_ep_combine_slots) bit-exact against their CPU
    restatement (oracle/ep_oracle.py), at
    the full-width shape (T=1024, k=8, E=896, n=8) and ragged ones, invalid ids included;
  * two GPUs: ExpertParallelLayer over NCCL, each rank holding its block of experts and half
    of the tokens, against the single-process reference-algorithm oracle over all tokens and
    all experts (relative L2 2e-3 on out, grad_h, grad_w and the all-reduced LoRA grads).
"""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from lazylora_b200.synthetic import CONFIGS, make_layer
from oracle import ep_oracle as EPO
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu
TOL = 2e-3


@pytest.mark.parametrize("T,k,E,n,bad", [(1024, 8, 896, 8, 0), (1024, 8, 896, 2, 0), (37, 3, 10, 4, 0),
                                         (300, 8, 896, 8, 5), (1, 1, 5, 5, 0), (0, 2, 8, 2, 0)])
def test_plan_and_combines_bit_exact(T, k, E, n, bad):
    from lazylora_b200.trainer.expert_parallel import CudaEPOps
    gen = torch.Generator().manual_seed(T * 31 + n)
    idx = torch.stack([torch.randperm(E, generator=gen)[:k] for _ in range(T)]) if T else \
        torch.zeros((0, k), dtype=torch.int64)
    if bad:
        flat = idx.view(-1)
        flat[torch.randperm(flat.numel(), generator=gen)[:bad]] = E + 3
    w = torch.rand((T, k), generator=gen)
    ref = EPO.OracleEPOps()
    got = CudaEPOps()
    rc, rpos, rtok, ridx, rw = ref.plan(idx, w, E, n)
    gc, gpos, gtok, gidx, gw = got.plan(idx.cuda(), w.cuda(), E, n)
    S = int(rc[:n].sum())
    assert gc.cpu().tolist() == rc.tolist()
    assert torch.equal(gpos.cpu(), rpos)
    assert torch.equal(gtok[:S].cpu(), rtok[:S])
    assert torch.equal(gidx[:S].cpu(), ridx.reshape(-1, k)[:S])
    assert torch.equal(gw[:S].cpu(), rw.reshape(-1, k)[:S])
    d = 64
    x = torch.randn(T, d, generator=gen)
    assert torch.equal(got.gather_rows(x.cuda().to(torch.bfloat16), gtok, S).cpu(),
                       ref.gather_rows(x.to(torch.bfloat16), rtok, S))
    part = torch.randn(S, d, generator=gen)
    assert torch.equal(got.combine(part.cuda(), gpos, T, d).cpu(), ref.combine(part, rpos, T, d))
    # the packed return rows: same bits as the restatement, rounding included
    part[:1] *= 1e6
    gp, rp = got.pack_rows(part.cuda()), ref.pack_rows(part)
    assert torch.equal(gp.cpu(), rp)
    assert torch.equal(got.combine_packed(gp, gpos, T, d).cpu(), ref.combine_packed(rp, rpos, T, d))
    pw = torch.randn(S, k, generator=gen)
    assert torch.equal(got.combine_slots(pw.cuda(), gpos, idx.cuda(), E).cpu(), ref.combine_slots(pw, rpos, idx, E))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _local_layer(local_inp, cfg, streamed):
    """The rank's block of experts: resident, or (streamed) held in pinned host memory and
    streamed into HBM three experts at a time for every forward and backward."""
    from lazylora_b200.trainer.routed_experts import RoutedExpertsLayer
    if not streamed:
        return RoutedExpertsLayer.from_inputs(local_inp, cfg.scaling)
    from lazylora_b200.trainer.expert_streamer import ExpertStreamer, HostExpertStore, StreamedLocalExperts
    store = HostExpertStore()
    store.add_layer(0, {n: local_inp[n] for n in ("w1p", "w1s", "w3p", "w3s", "w2p", "w2s")})
    lora = {n: local_inp[n].cuda() for n in ("A_g", "B_g", "A_u", "B_u", "A_d", "B_d")}
    return StreamedLocalExperts(ExpertStreamer(store, lora, cfg.scaling, group_experts=3), 0)


def _rank_main(rank, world, port, case, streamed=False):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        from lazylora_b200.trainer.expert_parallel import ExpertParallelLayer
        cfg = CONFIGS[case]
        inp = make_layer(cfg)
        x, g = inp["x"], inp["g"]
        idx, w = O.route(x.float(), inp["router_w"], inp["router_b"], cfg.k)
        local_inp, lo, hi = EPO.split_experts(inp, cfg.E, world, rank)
        ep = ExpertParallelLayer(_local_layer(local_inp, cfg, streamed), cfg.E)
        bounds = [(cfg.T * r) // world for r in range(world + 1)]
        t0, t1 = bounds[rank], bounds[rank + 1]
        xd = x[t0:t1].cuda()
        gd = g[t0:t1].cuda()
        if cfg.x_dtype == "bf16":
            xd, gd = xd.to(torch.bfloat16), gd.to(torch.bfloat16)
        got = {}
        got["out"] = ep.forward(xd, idx[t0:t1].cuda(), w[t0:t1].cuda())
        got["grad_h"], got["grad_w"], grads = ep.backward(gd)
        got.update(grads)
        if ep._ctx["R"] and not streamed:
            ep.local.check_status(ep._ctx["R"], cfg.k)
        # the single-process reference algorithm over all tokens and all experts
        layer = O.Layer.from_inputs(inp, cfg.scaling)
        kk = O.MXFP4Checker("oracle")
        want = {"out": O.experts_forward(kk, layer, x.float(), idx, w)}
        want["grad_h"], want["grad_w"] = O.experts_backward(kk, layer, x.float(), idx, w, g.float())
        for key in ("out", "grad_h", "grad_w"):
            err = O.rel_l2(got[key].cpu(), want[key][t0:t1])
            assert err <= TOL, f"{case} rank {rank} {key}: {err:.3e}"
        for key, t in (("dA_g", layer.gate.grad_A), ("dB_g", layer.gate.grad_B), ("dA_u", layer.up.grad_A),
                       ("dB_u", layer.up.grad_B), ("dA_d", layer.down.grad_A), ("dB_d", layer.down.grad_B)):
            err = O.rel_l2(got[key].cpu(), t)
            assert err <= TOL, f"{case} rank {rank} {key}: {err:.3e}"
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("case", ["small", "c0"])
def test_expert_parallel_two_gpus_matches_oracle(case):
    O.build()
    mp.start_processes(_rank_main, args=(2, _free_port(), case), nprocs=2, start_method="spawn")


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_expert_parallel_two_gpus_streamed_local_experts():
    """configs[4]'s composition: each rank streams only its own block of experts from pinned
    host memory (StreamedLocalExperts as the EP layer's local layer), against the oracle."""
    O.build()
    mp.start_processes(_rank_main, args=(2, _free_port(), "small", True), nprocs=2, start_method="spawn")


def test_expert_parallel_one_rank_streamed_local_experts():
    """The same composition on one GPU (a one-rank NCCL group): the exchanges are identities,
    the streamed local experts are the whole layer."""
    O.build()
    mp.start_processes(_rank_main, args=(1, _free_port(), "c0", True), nprocs=1, start_method="spawn")
