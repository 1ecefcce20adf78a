"""
Regenerate the golden vectors in this folder from the reference implementation itself.

Run from the repository root on a machine that has the reference tree:
    python tests/golden/make_golden.py --ref <path of the reference tree>

What it writes:
  ref_<case>.npz       outputs of the reference's own routed-expert code on the seeded inputs
                       of lazylora_b200.synthetic.CONFIGS[<case>]: router indices / weights
                       (KimiK3MoERouter.forward, lazy_lora/core/moe_router.py:55-100), the
                       per-expert row order (lazy_trainer.py:823-827), the forward sum
                       (LazyLoRATrainer._routed_experts_forward, lazy_trainer.py:806-834) and
                       the backward (grad_h, grad_w and the six LoRA gradients,
                       _routed_experts_backward, lazy_trainer.py:836-880). The MXFP4 GEMMs
                       run in the reference's C kernel (lazy_lora/native/mxfp4_gemm.c) built
                       from source by oracle/Makefile; at K > 4096 its `gemm` is summed over
                       K chunks of 3584 because its stack tile stops at 4096 (mxfp4_gemm.c:72).
  fx_router.npz, fx_situ_glu.npz, fx_moe.npz
                       the reference's vendored op fixtures for this path
                       (tests/fixtures/ops/{router,situ_glu,moe}.json, recorded by the
                       independent kimi-k3-in-c implementation, Apache-2.0), converted to
                       npz unchanged.
  dequant_edges.npz    reference C dequant of a block with every code and the scale bytes
                       0, 1, 104, 117..121, 140, 141, 252, 253, 254, 255.
Inputs are not stored: both sides regenerate them from the seed.
"""
import argparse
import ctypes
import json
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from lazylora_b200.synthetic import CONFIGS, make_layer  # noqa: E402

CASES = ("tiny", "small", "k3", "c0")


def _fixture(path, out_path):
    with open(path, encoding="utf-8") as fh:
        fx = json.load(fh)
    arrays = {}
    for key, val in fx.items():
        if isinstance(val, dict) and "data" in val:
            arrays[key] = np.asarray(val["data"], dtype=np.float32).reshape(val["shape"])
        elif isinstance(val, (int, float)):
            arrays[key] = np.asarray(val)
        elif isinstance(val, list) and all(isinstance(v, (int, float)) for v in val):
            arrays[key] = np.asarray(val)
    np.savez_compressed(out_path, **arrays)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="path of the reference tree")
    ap.add_argument("--cases", default=",".join(CASES))
    args = ap.parse_args()
    sys.path.insert(0, args.ref)
    os.environ.setdefault("LAZYLORA_ALLOW_SYNTHETIC", "1")

    import subprocess
    subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), f"REF_ROOT={args.ref}"], check=True)
    ref_so = os.path.join(ROOT, "oracle", "_ref", "libmxfp4_ref.so")

    import lazy_lora.native as native
    from lazy_lora.core.lora_layer import LazyLoRALinear
    from lazy_lora.core.moe_router import KimiK3MoERouter
    from lazy_lora.streaming.expert_streamer import ExpertWeightBundle
    from lazy_lora.trainer import lazy_trainer as LT

    class ChunkedKernel(native.MXFP4Kernel):
        """The reference kernel, with gemm summed over K chunks of 3584 when K > 4096."""

        def gemm(self, x, packed, scales):
            K = packed.shape[1] * 2
            if K <= 4096:
                return super().gemm(x, packed, scales)
            y = None
            for k0 in range(0, K, 3584):
                k1 = min(K, k0 + 3584)
                part = super().gemm(x[:, k0:k1].contiguous(), packed[:, k0 // 2:k1 // 2].contiguous(),
                                    scales[:, k0 // 32:k1 // 32].contiguous())
                y = part if y is None else y + part
            return y

    native._lib = ChunkedKernel(ctypes.CDLL(ref_so))
    native._tried = True
    torch.set_num_threads(os.cpu_count() or 1)

    # ---- the reference's vendored fixtures for this path
    fxdir = os.path.join(args.ref, "tests", "fixtures", "ops")
    for name in ("router", "situ_glu", "moe"):
        _fixture(os.path.join(fxdir, f"{name}.json"), os.path.join(HERE, f"fx_{name}.npz"))

    # ---- dequant edge block through the reference C kernel
    codes = np.arange(64, dtype=np.uint8) % 16
    packed_rows, scale_rows = [], []
    edge_scales = [0, 1, 104, 117, 118, 119, 120, 121, 140, 141, 252, 253, 254, 255]
    for b in edge_scales:
        packed_rows.append((codes[0::2] | (codes[1::2] << 4)).astype(np.uint8))
        scale_rows.append(np.asarray([b, (b + 7) % 256], dtype=np.uint8))
    packed = torch.from_numpy(np.stack(packed_rows))
    scales = torch.from_numpy(np.stack(scale_rows))
    deq = native._lib.dequant(packed, scales)
    np.savez_compressed(os.path.join(HERE, "dequant_edges.npz"), packed=packed.numpy(),
                        scales=scales.numpy(), out=deq.numpy())

    # ---- whole routed-expert layer through the reference's own trainer methods
    for case in args.cases.split(","):
        cfg = CONFIGS[case]
        inp = make_layer(cfg)
        x = inp["x"].float()
        router = KimiK3MoERouter(hidden_size=cfg.d, num_experts=cfg.E, top_k=cfg.k)
        idx, w = router.forward(x, weight=inp["router_w"], bias=inp["router_b"])
        active = router.get_active_expert_set(idx)

        bundle = types.SimpleNamespace()
        for name, (i_f, o_f, A, B) in {
            "gate_lora": (cfg.d, cfg.f, inp["A_g"], inp["B_g"]),
            "up_lora": (cfg.d, cfg.f, inp["A_u"], inp["B_u"]),
            "down_lora": (cfg.f, cfg.d, inp["A_d"], inp["B_d"]),
        }.items():
            mod = LazyLoRALinear(i_f, o_f, r=cfg.r, lora_alpha=cfg.alpha)
            with torch.no_grad():
                mod.lora_A.copy_(A)
                mod.lora_B.copy_(B)
            setattr(bundle, name, mod)

        class Streamer:
            def stream_experts(self, layer_idx, ids, depth=2):
                for e in ids:
                    yield e, ExpertWeightBundle(
                        e, gate_packed=inp["w1p"][e], gate_scale=inp["w1s"][e],
                        up_packed=inp["w3p"][e], up_scale=inp["w3s"][e],
                        down_packed=inp["w2p"][e], down_scale=inp["w2s"][e])

        st = types.SimpleNamespace(gpu=False, _prof={}, expert_streamer=Streamer())
        for meth in ("_expert_matrices", "_expert_forward", "_expert_dx"):
            setattr(st, meth, types.MethodType(getattr(LT.LazyLoRATrainer, meth), st))
        out = LT.LazyLoRATrainer._routed_experts_forward(st, 0, bundle, x, idx, w, active)
        gh, gw = LT.LazyLoRATrainer._routed_experts_backward(st, 0, bundle, x, idx, w, active, inp["g"].float())

        # per-expert row order, exactly as the expert loop gathers rows
        offs, toks, slots = [0], [], []
        for e in range(cfg.E):
            mask = idx == e
            rows = mask.any(dim=-1).nonzero(as_tuple=False).squeeze(-1)
            offs.append(offs[-1] + rows.numel())
            toks.append(rows)
            slots.append(mask[rows].to(torch.int64).argmax(dim=-1))
        res = dict(idx=idx, w=w, offsets=torch.tensor(offs), perm_token=torch.cat(toks),
                   perm_slot=torch.cat(slots), out=out, grad_h=gh, grad_w=gw,
                   dA_g=bundle.gate_lora.lora_A.grad, dB_g=bundle.gate_lora.lora_B.grad,
                   dA_u=bundle.up_lora.lora_A.grad, dB_u=bundle.up_lora.lora_B.grad,
                   dA_d=bundle.down_lora.lora_A.grad, dB_d=bundle.down_lora.lora_B.grad)
        np.savez_compressed(os.path.join(HERE, f"ref_{case}.npz"),
                            **{k: v.detach().cpu().numpy() for k, v in res.items()})
        print(f"{case}: active {len(active)} experts, |out| {out.norm():.4f}, |grad_h| {gh.norm():.4f}")


if __name__ == "__main__":
    main()
