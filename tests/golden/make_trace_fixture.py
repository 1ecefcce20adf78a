"""
Make tests/golden/routing_traces.npz: real routing decisions (expert ids and combining
weights, nothing else) of Kimi K3 on five prompts, from the reference's recorded expert traces
(evidence/traces/*/trace.bin). Run on a machine that has the reference tree:
    python tests/golden/make_trace_fixture.py <path of the reference tree>
The fixture travels with the repository.

trace.bin format (lazy_lora/monitor/trace.py:10-13): records of int32 layer, int32 N, int32 K,
int16[N*K] expert ids (row-major), float16[N*K] combining weights. Kept: layers 1, 31, 61, 91
of every trace (N = 111..264 tokens, K = 16 of 896 experts).
"""
import glob
import os
import struct
import sys

import numpy as np

KEEP = (1, 31, 61, 91)


def read_trace_bin(path):
    out = {}
    with open(path, "rb") as f:
        while True:
            head = f.read(12)
            if len(head) < 12:
                break
            layer, n, k = struct.unpack("<iii", head)
            idx = np.frombuffer(f.read(n * k * 2), dtype=np.int16).reshape(n, k)
            w = np.frombuffer(f.read(n * k * 2), dtype=np.float16).reshape(n, k)
            out[layer] = (idx.copy(), w.copy())
    return out


def main(ref_root):
    arrays = {}
    for d in sorted(glob.glob(os.path.join(ref_root, "evidence", "traces", "*"))):
        name = os.path.basename(d).split("_L")[0]
        layers = read_trace_bin(os.path.join(d, "trace.bin"))
        for layer in KEEP:
            idx, w = layers[layer]
            arrays[f"{name}/{layer}/idx"] = idx
            arrays[f"{name}/{layer}/w"] = w
    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "routing_traces.npz")
    np.savez_compressed(out, **arrays)
    print(out, len(arrays) // 2, "routings")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: python tests/golden/make_trace_fixture.py <path of the reference tree>")
    main(sys.argv[1])
