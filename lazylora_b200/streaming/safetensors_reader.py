"""
Routed-expert tensors of a safetensors checkpoint into the pinned-host stage of the expert
streamer, read in parallel.

The reference indexes every shard's JSON header (lazy_lora/streaming/mmap_loader.py:64-133:
an 8-byte little-endian header length, the header, then the data; a tensor's bytes are
[8 + header_len + data_offsets[0], 8 + header_len + data_offsets[1])) and reads each expert
tensor with its own os.pread (mmap_loader.py:260-341), by the names
`model.layers.{L}.block_sparse_moe.experts.{e}.w{1,2,3}.weight_packed / weight_scale`
(expert_streamer.py:230-238), resolving the "model." / "language_model." prefixes
(mmap_loader.py:194-205). Here `SafetensorsIndex` parses the same headers, and
`read_layer_experts` reads all six tensors of every requested expert of a layer with one
batched, multi-threaded pread (ll_pread_batch, same EIO retry policy) straight into
[E, rows, cols] host stacks — the layout HostExpertStore keeps and the GPU kernels take — so a
layer's experts land in pinned memory without a Python-level copy per tensor.
"""
import ctypes
import json
import os
import struct
from typing import Dict, List, Optional, Sequence, Tuple

import torch

from .. import _lib as L

DTYPES = {"U8": torch.uint8, "I8": torch.int8, "F16": torch.float16, "BF16": torch.bfloat16,
          "F32": torch.float32, "I32": torch.int32, "I64": torch.int64}
STACK_NAMES = {"w1p": ("w1", "weight_packed"), "w1s": ("w1", "weight_scale"),
               "w3p": ("w3", "weight_packed"), "w3s": ("w3", "weight_scale"),
               "w2p": ("w2", "weight_packed"), "w2s": ("w2", "weight_scale")}


class SafetensorsIndex:
    """name -> (shard path, start, end, shape, dtype) over every *.safetensors in a directory.
    Shards whose header cannot be read (empty, truncated, oversized or bad JSON) are listed in
    `bad_shards` and contribute no tensors."""

    def __init__(self, model_dir: str):
        self.model_dir = model_dir
        self.tensors: Dict[str, Tuple[str, int, int, List[int], str]] = {}
        self.bad_shards: List[str] = []
        for shard in sorted(f for f in os.listdir(model_dir) if f.endswith(".safetensors")):
            path = os.path.join(model_dir, shard)
            try:
                with open(path, "rb") as f:
                    head = f.read(8)
                    if len(head) < 8:
                        raise ValueError("short header length")
                    n = struct.unpack("<Q", head)[0]
                    if n > 100 * 1024 * 1024:
                        raise ValueError("header too large")
                    raw = f.read(n)
                    if len(raw) < n:
                        raise ValueError("short header")
                    header = json.loads(raw.decode("utf-8"))
                size = os.path.getsize(path)
                base = 8 + n
                for name, info in header.items():
                    if name == "__metadata__":
                        continue
                    a, b = info["data_offsets"]
                    if base + b > size:
                        raise ValueError(f"{name} runs past the end of the file")
                    self.tensors[name] = (path, base + a, base + b, list(info["shape"]), info["dtype"])
            except (OSError, ValueError, KeyError, json.JSONDecodeError, UnicodeDecodeError):
                self.bad_shards.append(shard)

    def resolve(self, name: str) -> Optional[str]:
        """The stored name for `name`, trying the reference's prefixes (mmap_loader.py:194-205)."""
        if name in self.tensors:
            return name
        for prefix in ("language_model.", "model.", "language_model.model."):
            if prefix + name in self.tensors:
                return prefix + name
        if name.startswith("model.") and "language_model." + name in self.tensors:
            return "language_model." + name
        return None

    def location(self, name: str):
        key = self.resolve(name)
        if key is None:
            raise KeyError(f"{name} is not in the checkpoint index")
        return self.tensors[key]


def expert_tensor_name(layer_idx: int, expert_idx: int, which: str) -> str:
    w, kind = STACK_NAMES[which]
    return f"model.layers.{layer_idx}.block_sparse_moe.experts.{expert_idx}.{w}.{kind}"


def read_layer_experts(index: SafetensorsIndex, layer_idx: int, expert_ids: Sequence[int],
                       out: Optional[Dict[str, torch.Tensor]] = None, pin: bool = True, threads: int = 16,
                       retries: int = 12, retry_ms: int = 2000) -> Tuple[Dict[str, torch.Tensor], int]:
    """Stacks {w1p, w1s, w3p, w3s, w2p, w2s} of shape [len(expert_ids), rows, cols] holding the
    experts in the given order, read with one parallel batch. `out` may supply the stacks
    (e.g. a streamer's pinned staging); otherwise they are allocated (pinned when `pin`).
    Returns (stacks, bytes read)."""
    ids = [int(e) for e in expert_ids]
    if not ids:
        raise ValueError("no experts requested")
    locs = {w: [index.location(expert_tensor_name(layer_idx, e, w)) for e in ids] for w in STACK_NAMES}
    stacks = {} if out is None else out
    for w, lst in locs.items():
        shape, dt = lst[0][3], lst[0][4]
        if any(l[3] != shape or l[4] != dt for l in lst):
            raise ValueError(f"{w}: experts of layer {layer_idx} differ in shape or dtype")
        if dt not in DTYPES:
            raise ValueError(f"{w}: unsupported dtype {dt}")
        want = (len(ids),) + tuple(shape)
        if w in stacks:
            t = stacks[w]
            if tuple(t.shape) != want or t.dtype != DTYPES[dt] or t.device.type != "cpu" or not t.is_contiguous():
                raise ValueError(f"{w}: supplied stack must be a contiguous CPU tensor {want} {DTYPES[dt]}")
        else:
            t = torch.empty(want, dtype=DTYPES[dt], pin_memory=pin and torch.cuda.is_available())
            stacks[w] = t
    paths, offs, sizes, dsts = [], [], [], []
    for w, lst in locs.items():
        t = stacks[w]
        per = t[0].numel() * t.element_size()
        for j, (path, a, b, _shape, _dt) in enumerate(lst):
            if b - a != per:
                raise ValueError(f"{w} of expert {ids[j]}: {b - a} bytes stored, {per} expected")
            paths.append(path.encode())
            offs.append(a)
            sizes.append(b - a)
            dsts.append(t.data_ptr() + j * per)
    n = len(paths)
    lib = L.load(build_if_needed=False)
    done, bad = ctypes.c_int64(0), ctypes.c_int(-1)
    rc = lib.ll_pread_batch(n, (ctypes.c_char_p * n)(*paths), (ctypes.c_int64 * n)(*offs),
                            (ctypes.c_int64 * n)(*sizes), (ctypes.c_void_p * n)(*dsts), threads, retries,
                            retry_ms, ctypes.byref(done), ctypes.byref(bad))
    L.check(rc, "ll_pread_batch")
    return stacks, int(done.value)


def write_layer_experts(path: str, layer_idx: int, stacks: Dict[str, torch.Tensor], expert_ids: Sequence[int],
                        prefix: str = "") -> None:
    """Write experts of one layer as a safetensors shard with the checkpoint's names (a helper
    for tests and synthetic checkpoints; not a general safetensors writer)."""
    rev = {v: k for k, v in DTYPES.items()}
    header, blobs, off = {}, [], 0
    for j, e in enumerate(expert_ids):
        for w in STACK_NAMES:
            t = stacks[w][j].contiguous()
            b = t.view(torch.uint8).numpy().tobytes() if t.dtype != torch.bfloat16 else \
                t.view(torch.int16).numpy().tobytes()
            header[prefix + expert_tensor_name(layer_idx, e, w)] = {
                "dtype": rev[t.dtype], "shape": list(t.shape), "data_offsets": [off, off + len(b)]}
            blobs.append(b)
            off += len(b)
    raw = json.dumps(header).encode("utf-8")
    raw += b" " * ((8 - len(raw) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(raw)))
        f.write(raw)
        for b in blobs:
            f.write(b)
