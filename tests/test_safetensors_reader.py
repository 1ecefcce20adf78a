"""
CPU tests of the checkpoint reader that feeds the pinned-host expert stage: header parsing and
name resolution as the reference's SafetensorsIndex (lazy_lora/streaming/mmap_loader.py:64-133,
194-205), bit-exact parallel reads of a layer's expert tensors into [E, rows, cols] stacks,
and the failure paths (unreadable shards are listed, a missing tensor or a range past the end
of its file is an error, never silent zeros).
"""
import os
import struct

import pytest
import torch

from lazylora_b200._lib import LLError
from lazylora_b200.streaming.safetensors_reader import (SafetensorsIndex, read_layer_experts,
                                                        write_layer_experts)


def _stacks(E, d=256, f=128, seed=0):
    g = torch.Generator().manual_seed(seed)
    rnd = lambda *s: torch.randint(0, 256, s, dtype=torch.uint8, generator=g)
    return {"w1p": rnd(E, f, d // 2), "w1s": rnd(E, f, d // 32), "w3p": rnd(E, f, d // 2), "w3s": rnd(E, f, d // 32),
            "w2p": rnd(E, d, f // 2), "w2s": rnd(E, d, f // 32)}


def _checkpoint(tmp_path, E=6, layer=3):
    st = _stacks(E)
    half = E // 2
    first = {k: v[:half] for k, v in st.items()}
    second = {k: v[half:] for k, v in st.items()}
    write_layer_experts(str(tmp_path / "model-00001.safetensors"), layer, first, range(half))
    write_layer_experts(str(tmp_path / "model-00002.safetensors"), layer, second, range(half, E),
                        prefix="language_model.")
    return st


def test_reads_layer_experts_bit_exact(tmp_path):
    st = _checkpoint(tmp_path)
    idx = SafetensorsIndex(str(tmp_path))
    assert not idx.bad_shards
    order = [4, 0, 2, 5]
    got, nbytes = read_layer_experts(idx, 3, order, pin=False, threads=3)
    for k in st:
        assert torch.equal(got[k], st[k][order]), k
    assert nbytes == sum(st[k][0].numel() for k in st) * len(order)
    # into supplied stacks
    out = {k: torch.zeros_like(v[:2]) for k, v in st.items()}
    read_layer_experts(idx, 3, [1, 3], out=out, pin=False)
    for k in st:
        assert torch.equal(out[k], st[k][[1, 3]]), k


def test_bad_shards_and_missing_tensors(tmp_path):
    _checkpoint(tmp_path)
    (tmp_path / "empty.safetensors").write_bytes(b"")
    (tmp_path / "short.safetensors").write_bytes(struct.pack("<Q", 1000) + b"{}")
    idx = SafetensorsIndex(str(tmp_path))
    assert sorted(idx.bad_shards) == ["empty.safetensors", "short.safetensors"]
    with pytest.raises(KeyError):
        read_layer_experts(idx, 3, [7], pin=False)          # no such expert
    with pytest.raises(KeyError):
        read_layer_experts(idx, 4, [0], pin=False)          # no such layer


def test_range_past_end_of_file_is_an_error(tmp_path):
    _checkpoint(tmp_path)
    idx = SafetensorsIndex(str(tmp_path))
    p = tmp_path / "model-00002.safetensors"
    size = os.path.getsize(p)
    with open(p, "r+b") as f:                               # truncated after indexing
        f.truncate(size - 100)
    with pytest.raises(LLError) as ei:
        read_layer_experts(idx, 3, [0, 1, 2, 3, 4, 5], pin=False, retries=0)
    assert "ends before the range" in str(ei.value)
    os.remove(p)
    with pytest.raises(LLError):
        read_layer_experts(idx, 3, [5], pin=False, retries=0)


def test_lowest_failing_range_is_reported(tmp_path):
    """With several failing ranges and many worker threads, ll_pread_batch reports the lowest
    failing index every time (ranges are handed out in index order and every range below a
    failure is finished before the batch returns)."""
    import ctypes
    from lazylora_b200 import _lib as L
    lib = L.load()
    p = tmp_path / "blob.bin"
    p.write_bytes(bytes(range(256)) * 64)                   # 16 KB
    n = 64
    bufs = [ctypes.create_string_buffer(256) for _ in range(n)]
    offs = [i * 256 for i in range(n)]
    for bad in (5, 17, 40):                                 # these ranges start past the end
        offs[bad] = 1 << 20
    paths = (ctypes.c_char_p * n)(*[str(p).encode()] * n)
    o = (ctypes.c_int64 * n)(*offs)
    sz = (ctypes.c_int64 * n)(*[256] * n)
    dst = (ctypes.c_void_p * n)(*[ctypes.addressof(b) for b in bufs])
    for _ in range(20):
        done, failed = ctypes.c_int64(0), ctypes.c_int(-2)
        rc = lib.ll_pread_batch(n, paths, o, sz, dst, 16, 0, 0, ctypes.byref(done), ctypes.byref(failed))
        assert rc == 7 and failed.value == 5                # LL_ERR_IO, the lowest failing range
    for i in range(5):                                      # every range below it was read
        assert bufs[i].raw == bytes(range(256))
