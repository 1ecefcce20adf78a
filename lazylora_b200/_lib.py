"""
ctypes binding of liblazylora_b200.so (the C ABI in include/lazylora_b200.h).

There is no fallback: if the library is missing or the device is not a B200, every entry
point raises. `load()` builds the library in-tree first when nvcc is available and the
sources are newer than the library.
"""
import ctypes
import os
import threading

import torch

from . import build as _build

_lock = threading.Lock()
_lib = None

c_int, c_float, c_size_t, c_void_p, c_int64 = ctypes.c_int, ctypes.c_float, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_int64

STATUS = {0: "ok", 1: "invalid argument", 2: "CUDA error", 3: "device-side wait timed out",
          4: "workspace too small", 5: "value out of range", 6: "device is not sm_100"}


class LLError(RuntimeError):
    def __init__(self, code, where, detail=""):
        self.code = code
        super().__init__(f"{where}: {STATUS.get(code, code)} ({code}){': ' + detail if detail else ''}")


class MoELayerDesc(ctypes.Structure):
    """Mirror of ll_moe_layer."""
    _fields_ = [
        ("d", c_int), ("f", c_int), ("E", c_int), ("r", c_int), ("lora_scaling", c_float),
        ("w1p", c_void_p), ("w1s", c_void_p), ("w3p", c_void_p), ("w3s", c_void_p),
        ("w2p", c_void_p), ("w2s", c_void_p),
        ("s13_stride", c_int64), ("s2_stride", c_int64),
        ("beta", c_void_p),
        ("A_g", c_void_p), ("B_g", c_void_p), ("A_u", c_void_p), ("B_u", c_void_p),
        ("A_d", c_void_p), ("B_d", c_void_p),
        ("w1t", c_void_p), ("w3t", c_void_p), ("w2t", c_void_p),
        ("s1t", c_void_p), ("s3t", c_void_p), ("s2t", c_void_p),
        ("rows_hint", c_int),
        ("w1sf", c_void_p), ("w3sf", c_void_p), ("w2sf", c_void_p),
    ]


_SIGS = {
    "ll_status_string": (ctypes.c_char_p, [c_int]),
    "ll_last_cuda_error": (ctypes.c_char_p, []),
    "ll_last_launch_count": (c_int, []),
    "ll_mxfp4_threads": (c_int, []),
    "ll_mxfp4_workspace_bytes": (c_size_t, [c_int, c_int, c_int]),
    "ll_mxfp4_sf_bytes": (c_size_t, [c_int, c_int, c_int]),
    "ll_mxfp4_gemm": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int64,
                              c_void_p, c_size_t, c_void_p]),
    "ll_mxfp4_gemm_t": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int64,
                                c_void_p, c_size_t, c_void_p]),
    "ll_mxfp4_gemm_noalloc": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int64,
                                      c_void_p]),
    "ll_mxfp4_dequant": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int64, c_int, c_void_p]),
    "ll_route_workspace_bytes": (c_size_t, [c_int, c_int, c_int]),
    "ll_route_topk": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_float,
                              c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
    "ll_route_prepare": (c_int, [c_void_p, c_int, c_int, c_void_p, c_void_p]),
    "ll_route_topk_prepared": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_float,
                                       c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
    "ll_route_select": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_float, c_void_p, c_void_p,
                                c_void_p]),
    "ll_moe_prepare": (c_int, [ctypes.POINTER(MoELayerDesc), c_void_p, c_void_p]),
    "ll_mxfp4_transposed_bytes": (c_size_t, [c_int, c_int, c_int, c_int]),
    "ll_moe_workspace_bytes": (c_size_t, [ctypes.POINTER(MoELayerDesc), c_int, c_int]),
    "ll_moe_forward": (c_int, [ctypes.POINTER(MoELayerDesc), c_int, c_int, c_void_p, c_int, c_void_p, c_void_p,
                               c_void_p, c_void_p, c_size_t, c_void_p]),
    "ll_moe_forward_rmsnorm": (c_int, [ctypes.POINTER(MoELayerDesc), c_int, c_int, c_void_p, c_int, c_void_p,
                                       c_void_p, c_void_p, ctypes.c_float, c_void_p, c_void_p, c_void_p, c_void_p,
                                       c_size_t, c_void_p]),
    "ll_moe_backward": (c_int, [ctypes.POINTER(MoELayerDesc), c_int, c_int, c_void_p, c_int, c_void_p, c_void_p,
                                c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
    "ll_moe_status": (c_int, [ctypes.POINTER(MoELayerDesc), c_int, c_int, c_void_p, c_void_p]),
    "ll_moe_permutation": (c_int, [ctypes.POINTER(MoELayerDesc), c_int, c_int, c_void_p, c_void_p, c_void_p,
                                   c_void_p, c_void_p]),
    "ll_ep_experts_of_rank": (c_int, [c_int, c_int, c_int, ctypes.POINTER(c_int), ctypes.POINTER(c_int)]),
    "ll_ep_plan": (c_int, [c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                           c_void_p, c_void_p]),
    "ll_ep_gather_rows": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int64, c_void_p]),
    "ll_ep_combine": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p]),
    "ll_ep_pack_rows": (c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p]),
    "ll_ep_combine_packed": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p]),
    "ll_ep_combine_slots": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p]),
    "ll_profile_gemm_events": (c_int, [ctypes.POINTER(c_void_p), c_int]),
    "ll_pread_batch": (c_int, [c_int, ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(c_int64),
                               ctypes.POINTER(c_int64), ctypes.POINTER(c_void_p), c_int, c_int, c_int,
                               ctypes.POINTER(c_int64), ctypes.POINTER(c_int)]),
    "ll_shared_glu_forward": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_float, c_int,
                                      c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p]),
    "ll_shared_glu_backward": (c_int, [c_void_p, c_void_p, c_void_p, c_float, c_void_p, c_void_p, c_int, c_int,
                                       c_int, c_void_p, c_void_p, c_void_p]),
    "ll_lora_down": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_int, c_int, c_int, c_float,
                             c_void_p, c_void_p, c_void_p, ctypes.c_size_t, c_void_p]),
    "ll_lora_outer": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_float, c_int, c_void_p, c_void_p,
                              ctypes.c_size_t, c_void_p]),
    "ll_lora_add_bf16": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_float, c_int,
                                 c_int, c_void_p, c_void_p]),
    "ll_gemm_bf16": (c_int, [c_int, c_int, c_int, c_void_p, ctypes.c_int64, c_void_p, ctypes.c_int64, c_int, c_void_p,
                             ctypes.c_int64, c_int, c_void_p]),
    "ll_gemm_bf16_two_outputs": (c_int, [c_int, c_int, c_int, c_void_p, ctypes.c_int64, c_void_p, c_void_p,
                                         ctypes.c_int64, c_int, c_void_p, c_void_p, ctypes.c_int64, c_int, c_void_p]),
    "ll_gemm_bf16_sum2": (c_int, [c_int, c_int, c_void_p, c_int, ctypes.c_int64, c_void_p, ctypes.c_int64, c_int,
                                  c_void_p, c_int, ctypes.c_int64, c_void_p, ctypes.c_int64, c_int, c_void_p,
                                  ctypes.c_int64, c_int, c_void_p]),
    "ll_gemm_bf16_status": (c_int, [c_void_p]),
    "ll_rmsnorm_forward": (c_int, [c_void_p, c_void_p, c_int, c_int, ctypes.c_float, c_void_p, c_int, c_void_p,
                                   c_void_p]),
    "ll_rmsnorm_backward": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_void_p]),
    "ll_profile_launch_events": (c_int, [ctypes.POINTER(c_void_p), c_int]),
    "ll_profile_launch_recorded": (c_int, []),
    "ll_profile_launch_name": (ctypes.c_char_p, [c_int]),
}


def exported_symbols():
    return list(_SIGS)


def load(build_if_needed: bool = True):
    """The loaded library (ctypes.CDLL with signatures set). Raises if it cannot be loaded."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if build_if_needed and not _build.up_to_date():
            try:
                _build.build()
            except Exception as exc:   # no nvcc on this machine: fall through to the prebuilt file
                if not os.path.exists(_build.LIB):
                    raise RuntimeError(f"lazylora_b200 CUDA library missing and not buildable: {exc}") from exc
        if not os.path.exists(_build.LIB):
            raise RuntimeError(f"lazylora_b200 CUDA library not found at {_build.LIB}")
        lib = ctypes.CDLL(_build.LIB)
        for name, (res, args) in _SIGS.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return _lib


def check(rc: int, where: str):
    if rc != 0:
        detail = load().ll_last_cuda_error().decode(errors="replace")
        raise LLError(rc, where, detail)


def require_cuda(*tensors):
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise ValueError("lazylora_b200 works on CUDA tensors only (no CPU fallback)")


def stream_ptr(stream=None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def ptr(t):
    return None if t is None else t.data_ptr()
