"""ctypes binding of libdinov3.so (include/dinov3.h and include/dinov3_kernels.h).

There is no fallback: if the library has not been built, loading raises LibraryMissing.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libdinov3.so")


class LibraryMissing(ImportError):
    pass


class Options(ctypes.Structure):
    """dv3_options (src/lib.rs:15-27)."""

    _fields_ = [("device", ctypes.c_int32), ("max_batch", ctypes.c_size_t)]

    def __init__(self, device: int = 0, max_batch: int = 32):
        super().__init__(device, max_batch)

    def __repr__(self):
        return f"Options(device={self.device}, max_batch={self.max_batch})"


class Distribution(ctypes.Structure):
    _fields_ = [("median_ms", ctypes.c_double), ("p95_ms", ctypes.c_double)]

    def __repr__(self):
        return f"Distribution(median_ms={self.median_ms:.4f}, p95_ms={self.p95_ms:.4f})"


class ForwardTimings(ctypes.Structure):
    _fields_ = [("samples", ctypes.c_size_t), ("graph", Distribution), ("direct", Distribution)]

    def as_dict(self):
        return {
            "samples": self.samples,
            "graph": {"median_ms": self.graph.median_ms, "p95_ms": self.graph.p95_ms},
            "direct": {"median_ms": self.direct.median_ms, "p95_ms": self.direct.p95_ms},
        }


# Exported symbols and their signatures (argtypes, restype).
_P = ctypes.c_void_p
_SZ = ctypes.c_size_t
_U32 = ctypes.c_uint32
_I = ctypes.c_int
SIGNATURES = {
    # dinov3.h
    "dv3_default_options": ([], Options),
    "dv3_load": ([ctypes.c_char_p, Options, ctypes.POINTER(_P)], _I),
    "dv3_forward": ([_P, _P, _SZ, _P, _SZ], _I),
    "dv3_cls": ([_P, _P, _SZ, _P, _SZ], _I),
    "dv3_patch_mean": ([_P, _P, _SZ, _P, _SZ], _I),
    "dv3_benchmark": ([_P, _P, _SZ, _SZ, ctypes.POINTER(ForwardTimings)], _I),
    "dv3_free": ([_P], None),
    "dv3_last_error": ([], ctypes.c_char_p),
    "dv3_input_buffer": ([_P], _P),
    "dv3_output_buffer": ([_P], _P),
    "dv3_stream": ([_P], _P),
    "dv3_run": ([_P, _SZ], _I),
    "dv3_synchronize": ([_P], _I),
    "dv3_forward_device": ([_P, _P, _SZ, _P, _SZ], _I),
    "dv3_submit": ([_P, _P, _SZ, _P, _SZ, ctypes.POINTER(ctypes.c_uint64)], _I),
    "dv3_wait": ([_P, ctypes.c_uint64], _I),
    "dv3_launches_per_forward": ([_P, _SZ, ctypes.POINTER(_SZ)], _I),
    "dv3_profile_launches": ([_P, _SZ, _SZ, _P, _P, _SZ, ctypes.POINTER(_SZ)], _I),
    "dv3_profile_forward": ([_P, _SZ, _SZ, _SZ, _P, _P, _SZ, ctypes.POINTER(_SZ)], _I),
    "dv3_debug_inject_fault": ([_P, _U32], _I),
    "dv3_pack_f16": ([ctypes.c_char_p, _P, _SZ, _P, ctypes.POINTER(_SZ)], _I),
    "dv3_hub_weights": ([_I, ctypes.c_char_p, _SZ], _I),
    "dv3_from_pretrained": ([Options, ctypes.POINTER(_P)], _I),
    # dinov3_kernels.h
    "dv3k_patchify": ([_P, _U32, _P, _P, _P, _P, _P], _I),
    "dv3k_patch_embed": ([_P, _U32, _P, _P, _P, _P, _P], _I),
    "dv3k_layernorm_f16": ([_P, _U32, _P, _P, _P, _P], _I),
    "dv3k_layernorm_f32out": ([_P, _U32, _P, _P, _P, _P], _I),
    "dv3k_qkv_rope": ([_P, _U32, _P, _P, _P, _P, _P, _P, _P], _I),
    "dv3k_attention": ([_P, _U32, _P, _P, _P], _I),
    "dv3k_matmul_resid": ([_P, _U32, _U32, _P, _P, _P, _P, _P, _P], _I),
    "dv3k_matmul_resid_layernorm": ([_P, _U32, _U32, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P], _I),
    "dv3k_matmul_swiglu": ([_P, _U32, _P, _P, _P, _P, _P], _I),
    "dv3k_matmul_splitk": ([_P, _U32, _P, _U32, _P, _P, _P], _I),
    "dv3k_splitk_reduce": ([_P, _U32, _U32, _P, _P, _P, _P], _I),
    "dv3k_splitk_reduce_layernorm": ([_P, _U32, _U32, _P, _P, _P, _P, _P, _P, _P, _P], _I),
    "dv3k_down_splitk_noalloc": ([_P, _U32, _P, _U32, _P, _P, _P, _P, _P], _I),
    "dv3k_matmul_resid_rowstat": ([_P, _U32, _U32, _P, _P, _P, _P, _P, _P, _P, _P], _I),
    "dv3k_layernorm_rowstat": ([_P, _U32, _P, _P, _P], _I),
    "dv3k_qkv_rope_folded": ([_P, _U32, _P, _P, _P, _P, _P, _P, _P, _P, _P], _I),
    "dv3k_matmul_swiglu_folded": ([_P, _U32, _P, _P, _P, _P, _P, _P, _P], _I),
    "dv3k_gateup_source_row": ([_U32], _U32),
    "dv3k_bounded_wait_selftest": ([ctypes.c_uint64, _P, _P], _I),
}

_lib = None


def load() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise LibraryMissing(
                f"{LIB_PATH} is not built; run `python dinov3-loom_b200/build.py` (nvcc, sm_100a)")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (args, res) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = res
        _lib = lib
    return _lib


def last_error() -> str:
    return load().dv3_last_error().decode("utf-8", "replace")
