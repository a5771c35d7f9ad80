"""ctypes loader for oracle/ref_f64.c (the C float64 restatement of the reference's oracle).

TEST INFRASTRUCTURE ONLY: for tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "libref_f64.so")


def build(force: bool = False) -> str:
    """Compile the oracle with its Makefile (system gcc, OpenMP)."""
    if force or not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(
        os.path.join(HERE, "ref_f64.c")
    ):
        env = dict(os.environ)
        env.pop("CC", None)
        subprocess.run(["make", "-C", HERE, "-B" if force else "all"], check=True, env=env,
                       stdout=subprocess.PIPE, stderr=subprocess.STDOUT)
    return LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        build()
        l = ctypes.CDLL(LIB_PATH)
        l.ref_model_new.restype = ctypes.c_void_p
        l.ref_model_free.argtypes = [ctypes.c_void_p]
        l.ref_model_set.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_void_p, ctypes.c_size_t]
        l.ref_model_set.restype = ctypes.c_int
        l.ref_model_missing.argtypes = [ctypes.c_void_p]
        l.ref_model_missing.restype = ctypes.c_int
        l.ref_forward.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int]
        l.ref_forward.restype = ctypes.c_int
        l.ref_patchify.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
        l.ref_rope_tables.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
        l.ref_max_threads.restype = ctypes.c_int
        _lib = l
    return _lib


class Model:
    """Float64 CPU model built from a {name: float32 array} dict (Hugging Face names)."""

    def __init__(self, weights: dict):
        self._l = lib()
        self._m = self._l.ref_model_new()
        for name, value in weights.items():
            if name == "embeddings.mask_token":
                continue
            arr = np.ascontiguousarray(value, dtype=np.float32)
            rc = self._l.ref_model_set(self._m, name.encode(), arr.ctypes.data, arr.size)
            if rc != 0:
                raise ValueError(f"oracle rejected tensor {name} {arr.shape}")
        missing = self._l.ref_model_missing(self._m)
        if missing != 0:
            raise ValueError(f"oracle model is missing {missing} tensors")

    def forward(self, images: np.ndarray, threads: int = 0) -> np.ndarray:
        imgs = np.ascontiguousarray(images, dtype=np.float32).reshape(-1, 3, 224, 224)
        n = imgs.shape[0]
        out = np.empty((n, 201, 384), dtype=np.float64)
        rc = self._l.ref_forward(self._m, imgs.ctypes.data, n, out.ctypes.data, threads)
        if rc != 0:
            raise RuntimeError("oracle forward failed")
        return out

    def __del__(self):
        if getattr(self, "_m", None):
            self._l.ref_model_free(self._m)
            self._m = None


def patchify(image: np.ndarray) -> np.ndarray:
    img = np.ascontiguousarray(image, dtype=np.float32)
    out = np.empty((196, 768), dtype=np.float64)
    lib().ref_patchify(img.ctypes.data, out.ctypes.data)
    return out


def rope_tables():
    c = np.empty((196, 64), dtype=np.float64)
    s = np.empty((196, 64), dtype=np.float64)
    lib().ref_rope_tables(c.ctypes.data, s.ctypes.data)
    return c, s


def max_threads() -> int:
    return int(lib().ref_max_threads())
