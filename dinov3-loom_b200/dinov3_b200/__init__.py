"""dinov3_b200 - DINOv3 ViT-S+/16 (224x224) forward on NVIDIA B200 (sm_100a).

Python face of the C ABI in include/dinov3.h, mirroring the reference crate's API
(src/lib.rs of zacharydenton/dinov3-loom):

    model = DINOv3.load("model.safetensors", Options(device=0, max_batch=32))
    tokens = model.forward(pixels)        # [n, 201, 384] float32 (CLS, 4 registers, 196 patches)
    cls = model.cls(pixels)               # [n, 384]
    mean = model.patch_mean(pixels)       # [n, 384]
    timings = model.benchmark(pixels, samples=20)

`pixels` are normalised NCHW float32 images, n x 3 x 224 x 224 (any shape with that many
floats). Errors raise DINOv3Error carrying the library's status code and message (the
reference's error texts). All compute runs in the CUDA library; there is no CPU path.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib
from ._lib import Distribution, ForwardTimings, LibraryMissing, Options

IMAGE_ELEMENTS = 3 * 224 * 224
TOKENS = 201
HIDDEN = 384

OK, INVALID_ARGUMENT, WEIGHTS, DEVICE, POISONED = range(5)

__all__ = [
    "DINOv3", "DINOv3Error", "Options", "ForwardTimings", "Distribution", "LibraryMissing",
    "IMAGE_ELEMENTS", "TOKENS", "HIDDEN", "pack_f16", "hub_weights",
]


class DINOv3Error(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


def _check(rc: int) -> None:
    if rc != OK:
        raise DINOv3Error(rc, _lib.last_error())


def _is_torch(x) -> bool:
    return hasattr(x, "data_ptr") and hasattr(x, "is_cuda")


def _host_floats(pixels):
    """(pointer, n_floats, keepalive) of a contiguous float32 host buffer."""
    if _is_torch(pixels):
        import torch

        if pixels.dtype != torch.float32 or not pixels.is_contiguous():
            pixels = pixels.to(torch.float32).contiguous()
        return pixels.data_ptr(), pixels.numel(), pixels
    arr = np.ascontiguousarray(pixels, dtype=np.float32)
    return arr.ctypes.data, arr.size, arr


class DINOv3:
    """A resident model on one GPU (src/lib.rs:29-35). One caller at a time; use separate
    models for concurrent callers."""

    def __init__(self, handle: int):
        self._h = ctypes.c_void_p(handle)
        self._inflight = {}  # ticket -> buffers kept alive until wait()

    # -- construction -------------------------------------------------------------------------
    @classmethod
    def load(cls, path, options: Options | None = None) -> "DINOv3":
        """DINOv3::load (src/lib.rs:49-88)."""
        lib = _lib.load()
        if options is None:
            options = lib.dv3_default_options()
        h = ctypes.c_void_p()
        _check(lib.dv3_load(str(path).encode(), options, ctypes.byref(h)))
        m = cls(h.value)
        m.options = Options(options.device, options.max_batch)
        return m

    @classmethod
    def from_pretrained(cls, options: Options | None = None) -> "DINOv3":
        """DINOv3::from_pretrained (src/lib.rs:40-46): the pinned weights from the Hugging Face
        cache (hub_weights); a miss raises DINOv3Error, nothing is downloaded."""
        lib = _lib.load()
        if options is None:
            options = lib.dv3_default_options()
        h = ctypes.c_void_p()
        _check(lib.dv3_from_pretrained(options, ctypes.byref(h)))
        m = cls(h.value)
        m.options = Options(options.device, options.max_batch)
        return m

    def close(self) -> None:
        if getattr(self, "_h", None) and self._h.value:
            _lib.load().dv3_free(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    # -- inference (host buffers) -------------------------------------------------------------
    def forward(self, pixels, out=None):
        """DINOv3::forward (src/lib.rs:90-114) -> [n, 201, 384] float32.

        pixels: numpy array or CPU torch tensor (pinned memory transfers faster), or a CUDA
        torch tensor on the model's device (then the result is a CUDA tensor). `out` may be a
        preallocated float32 buffer of n*201*384 elements of the same kind.
        """
        if _is_torch(pixels) and pixels.is_cuda:
            return self.forward_device(pixels, out)
        ptr, n, keep = _host_floats(pixels)
        batch = n // IMAGE_ELEMENTS
        if out is None:
            out = np.empty((batch, TOKENS, HIDDEN), dtype=np.float32)
        optr = out.data_ptr() if _is_torch(out) else out.ctypes.data
        onum = out.numel() if _is_torch(out) else out.size
        _check(_lib.load().dv3_forward(self._h, ptr, n, optr, onum))
        del keep
        return out

    def cls(self, pixels):
        """DINOv3::cls (src/lib.rs:126-132) -> [n, 384]."""
        ptr, n, keep = _host_floats(pixels)
        out = np.empty((n // IMAGE_ELEMENTS, HIDDEN), dtype=np.float32)
        _check(_lib.load().dv3_cls(self._h, ptr, n, out.ctypes.data, out.size))
        del keep
        return out

    def patch_mean(self, pixels):
        """DINOv3::patch_mean (src/lib.rs:134-148) -> [n, 384]."""
        ptr, n, keep = _host_floats(pixels)
        out = np.empty((n // IMAGE_ELEMENTS, HIDDEN), dtype=np.float32)
        _check(_lib.load().dv3_patch_mean(self._h, ptr, n, out.ctypes.data, out.size))
        del keep
        return out

    def benchmark(self, pixels, samples: int) -> ForwardTimings:
        """DINOv3::benchmark (src/lib.rs:116-124): graph replay vs direct dispatch."""
        ptr, n, keep = _host_floats(pixels)
        t = ForwardTimings()
        _check(_lib.load().dv3_benchmark(self._h, ptr, n, samples, ctypes.byref(t)))
        del keep
        return t

    # -- serving path (asynchronous) ----------------------------------------------------------
    def submit(self, pixels, out) -> int:
        """Enqueue upload, forward and download of 1..max_batch images; returns a ticket at once.

        `pixels` and `out` (n*201*384 float32) are host buffers (pinned CPU torch tensors overlap
        best) that must stay alive and unchanged until wait(ticket) returns; the model keeps a
        reference to both until then.
        """
        ptr, n, keep = _host_floats(pixels)
        optr = out.data_ptr() if _is_torch(out) else out.ctypes.data
        onum = out.numel() if _is_torch(out) else out.size
        t = ctypes.c_uint64()
        _check(_lib.load().dv3_submit(self._h, ptr, n, optr, onum, ctypes.byref(t)))
        self._inflight[t.value] = (keep, pixels, out)
        return t.value

    def wait(self, ticket: int):
        """Block until submission `ticket` is done; returns its output buffer."""
        held = self._inflight.pop(ticket, None)
        _check(_lib.load().dv3_wait(self._h, ticket))
        return held[2] if held else None

    # -- device-resident path -----------------------------------------------------------------
    def forward_device(self, pixels, out=None):
        """Forward of CUDA float32 tensors on the model's device; returns a CUDA tensor."""
        import torch

        pixels = pixels.to(torch.float32).contiguous()
        batch = pixels.numel() // IMAGE_ELEMENTS
        if out is None:
            out = torch.empty((batch, TOKENS, HIDDEN), dtype=torch.float32, device=pixels.device)
        _check(_lib.load().dv3_forward_device(self._h, pixels.data_ptr(), pixels.numel(),
                                              out.data_ptr(), out.numel()))
        return out

    @property
    def input_buffer(self) -> int:
        """Device address of the resident input (max_batch x 3 x 224 x 224 float32)."""
        return _lib.load().dv3_input_buffer(self._h) or 0

    @property
    def output_buffer(self) -> int:
        """Device address of the resident output (max_batch x 201 x 384 float32)."""
        return _lib.load().dv3_output_buffer(self._h) or 0

    @property
    def stream(self) -> int:
        """The model's cudaStream_t."""
        return _lib.load().dv3_stream(self._h) or 0

    def run(self, batch: int) -> None:
        """Enqueue one graph replay over the first `batch` staged images (asynchronous)."""
        _check(_lib.load().dv3_run(self._h, batch))

    def synchronize(self) -> None:
        _check(_lib.load().dv3_synchronize(self._h))

    def launches_per_forward(self, batch: int) -> int:
        n = ctypes.c_size_t()
        _check(_lib.load().dv3_launches_per_forward(self._h, batch, ctypes.byref(n)))
        return n.value

    def profile_launches(self, batch: int, iterations: int = 10):
        """[(kernel name, average device ms)] for every launch of one forward, in order."""
        cap = 256
        ms = (ctypes.c_double * cap)()
        names = (ctypes.c_char_p * cap)()
        count = ctypes.c_size_t()
        _check(_lib.load().dv3_profile_launches(self._h, batch, iterations, ms, names, cap,
                                                ctypes.byref(count)))
        return [(names[i].decode(), ms[i]) for i in range(min(count.value, cap))]

    def profile_forward(self, batch: int, replays: int = 10, flush_bytes: int = 256 << 20):
        """[(kernel name, average device ms)] for every launch of one forward, in order, timed
        inside whole forwards with an L2 flush of `flush_bytes` before each (dv3_profile_forward)."""
        cap = 256
        ms = (ctypes.c_double * cap)()
        names = (ctypes.c_char_p * cap)()
        count = ctypes.c_size_t()
        _check(_lib.load().dv3_profile_forward(self._h, batch, replays, flush_bytes, ms, names,
                                               cap, ctypes.byref(count)))
        return [(names[i].decode(), ms[i]) for i in range(min(count.value, cap))]

    def debug_inject_fault(self, bits: int = 1 << 30) -> None:
        """Test hook: the next forward reports a device failure (DV3_POISONED) without one."""
        _check(_lib.load().dv3_debug_inject_fault(self._h, bits))


def pack_f16(name: str, values) -> np.ndarray:
    """The packer's f32 -> f16 narrowing (src/weights.rs:6-17); raises DINOv3Error on the first
    value that is not finite in f16."""
    arr = np.ascontiguousarray(values, dtype=np.float32)
    out = np.empty(arr.shape, dtype=np.uint16)
    bad = ctypes.c_size_t()
    _check(_lib.load().dv3_pack_f16(name.encode(), arr.ctypes.data, arr.size, out.ctypes.data,
                                    ctypes.byref(bad)))
    return out.view(np.float16)


def hub_weights(offline: bool = False) -> str:
    """Path of the pinned model.safetensors in the shared Hugging Face cache (src/hub.rs:17-54).
    Offline when `offline` or HF_HUB_OFFLINE is set to anything but "" or "0"; a file that is not
    cached raises DINOv3Error (WEIGHTS) with the reference's message. Nothing is downloaded."""
    buf = ctypes.create_string_buffer(4096)
    _check(_lib.load().dv3_hub_weights(1 if offline else 0, buf, len(buf)))
    return buf.value.decode()
