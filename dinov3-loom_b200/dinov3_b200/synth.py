"""Seeded synthetic weights and images for DINOv3 ViT-S+/16 at 224x224.

The pretrained checkpoint (facebook/dinov3-vits16plus-pretrain-lvd1689m) is gated and there is
no network, so the model is exercised with random-init weights of the same architecture, written
as an F32 safetensors file with the Hugging Face tensor names and shapes that the reference's
packer reads (src/weights.rs:62-126) and its float64 test oracle reads
(tests/support/reference.rs:80-191).

Every value is a pure function of (seed, tensor name, element index): a splitmix64-style
counter hash feeds Box-Muller normals. Any tensor can be regenerated on any machine without
replaying a stream, and the same numbers come out of numpy on the build container and on the
GPU box.

Two weight flavours:
  * "baseline" - the benchmark configuration: Linear/conv weights truncated normal (std 0.02,
    cut at +-2 sigma, resampled), every bias 0 (k has none), LayerNorm gamma 1 / beta 0,
    LayerScale 0.1, CLS and register tokens N(0, 0.02^2).
  * "stress" - the same matrices, but nonzero biases, gammas, betas and per-channel LayerScale,
    so that parity tests exercise every bias / affine / LayerScale path of the GPU epilogues
    (with "baseline" those terms are all identities and a wrong index would go unseen).
"""
from __future__ import annotations

import numpy as np

HIDDEN = 384
TOKENS = 201
PATCHES = 196
PREFIX = 5
LAYERS = 12
HEADS = 6
HEAD_DIM = 64
MLP = 1536
IMAGE_ELEMENTS = 3 * 224 * 224

MEAN = (0.485, 0.456, 0.406)
STD = (0.229, 0.224, 0.225)

_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)
_GOLD = np.uint64(0x9E3779B97F4A7C15)
_MASK64 = (1 << 64) - 1


def _mix(z: np.ndarray) -> np.ndarray:
    """splitmix64 finaliser on a uint64 array (wrapping arithmetic)."""
    z = z ^ (z >> np.uint64(30))
    z = z * _M1
    z = z ^ (z >> np.uint64(27))
    z = z * _M2
    return z ^ (z >> np.uint64(31))


def _key(seed: int, name: str) -> np.uint64:
    h = 0xCBF29CE484222325  # FNV-1a over the stream name
    for b in name.encode():
        h = ((h ^ b) * 0x100000001B3) & _MASK64
    h ^= (int(seed) * 0x9E3779B97F4A7C15) & _MASK64
    return _mix(np.array([h], dtype=np.uint64))[0]


def uniform(seed: int, name: str, index: np.ndarray) -> np.ndarray:
    """U[0,1) doubles for the given element indices of stream `name`."""
    idx = np.asarray(index, dtype=np.uint64)
    with np.errstate(over="ignore"):
        bits = _mix(idx * _GOLD + _key(seed, name))
    return (bits >> np.uint64(11)).astype(np.float64) * (2.0 ** -53)


def normal(seed: int, name: str, index: np.ndarray) -> np.ndarray:
    u1 = uniform(seed, name + "#u1", index)
    u2 = uniform(seed, name + "#u2", index)
    return np.sqrt(-2.0 * np.log1p(-u1)) * np.cos(2.0 * np.pi * u2)


def trunc_normal(seed: int, name: str, n: int, std: float, bound: float = 2.0) -> np.ndarray:
    """N(0, std^2) truncated at +-bound*std by per-element resampling."""
    idx = np.arange(n, dtype=np.uint64)
    z = normal(seed, name, idx)
    attempt = 0
    while True:
        bad = np.nonzero(np.abs(z) > bound)[0]
        if bad.size == 0:
            break
        attempt += 1
        z[bad] = normal(seed, f"{name}#retry{attempt}", idx[bad])
    return z * std


def _normal(seed: int, name: str, n: int, std: float) -> np.ndarray:
    return normal(seed, name, np.arange(n, dtype=np.uint64)) * std


def weights(seed: int = 0, flavor: str = "baseline") -> dict[str, np.ndarray]:
    """All model tensors as float32 arrays keyed by Hugging Face name."""
    if flavor not in ("baseline", "stress"):
        raise ValueError(f"unknown weight flavor {flavor!r}")
    stress = flavor == "stress"
    out: dict[str, np.ndarray] = {}

    def mat(name, shape):
        out[name] = trunc_normal(seed, name, int(np.prod(shape)), 0.02).reshape(shape).astype(np.float32)

    def bias(name, n, std=0.02):
        v = _normal(seed, name, n, std) if stress else np.zeros(n)
        out[name] = v.astype(np.float32)

    def gamma(name, n):
        v = 1.0 + _normal(seed, name, n, 0.1) if stress else np.ones(n)
        out[name] = v.astype(np.float32)

    def scale(name, n):
        v = 0.05 + 0.15 * uniform(seed, name, np.arange(n)) if stress else np.full(n, 0.1)
        out[name] = v.astype(np.float32)

    mat("embeddings.patch_embeddings.weight", (HIDDEN, 3, 16, 16))
    bias("embeddings.patch_embeddings.bias", HIDDEN)
    out["embeddings.cls_token"] = _normal(seed, "embeddings.cls_token", HIDDEN, 0.02).reshape(1, 1, HIDDEN).astype(np.float32)
    out["embeddings.register_tokens"] = (
        _normal(seed, "embeddings.register_tokens", 4 * HIDDEN, 0.02).reshape(1, 4, HIDDEN).astype(np.float32)
    )
    # Present in Hugging Face checkpoints; unused by the forward (masking is training-only).
    out["embeddings.mask_token"] = np.zeros((1, 1, HIDDEN), np.float32)
    for i in range(LAYERS):
        p = f"layer.{i}."
        gamma(p + "norm1.weight", HIDDEN)
        bias(p + "norm1.bias", HIDDEN, 0.05)
        for q in ("q", "k", "v", "o"):
            mat(p + f"attention.{q}_proj.weight", (HIDDEN, HIDDEN))
        for q in ("q", "v", "o"):
            bias(p + f"attention.{q}_proj.bias", HIDDEN)
        scale(p + "layer_scale1.lambda1", HIDDEN)
        gamma(p + "norm2.weight", HIDDEN)
        bias(p + "norm2.bias", HIDDEN, 0.05)
        mat(p + "mlp.gate_proj.weight", (MLP, HIDDEN))
        mat(p + "mlp.up_proj.weight", (MLP, HIDDEN))
        mat(p + "mlp.down_proj.weight", (HIDDEN, MLP))
        bias(p + "mlp.gate_proj.bias", MLP)
        bias(p + "mlp.up_proj.bias", MLP)
        bias(p + "mlp.down_proj.bias", HIDDEN)
        scale(p + "layer_scale2.lambda1", HIDDEN)
    gamma("norm.weight", HIDDEN)
    bias("norm.bias", HIDDEN, 0.05)
    return out


def write_weights(path: str, seed: int = 0, flavor: str = "baseline") -> str:
    from safetensors.numpy import save_file

    save_file(weights(seed, flavor), str(path))
    return str(path)


def images(seed: int, n: int, first: int = 0) -> np.ndarray:
    """n normalised NCHW float32 images: U[0,1) pixels, then (u - mean[c]) / std[c].

    Image `first + i` depends only on (seed, first + i), so a large batch can be produced in
    slices that agree with one big call.
    """
    idx = np.arange(first * IMAGE_ELEMENTS, (first + n) * IMAGE_ELEMENTS, dtype=np.uint64)
    u = uniform(seed, "images", idx).reshape(n, 3, 224, 224)
    mean = np.asarray(MEAN).reshape(1, 3, 1, 1)
    std = np.asarray(STD).reshape(1, 3, 1, 1)
    return ((u - mean) / std).astype(np.float32)


def reference_test_images(n: int) -> np.ndarray:
    """The input of the reference's GPU parity test (tests/model.rs:72-74): sin(0.037 i) * 0.6."""
    i = np.arange(n * IMAGE_ELEMENTS, dtype=np.float64)
    return (np.sin(i * 0.037) * 0.6).astype(np.float32).reshape(n, 3, 224, 224)
