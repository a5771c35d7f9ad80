"""numpy float64 restatement of the reference's test oracle.

TEST INFRASTRUCTURE ONLY. This module is a checker: only tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline legs may import it. The product path never routes through it.

It restates tests/support/reference.rs (the reference's straight-line float64 ViT forward for
one image) with numpy BLAS in place of matrixmultiply 0.3.11's dgemm. Line citations below
are to that file unless another file is named. Its C twin is oracle/ref_f64.c; the two are
written independently and are checked against each other and against the golden fixtures in
tests/golden/ (made by tests/golden/make_golden.py from Hugging Face transformers'
DINOv3ViTModel in float64).
"""
from __future__ import annotations

import numpy as np

T, H, HEADS, D, PREFIX = 201, 384, 6, 64, 5


def patchify(image: np.ndarray) -> np.ndarray:
    """[3,224,224] -> [196, 768] with inner order (c, dy, dx); reference.rs:67-79 and
    src/lib.rs:265-280 (pinned by src/lib.rs:304-328)."""
    x = np.asarray(image, dtype=np.float64).reshape(3, 14, 16, 14, 16)  # c, gy, dy, gx, dx
    return x.transpose(1, 3, 0, 2, 4).reshape(196, 768)


def linear(x, w, b=None):
    """x[m,k] @ w[n,k]^T + b; reference.rs:5-37."""
    out = x @ w.T
    if b is not None:
        out = out + b
    return out


def norm(x, w, b):
    """LayerNorm, eps 1e-5, two-pass biased variance; reference.rs:38-48."""
    mean = x.mean(axis=-1, keepdims=True)
    var = ((x - mean) ** 2).mean(axis=-1, keepdims=True)
    return (x - mean) / np.sqrt(var + 1e-5) * w + b


def rope_tables():
    """cos/sin [196, 64]: channel c uses the patch row (c%32<16) or column (c%32>=16) and
    frequency index c%16; angle = 2*pi*(2*(pos+0.5)/14-1) / 100^(j/16).
    reference.rs:112-118 and src/weights.rs:127-144."""
    patch = np.arange(196)
    c = np.arange(64)
    pos = np.where((c % 32) < 16, patch[:, None] // 14, patch[:, None] % 14)
    coord = 2.0 * (pos + 0.5) / 14.0 - 1.0
    angle = 2.0 * np.pi * coord / (100.0 ** ((c % 16) / 16.0))
    return np.cos(angle), np.sin(angle)


def rope(values, cos, sin):
    """In-place rotation of q or k patch tokens; reference.rs:108-128.
    c < 32: x_c cos - x_{c+32} sin; c >= 32: x_c cos + x_{c-32} sin."""
    v = values[PREFIX:].reshape(196, HEADS, D)
    rot = np.concatenate([-v[..., 32:], v[..., :32]], axis=-1)
    values[PREFIX:] = (v * cos[:, None, :] + rot * sin[:, None, :]).reshape(196, H)


def forward(weights: dict, image: np.ndarray) -> np.ndarray:
    """One normalised [3,224,224] image -> [201, 384] float64; reference.rs:49-192."""
    w = {k: np.asarray(v, dtype=np.float64) for k, v in weights.items()}
    cos, sin = rope_tables()
    patches = patchify(image)
    x = np.concatenate(
        [
            w["embeddings.cls_token"].reshape(1, H),
            w["embeddings.register_tokens"].reshape(4, H),
            linear(patches, w["embeddings.patch_embeddings.weight"].reshape(H, 768),
                   w["embeddings.patch_embeddings.bias"]),
        ]
    )  # reference.rs:80-88
    for layer in range(12):
        p = f"layer.{layer}."
        h = norm(x, w[p + "norm1.weight"], w[p + "norm1.bias"])
        q = linear(h, w[p + "attention.q_proj.weight"], w[p + "attention.q_proj.bias"])
        k = linear(h, w[p + "attention.k_proj.weight"])  # no key bias; reference.rs:100
        v = linear(h, w[p + "attention.v_proj.weight"], w[p + "attention.v_proj.bias"])
        rope(q, cos, sin)
        rope(k, cos, sin)
        # reference.rs:129-151: per head softmax(q k^T * 0.125) v
        qh = q.reshape(T, HEADS, D).transpose(1, 0, 2)
        kh = k.reshape(T, HEADS, D).transpose(1, 0, 2)
        vh = v.reshape(T, HEADS, D).transpose(1, 0, 2)
        s = qh @ kh.transpose(0, 2, 1) * 0.125
        s = np.exp(s - s.max(axis=-1, keepdims=True))
        a = s / s.sum(axis=-1, keepdims=True)
        context = (a @ vh).transpose(1, 0, 2).reshape(T, H)
        o = linear(context, w[p + "attention.o_proj.weight"], w[p + "attention.o_proj.bias"])
        x = x + o * w[p + "layer_scale1.lambda1"]  # reference.rs:159-161
        h = norm(x, w[p + "norm2.weight"], w[p + "norm2.bias"])
        g = linear(h, w[p + "mlp.gate_proj.weight"], w[p + "mlp.gate_proj.bias"])
        u = linear(h, w[p + "mlp.up_proj.weight"], w[p + "mlp.up_proj.bias"])
        g = g / (1.0 + np.exp(-g)) * u  # reference.rs:177-179
        d = linear(g, w[p + "mlp.down_proj.weight"], w[p + "mlp.down_proj.bias"])
        x = x + d * w[p + "layer_scale2.lambda1"]  # reference.rs:187-189
    return norm(x, w["norm.weight"], w["norm.bias"])  # reference.rs:191


def forward_batch(weights: dict, images: np.ndarray) -> np.ndarray:
    images = np.asarray(images).reshape(-1, 3, 224, 224)
    return np.stack([forward(weights, im) for im in images])


def cosine(a, b) -> float:
    """The reference test's comparison (tests/model.rs:79-84)."""
    a = np.asarray(a, dtype=np.float64).ravel()
    b = np.asarray(b, dtype=np.float64).ravel()
    return float(a @ b / np.sqrt((a @ a) * (b @ b)))
