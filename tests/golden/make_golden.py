"""Generate the golden fixtures that pin the float64 oracle.

The reference ships no golden output vectors, and its own float64 oracle
(tests/support/reference.rs) is Rust, which cannot be built here. The fixtures therefore come
from an independent implementation of the same published architecture: Hugging Face
transformers' DINOv3ViTModel (transformers 5.5.0, the library whose checkpoint names the
reference reads), run in float64 on CPU on the seeded synthetic weights and images of
dinov3_b200.synth.

Hugging Face computes its RoPE angles in float32 even when the model runs in float64
(DINOv3ViTRopePositionEmbedding.forward forces float32); the reference computes them in
float64 (tests/support/reference.rs:112-118). This script replaces that one method with a
float64 evaluation of the same formula, so the fixtures carry no float32 rounding and the
oracle must agree with them to ~1e-12.

Stored per case (float64): the output rows listed in ROWS (CLS, the 4 registers and 11 patch
tokens), the L2 norm of every one of the 201 output rows, and the sum of all outputs; plus
sha256 digests of the generated weights and image, so that a change in the generator shows up
as its own failure rather than as an oracle mismatch.

Run from the repository root:  python tests/golden/make_golden.py
"""
from __future__ import annotations

import math
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "dinov3-loom_b200"))

from dinov3_b200 import synth  # noqa: E402

ROWS = [0, 1, 2, 3, 4, 5, 6, 18, 19, 60, 100, 104, 150, 187, 199, 200]
# (name, weight seed, weight flavour, image source, image seed or count)
CASES = [
    ("baseline_seed0_img7", 0, "baseline", "seeded", 7),
    ("stress_seed1_img3", 1, "stress", "seeded", 3),
    ("stress_seed1_sin", 1, "stress", "sin", 0),
]


def hf_forward(weights: dict, image: np.ndarray) -> np.ndarray:
    import torch
    from transformers import DINOv3ViTConfig, DINOv3ViTModel
    from transformers.models.dinov3_vit import modeling_dinov3_vit as mod

    def rope_f64(self, pixel_values):
        n = 224 // 16
        c = (torch.arange(n, dtype=torch.float64) + 0.5) / n * 2.0 - 1.0
        coords = torch.stack(torch.meshgrid(c, c, indexing="ij"), dim=-1).flatten(0, 1)
        inv = 1.0 / 100.0 ** torch.arange(0, 1, 4 / 64, dtype=torch.float64)
        angles = (2 * math.pi * coords[:, :, None] * inv[None, None, :]).flatten(1, 2).tile(2)
        return torch.cos(angles).to(pixel_values.dtype), torch.sin(angles).to(pixel_values.dtype)

    mod.DINOv3ViTRopePositionEmbedding.forward = rope_f64
    cfg = DINOv3ViTConfig(
        hidden_size=384, intermediate_size=1536, num_hidden_layers=12, num_attention_heads=6,
        hidden_act="silu", use_gated_mlp=True, num_register_tokens=4, rope_theta=100.0,
        layer_norm_eps=1e-5, image_size=224, patch_size=16, query_bias=True, key_bias=False,
        value_bias=True, proj_bias=True, mlp_bias=True, layerscale_value=0.1,
    )
    model = DINOv3ViTModel(cfg).double().eval()
    # transformers 5.x nests the encoder under `model.`; checkpoints (and the reference) use the
    # bare `layer.{i}.` names.
    state = {("model." + k if k.startswith("layer.") else k): torch.from_numpy(np.asarray(v, dtype=np.float64))
             for k, v in weights.items()}
    missing, unexpected = model.load_state_dict(state, strict=False)
    if unexpected or any(not k.endswith("inv_freq") for k in missing):
        raise SystemExit(f"state dict mismatch: missing={missing} unexpected={unexpected}")
    with torch.no_grad():
        out = model(pixel_values=torch.from_numpy(image[None].astype(np.float64))).last_hidden_state
    return out[0].numpy()


def digest(weights: dict) -> str:
    """sha256 over every tensor's float32 bytes, in name order."""
    import hashlib

    h = hashlib.sha256()
    for k in sorted(weights):
        h.update(k.encode())
        h.update(np.ascontiguousarray(weights[k], dtype=np.float32).tobytes())
    return h.hexdigest()


def case_image(source: str, arg: int) -> np.ndarray:
    if source == "seeded":
        return synth.images(arg, 1)[0]
    return synth.reference_test_images(1)[0]


def main() -> None:
    for name, seed, flavor, source, arg in CASES:
        w = synth.weights(seed, flavor)
        img = case_image(source, arg)
        out = hf_forward(w, img)
        np.savez(
            os.path.join(HERE, f"{name}.npz"),
            rows=np.asarray(ROWS),
            values=out[ROWS],
            row_norms=np.linalg.norm(out, axis=1),
            total=np.asarray(out.sum()),
            weight_seed=np.asarray(seed),
            flavor=np.asarray(flavor),
            image_source=np.asarray(source),
            image_arg=np.asarray(arg),
            weights_sha256=np.asarray(digest(w)),
            image_sha256=np.asarray(digest({"image": img})),
        )
        print(name, "max|out|", np.abs(out).max(), "sum", out.sum())


if __name__ == "__main__":
    main()
