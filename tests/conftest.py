"""Shared test setup.

Markers: `gpu` tests need a B200 (sm_100a) and the built CUDA library; everything else runs on
CPU. Paths: the product package lives in dinov3-loom_b200/ (a directory name that is not a
Python identifier), and the float64 oracle in oracle/.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for sub in ("dinov3-loom_b200", "oracle"):
    p = os.path.join(ROOT, sub)
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU and the built CUDA library")


GOLDEN = os.path.join(ROOT, "tests", "golden")


@pytest.fixture(scope="session")
def weights_file(tmp_path_factory):
    """Factory: path of an F32 safetensors file for (seed, flavor), written once per session."""
    from dinov3_b200 import synth

    cache = {}
    base = tmp_path_factory.mktemp("weights")

    def get(seed=0, flavor="baseline"):
        key = (seed, flavor)
        if key not in cache:
            cache[key] = synth.write_weights(str(base / f"w_{seed}_{flavor}.safetensors"), seed, flavor)
        return cache[key]

    return get


@pytest.fixture(scope="session")
def weights_dict():
    from dinov3_b200 import synth

    cache = {}

    def get(seed=0, flavor="baseline"):
        key = (seed, flavor)
        if key not in cache:
            cache[key] = synth.weights(seed, flavor)
        return cache[key]

    return get


def write_safetensors_raw(path, tensors):
    """tensors: {name: (dtype str, shape, raw bytes)} in the safetensors layout (8-byte header
    length, JSON header, data)."""
    import json
    import struct

    header, blob = {}, b""
    for name, (dtype, shape, raw) in tensors.items():
        header[name] = {"dtype": dtype, "shape": list(shape),
                        "data_offsets": [len(blob), len(blob) + len(raw)]}
        blob += raw
    h = json.dumps(header).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)) + h + blob)


@pytest.fixture(scope="session")
def weights_file_lowp(tmp_path_factory):
    """Factory: (path of an F16 or BF16 safetensors file of the seeded weights, path of an F32
    file holding the same values), written once per session."""
    import numpy as np
    from dinov3_b200 import synth

    cache = {}
    base = tmp_path_factory.mktemp("weights_lowp")

    def get(dtype, seed=0, flavor="baseline"):
        key = (dtype, seed, flavor)
        if key not in cache:
            low, f32 = {}, {}
            for name, v in synth.weights(seed, flavor).items():
                v = np.ascontiguousarray(v, dtype=np.float32)
                if dtype == "F16":
                    r = v.astype(np.float16)
                    low[name] = ("F16", v.shape, r.tobytes())
                    back = r.astype(np.float32)
                else:  # BF16, round to nearest even
                    bits = v.view(np.uint32).astype(np.uint64)
                    r = ((bits + 0x7FFF + ((bits >> 16) & 1)) >> 16).astype(np.uint16)
                    low[name] = ("BF16", v.shape, r.tobytes())
                    back = (r.astype(np.uint32) << 16).view(np.float32)
                f32[name] = ("F32", v.shape, np.ascontiguousarray(back).tobytes())
            p_low = base / f"w_{seed}_{flavor}_{dtype}.safetensors"
            p_f32 = base / f"w_{seed}_{flavor}_{dtype}_as_f32.safetensors"
            write_safetensors_raw(p_low, low)
            write_safetensors_raw(p_f32, f32)
            cache[key] = (str(p_low), str(p_f32))
        return cache[key]

    return get
