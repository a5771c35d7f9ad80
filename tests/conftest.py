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
