"""Host-side behaviour of the C ABI that needs no GPU: symbol exports, option and weight
validation order and messages (tests/model.rs:5-59), f16 packing (src/weights.rs:148-169),
the gate/up packing permutation, and argument checks of the per-kernel entry points."""
import ctypes
import json
import os
import re
import struct

import numpy as np
import pytest

import dinov3_b200 as dv
from dinov3_b200 import _lib

from conftest import ROOT


def _declared(header):
    text = open(os.path.join(ROOT, "include", header)).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"\b(dv3k?_\w+)\s*\(", text))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = _declared("dinov3.h") | _declared("dinov3_kernels.h")
    assert len(names) >= 25
    for n in names:
        assert hasattr(lib, n), n
    assert names == set(_lib.SIGNATURES), names ^ set(_lib.SIGNATURES)


def test_default_options():
    o = _lib.load().dv3_default_options()
    assert (o.device, o.max_batch) == (0, 32)  # src/lib.rs:20-27


@pytest.mark.parametrize("max_batch", [0, 65])
def test_rejects_options_before_loading(max_batch):
    """tests/model.rs:5-27: max_batch 0 and 65 are rejected before the file is read."""
    with pytest.raises(dv.DINOv3Error) as e:
        dv.DINOv3.load("/nonexistent", dv.Options(0, max_batch))
    assert e.value.code == dv.INVALID_ARGUMENT
    assert "max_batch must be 1..=64" in str(e.value)


def _write_safetensors(path, tensors):
    """tensors: {name: (dtype str, shape, raw bytes)}."""
    header, blob = {}, b""
    for name, (dtype, shape, raw) in tensors.items():
        header[name] = {"dtype": dtype, "shape": list(shape), "data_offsets": [len(blob), len(blob) + len(raw)]}
        blob += raw
    h = json.dumps(header).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)) + h + blob)


def _bf16(v):
    return struct.pack("<I", struct.unpack("<I", struct.pack("<f", v))[0])[2:]


@pytest.mark.parametrize("dtype", ["F32", "BF16"])
@pytest.mark.parametrize("value", [100_000.0, -100_000.0])
def test_rejects_overflowing_weights_before_gpu_initialization(tmp_path, dtype, value):
    """tests/model.rs:29-59: the first packed tensor fails, naming patch_w[0] and float16, before
    any other tensor is read or any GPU is touched (this machine has none: reaching the device
    check would report a device error instead)."""
    n = 384 * 3 * 16 * 16
    size = 4 if dtype == "F32" else 2
    data = bytearray(n * size)
    data[:size] = struct.pack("<f", value) if dtype == "F32" else _bf16(value)
    p = tmp_path / "model.safetensors"
    _write_safetensors(p, {"embeddings.patch_embeddings.weight": (dtype, [384, 3, 16, 16], bytes(data))})
    with pytest.raises(dv.DINOv3Error) as e:
        dv.DINOv3.load(p, dv.Options())
    assert e.value.code == dv.WEIGHTS
    assert "patch_w[0]" in str(e.value) and "finite float16" in str(e.value)


def test_weight_errors_name_the_tensor(tmp_path):
    p = tmp_path / "m.safetensors"
    _write_safetensors(p, {"embeddings.patch_embeddings.weight": ("F32", [384, 3, 16, 15], bytes(384 * 3 * 16 * 15 * 4))})
    with pytest.raises(dv.DINOv3Error) as e:
        dv.DINOv3.load(p, dv.Options())
    assert "embeddings.patch_embeddings.weight: expected [384, 3, 16, 16], found [384, 3, 16, 15]" in str(e.value)
    _write_safetensors(p, {"embeddings.patch_embeddings.weight": ("F32", [384, 3, 16, 16], bytes(384 * 768 * 4))})
    with pytest.raises(dv.DINOv3Error) as e:
        dv.DINOv3.load(p, dv.Options())
    assert "missing tensor embeddings.patch_embeddings.bias" in str(e.value)
    nan = bytearray(384 * 768 * 4)
    nan[4:8] = struct.pack("<f", float("nan"))
    _write_safetensors(p, {"embeddings.patch_embeddings.weight": ("F32", [384, 3, 16, 16], bytes(nan))})
    with pytest.raises(dv.DINOv3Error) as e:
        dv.DINOv3.load(p, dv.Options())
    assert "non-finite tensor embeddings.patch_embeddings.weight" in str(e.value)
    with open(p, "wb") as f:
        f.write(b"\x05")
    with pytest.raises(dv.DINOv3Error) as e:
        dv.DINOv3.load(p, dv.Options())
    assert e.value.code == dv.WEIGHTS


def test_valid_weights_reach_the_device_check(weights_file):
    """A complete file packs without error; without a GPU the load then stops at the device."""
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(dv.DINOv3Error) as e:
        dv.DINOv3.load(weights_file(0, "stress"), dv.Options())
    assert e.value.code == dv.DEVICE


@pytest.mark.parametrize("dtype", ["F16", "BF16"])
def test_low_precision_checkpoints_pack(weights_file_lowp, dtype):
    """src/weights.rs:19-51 accepts F16 and BF16 tensors: a complete file of either packs without
    error; without a GPU the load then stops at the device."""
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    low, _ = weights_file_lowp(dtype)
    with pytest.raises(dv.DINOv3Error) as e:
        dv.DINOv3.load(low, dv.Options())
    assert e.value.code == dv.DEVICE


def test_packing_preserves_finite_values_at_float16_limits():
    """src/weights.rs:148-169: 65519 rounds to 65504; -0 keeps its sign."""
    out = dv.pack_f16("weights", [0.0, -0.0, 1.0, -1.0, 65504.0, -65504.0, 65519.0, -65519.0])
    assert out.astype(np.float32).tolist() == [0, -0.0, 1, -1, 65504, -65504, 65504, -65504]
    assert np.signbit(out[1])


def test_packing_rounds_like_ieee_and_fails_on_overflow():
    rng = np.random.default_rng(0)
    v = np.concatenate([
        rng.standard_normal(20000).astype(np.float32) * 0.02,
        rng.standard_normal(20000).astype(np.float32) * 1e-6,  # f16 subnormals
        (rng.random(2000) * 65519).astype(np.float32),
        np.array([6.1035156e-05, 5.9604645e-08, 2.9802322e-08, 2.9802326e-08, 65519.996], np.float32),
    ])
    got = dv.pack_f16("t", v)
    np.testing.assert_array_equal(got.view(np.uint16), v.astype(np.float16).view(np.uint16))
    with pytest.raises(dv.DINOv3Error) as e:
        dv.pack_f16("blk", np.array([1.0, 2.0, 65520.0], np.float32))
    assert "tensor blk[2] cannot be represented as finite float16: 65520" in str(e.value)


def test_gateup_packing_is_a_permutation_of_gate_then_up():
    lib = _lib.load()
    src = [lib.dv3k_gateup_source_row(r) for r in range(3072)]
    assert sorted(src) == list(range(3072))
    for r in range(3072):
        block, within = divmod(r, 128)
        want = block * 64 + within if within < 64 else 1536 + block * 64 + within - 64
        assert src[r] == want


def test_kernel_entry_points_check_arguments_without_launching():
    lib = _lib.load()
    assert lib.dv3k_layernorm_f16(None, 0, None, None, None, None) == 0  # rows 0: no launch
    assert lib.dv3k_attention(None, 0, None, None, None) == 0
    buf = ctypes.create_string_buffer(1024)
    base = (ctypes.addressof(buf) + 15) & ~15
    rc = lib.dv3k_matmul_resid(base, 201, 100, base, base, base, base, None, None)
    assert rc == dv.INVALID_ARGUMENT and "k must be 384 or 1536" in _lib.last_error()
    rc = lib.dv3k_attention(base, 200, base, None, None)
    assert rc == dv.INVALID_ARGUMENT and "multiple of 201" in _lib.last_error()
    rc = lib.dv3k_layernorm_f16(base + 2, 8, base, base, base, None)
    assert rc == dv.INVALID_ARGUMENT and "aligned" in _lib.last_error()


def test_null_model_is_an_error():
    lib = _lib.load()
    assert lib.dv3_forward(None, None, 0, None, 0) == dv.INVALID_ARGUMENT
    assert lib.dv3_run(None, 1) == dv.INVALID_ARGUMENT
    lib.dv3_free(None)


HUB_SNAPSHOT = ("models--facebook--dinov3-vits16plus-pretrain-lvd1689m/snapshots/"
                "c93d816fc9e567563bc068f01475bec89cc634a6/model.safetensors")


def test_hub_offline_miss_then_cached_hit(tmp_path, monkeypatch):
    """src/hub.rs:60-81: an offline miss names the file and says it is not cached; once the pinned
    snapshot file exists, both offline and online lookups return it without a server."""
    monkeypatch.setenv("HF_HUB_CACHE", str(tmp_path))
    monkeypatch.delenv("HF_HUB_OFFLINE", raising=False)
    with pytest.raises(dv.DINOv3Error) as e:
        dv.hub_weights(offline=True)
    assert e.value.code == dv.WEIGHTS
    assert "not cached" in str(e.value) and "model.safetensors" in str(e.value)
    assert "c93d816fc9e567563bc068f01475bec89cc634a6" in str(e.value)
    with pytest.raises(dv.DINOv3Error, match="cannot download"):   # no network client here
        dv.hub_weights(offline=False)
    path = tmp_path / HUB_SNAPSHOT
    path.parent.mkdir(parents=True)
    path.write_bytes(b"cached model")
    for offline in (True, False):
        assert dv.hub_weights(offline) == str(path)


@pytest.mark.parametrize("value,offline", [("1", True), ("0", False), ("", False)])
def test_hub_offline_environment(tmp_path, monkeypatch, value, offline):
    monkeypatch.setenv("HF_HUB_CACHE", str(tmp_path))
    monkeypatch.setenv("HF_HUB_OFFLINE", value)
    with pytest.raises(dv.DINOv3Error) as e:
        dv.hub_weights(offline=False)
    assert ("downloads are disabled" in str(e.value)) == offline


def test_hub_cache_directory_order(tmp_path, monkeypatch):
    """HF_HUB_CACHE, else HF_HOME/hub, else XDG_CACHE_HOME/huggingface/hub, else
    ~/.cache/huggingface/hub."""
    for var in ("HF_HUB_CACHE", "HF_HOME", "XDG_CACHE_HOME"):
        monkeypatch.delenv(var, raising=False)
    for base, cache in [("home", "home/.cache/huggingface/hub"),
                        ("xdg", "xdg/huggingface/hub"),
                        ("hf", "hf/hub")]:
        f = tmp_path / cache / HUB_SNAPSHOT
        f.parent.mkdir(parents=True)
        f.write_bytes(b"x")
    monkeypatch.setenv("HOME", str(tmp_path / "home"))
    assert dv.hub_weights(True) == str(tmp_path / "home/.cache/huggingface/hub" / HUB_SNAPSHOT)
    monkeypatch.setenv("XDG_CACHE_HOME", str(tmp_path / "xdg"))
    assert dv.hub_weights(True) == str(tmp_path / "xdg/huggingface/hub" / HUB_SNAPSHOT)
    monkeypatch.setenv("HF_HOME", str(tmp_path / "hf"))
    assert dv.hub_weights(True) == str(tmp_path / "hf/hub" / HUB_SNAPSHOT)
    monkeypatch.setenv("HF_HUB_CACHE", str(tmp_path / "xdg/huggingface/hub"))
    assert dv.hub_weights(True) == str(tmp_path / "xdg/huggingface/hub" / HUB_SNAPSHOT)


def test_hub_path_buffer_too_small(tmp_path, monkeypatch):
    monkeypatch.setenv("HF_HUB_CACHE", str(tmp_path))
    f = tmp_path / HUB_SNAPSHOT
    f.parent.mkdir(parents=True)
    f.write_bytes(b"x")
    buf = ctypes.create_string_buffer(8)
    assert _lib.load().dv3_hub_weights(1, buf, len(buf)) == dv.INVALID_ARGUMENT
    assert "too small" in _lib.last_error()


def test_from_pretrained_checks_options_then_the_cache(tmp_path, monkeypatch, weights_file):
    """src/lib.rs:40-46: max_batch first, then the cache lookup, then DINOv3::load (which stops at
    the device check on a machine without a GPU)."""
    import torch

    monkeypatch.setenv("HF_HUB_CACHE", str(tmp_path))
    monkeypatch.setenv("HF_HUB_OFFLINE", "1")
    with pytest.raises(dv.DINOv3Error, match=r"max_batch must be 1\.\.=64"):
        dv.DINOv3.from_pretrained(dv.Options(0, 65))
    with pytest.raises(dv.DINOv3Error, match="not cached") as e:
        dv.DINOv3.from_pretrained(dv.Options())
    assert e.value.code == dv.WEIGHTS
    if torch.cuda.is_available():
        return
    f = tmp_path / HUB_SNAPSHOT
    f.parent.mkdir(parents=True)
    f.symlink_to(weights_file(0, "baseline"))   # the cache's snapshot entries are symlinks
    with pytest.raises(dv.DINOv3Error) as e:
        dv.DINOv3.from_pretrained(dv.Options())
    assert e.value.code == dv.DEVICE
