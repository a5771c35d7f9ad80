"""The whole forward through the model C ABI (include/dinov3.h) against the float64 oracle, and
the reference's GPU-test properties (tests/model.rs:61-99):
  * all-token and CLS cosine > 0.9999 per image vs the float64 forward, plus a stated max-abs
    error bound (MAX_ABS below);
  * batched vs single-image cosine > 0.99999;
  * bitwise repeat determinism;
  * incomplete and non-finite input are errors, and the session stays usable after them.
Weights: seeded random-init ("baseline" = the benchmark distribution; "stress" = nonzero
biases, gammas, betas and per-channel LayerScale, so every epilogue term is exercised).
"""
import glob
import os

import numpy as np
import pytest

import ref_c
import ref_numpy
from dinov3_b200 import synth

from conftest import GOLDEN

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

import dinov3_b200 as dv  # noqa: E402

# Largest |gpu - float64| over every output element allowed in these tests (outputs are
# LayerNorm-normalised, O(1)); f16 weights and activations with f32 accumulation. The largest
# error seen over every image of batches of 32 and 64 is 0.020 (stress weights) and 0.018
# (baseline weights).
MAX_ABS = 0.03
MAX_ABS_FULL = MAX_ABS


@pytest.fixture(scope="module")
def models(weights_file):
    cache = {}

    def get(flavor="baseline", max_batch=4, seed=None):
        seed = {"baseline": 0, "stress": 1}[flavor] if seed is None else seed
        key = (flavor, max_batch, seed)
        if key not in cache:
            cache[key] = dv.DINOv3.load(weights_file(seed, flavor), dv.Options(0, max_batch))
        return cache[key]

    yield get
    for m in cache.values():
        m.close()


@pytest.fixture(scope="module")
def oracles(weights_dict):
    cache = {}

    def get(flavor):
        if flavor not in cache:
            seed = {"baseline": 0, "stress": 1}[flavor]
            cache[flavor] = ref_c.Model(weights_dict(seed, flavor))
        return cache[flavor]

    return get


def cos(a, b):
    return ref_numpy.cosine(a, b)


@pytest.mark.parametrize("flavor", ["baseline", "stress"])
def test_full_reference_and_changing_batch(models, oracles, flavor):
    """tests/model.rs:61-99 with seeded weights and the reference test's own input."""
    model = models(flavor, max_batch=4)
    images = synth.reference_test_images(4)
    batched = model.forward(images)
    want = oracles(flavor).forward(images, threads=0)
    for i in range(4):
        got = model.forward(images[i:i + 1])[0]
        assert cos(got, want[i]) > 0.9999, f"full image {i}"
        assert cos(got[0], want[i][0]) > 0.9999, f"CLS image {i}"
        assert cos(batched[i], got) > 0.99999, f"batch image {i}"
        assert np.abs(got - want[i]).max() < MAX_ABS
    np.testing.assert_array_equal(model.forward(images), batched)  # bitwise repeat
    with pytest.raises(dv.DINOv3Error) as e:
        model.forward(np.zeros(3, np.float32))
    assert "complete 3×224×224 images" in str(e.value)
    with pytest.raises(dv.DINOv3Error) as e:
        model.forward(np.full((1, 3, 224, 224), np.nan, np.float32))
    assert "input must be finite" in str(e.value)
    np.testing.assert_array_equal(model.forward(images), batched)  # still usable


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLDEN, "*.npz"))), ids=os.path.basename)
def test_gpu_matches_golden_fixtures(models, path):
    g = np.load(path)
    model = models(str(g["flavor"]), max_batch=4, seed=int(g["weight_seed"]))
    img = synth.images(int(g["image_arg"]), 1) if str(g["image_source"]) == "seeded" else synth.reference_test_images(1)
    out = model.forward(img)[0].astype(np.float64)
    rows = g["rows"]
    assert cos(out[rows], g["values"]) > 0.9999
    for i, r in enumerate(rows):
        assert cos(out[r], g["values"][i]) > 0.999, f"row {r}"
    assert np.abs(out[rows] - g["values"]).max() < MAX_ABS
    np.testing.assert_allclose(np.linalg.norm(out, axis=1), g["row_norms"], rtol=2e-3)


def test_seeded_images_against_oracle_with_error_bound(models, oracles):
    model = models("stress", max_batch=4)
    images = synth.images(123, 3)
    got = model.forward(images)
    want = oracles("stress").forward(images, threads=0)
    err = np.abs(got - want)
    for i in range(3):
        assert cos(got[i], want[i]) > 0.9999
        assert cos(got[i, 0], want[i, 0]) > 0.9999
    assert err.max() < MAX_ABS, err.max()


def test_chunking_matches_single_images(models):
    """5 images through max_batch=2 (chunks 2, 2, 1) equal per-image forwards bitwise, except
    that batch size 1 and 2 are different graphs, so compare against the same chunk sizes."""
    model = models("stress", max_batch=2)
    images = synth.images(7, 5)
    out = model.forward(images)
    np.testing.assert_array_equal(out[:2], model.forward(images[:2]))
    np.testing.assert_array_equal(out[2:4], model.forward(images[2:4]))
    np.testing.assert_array_equal(out[4:], model.forward(images[4:]))
    for i in range(5):
        assert cos(out[i], model.forward(images[i:i + 1])[0]) > 0.99999


def test_chunked_full_capacity_against_oracle(models, oracles):
    """130 images through the full resident capacity (max_batch 64: chunks of 64, 64 and 2,
    so two plans): the chunks equal their own forwards bitwise, cls and patch_mean read the same
    tokens, and images from every chunk (first and last of each) match the float64 oracle."""
    model = models("baseline", max_batch=64)
    images = synth.images(9000, 130)
    out = model.forward(images)
    assert out.shape == (130, 201, 384) and np.isfinite(out).all()
    np.testing.assert_array_equal(out[128:], model.forward(images[128:]))
    np.testing.assert_array_equal(out[64:128], model.forward(images[64:128]))
    np.testing.assert_array_equal(model.cls(images), out[:, 0])
    pm = model.patch_mean(images)
    want_pm = np.zeros((130, 384), np.float32)
    for r in range(5, 201):  # src/lib.rs:134-148 accumulation order
        want_pm += out[:, r] / np.float32(196.0)
    np.testing.assert_array_equal(pm, want_pm)
    picks = [0, 63, 64, 127, 128, 129]
    want = oracles("baseline").forward(images[picks], threads=0)
    for got, ref in zip(out[picks], want):
        assert cos(got, ref) > 0.9999 and cos(got[0], ref[0]) > 0.9999
        assert np.abs(got - ref).max() < MAX_ABS
    # a non-finite pixel in the second chunk is an argument error (the earlier chunk has run;
    # the output is unspecified on error) and the model stays usable
    bad = images.copy()
    bad[100, 2, 50, 60] = np.inf
    with pytest.raises(dv.DINOv3Error) as e:
        model.forward(bad)
    assert e.value.code == dv.INVALID_ARGUMENT and "input must be finite" in str(e.value)
    np.testing.assert_array_equal(model.forward(images[128:]), out[128:])


def test_cls_and_patch_mean(models):
    """cls reads back only row 0 of each image and patch_mean reduces on the device; both equal
    the reference's host arithmetic on the full output bit for bit, also across chunks."""
    model = models("stress", max_batch=4)
    images = synth.images(8, 6)
    full = model.forward(images)
    np.testing.assert_array_equal(model.cls(images), full[:, 0])
    pm = model.patch_mean(images)
    want = np.zeros((6, 384), np.float32)
    for r in range(5, 201):  # src/lib.rs:134-148 accumulation order
        want += full[:, r] / np.float32(196.0)
    np.testing.assert_array_equal(pm, want)


def test_empty_input_returns_empty(models):
    model = models("baseline", max_batch=4)
    assert model.forward(np.zeros(0, np.float32)).shape == (0, 201, 384)


def test_device_path_matches_host_path(models):
    model = models("stress", max_batch=4)
    images = synth.images(9, 3)
    host = model.forward(images)
    dev = model.forward_device(torch.from_numpy(images).cuda())
    np.testing.assert_array_equal(dev.cpu().numpy(), host)
    # staged input + graph replay + resident output
    inp = device_view(model.input_buffer, 3 * 3 * 224 * 224)
    inp.copy_(torch.from_numpy(images).reshape(-1))
    torch.cuda.synchronize()
    model.run(3)
    model.synchronize()
    out = device_view(model.output_buffer, 3 * 201 * 384).cpu().numpy()
    np.testing.assert_array_equal(out.reshape(3, 201, 384), host)


class _DeviceArray:
    def __init__(self, ptr, n):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (ptr, False), "version": 3}


def device_view(ptr, n):
    """A torch view (no copy) of n float32 at a device address owned by the model."""
    return torch.as_tensor(_DeviceArray(ptr, n), device="cuda")


@pytest.mark.parametrize("source", ["seeded", "reference"])
def test_full_size_batch_properties(models, oracles, source):
    """Batch 64 (the benchmark configuration), on seeded images and on the reference test's own
    input pattern (tests/model.rs:72-74): per-image results match single-image forwards, two
    images match the oracle, and repeats are bitwise identical."""
    model = models("baseline", max_batch=64)
    images = synth.images(2024, 64) if source == "seeded" else synth.reference_test_images(64)
    # batch 64 fuses the LayerNorms into the residual GEMMs; single images use the split plan
    assert model.launches_per_forward(64) == 3 + 12 * 5
    assert model.launches_per_forward(1) == 3 + 12 * 7
    out = model.forward(images)
    assert np.isfinite(out).all()
    for i in (0, 17, 63):
        assert cos(out[i], model.forward(images[i:i + 1])[0]) > 0.99999
    want = oracles("baseline").forward(images[[5, 63]], threads=0)
    assert cos(out[5], want[0]) > 0.9999 and cos(out[63], want[1]) > 0.9999
    np.testing.assert_array_equal(model.forward(images), out)


@pytest.mark.parametrize("flavor,batch,source", [
    ("baseline", 32, "seeded"), ("baseline", 32, "reference"),
    ("baseline", 64, "seeded"), ("baseline", 64, "reference"), ("stress", 64, "seeded")])
def test_every_image_of_full_batches_against_oracle(models, oracles, flavor, batch, source):
    """BASELINE config 1 (batch 32 with the default Options, resident capacity 32) and config 2
    (batch 64, capacity 64, the benchmark's plan): every image of the batch against the float64
    oracle, all-token and CLS cosine > 0.9999 each, and every output element within
    MAX_ABS_FULL, as tests/model.rs:75-94 checks every image of its batch."""
    model = models(flavor, max_batch=batch)
    # both run the full-row residual GEMMs with the LayerNorms folded (from 32 images on)
    assert model.launches_per_forward(batch) == 3 + 12 * 5
    images = synth.images(5000 + batch, batch) if source == "seeded" else \
        synth.reference_test_images(batch)
    out = model.forward(images)
    want = oracles(flavor).forward(images, threads=0)
    worst = []
    for i in range(batch):
        c_all, c_cls = cos(out[i], want[i]), cos(out[i, 0], want[i, 0])
        worst.append((c_all, c_cls, float(np.abs(out[i] - want[i]).max())))
        assert c_all > 0.9999, f"image {i}: all-token cosine {c_all}"
        assert c_cls > 0.9999, f"image {i}: CLS cosine {c_cls}"
    err = max(w[2] for w in worst)
    print(f"{flavor} b={batch} {source}: min all-token cosine {min(w[0] for w in worst):.8f}, "
          f"min CLS cosine {min(w[1] for w in worst):.8f}, max |err| {err:.5f}")
    assert err < MAX_ABS_FULL


def test_injected_device_failure_poisons_the_session(weights_file):
    """A device failure poisons the model (src/engine.rs:93,168-171,198-200): the forward that
    saw it returns DV3_POISONED with the reference's message, and so does every later call. The
    failure is injected on the host (dv3_debug_inject_fault writes the failure bits an expired
    device wait would record), so no GPU fault is made."""
    path = weights_file(1, "stress")
    images = synth.images(61, 2)
    pin_in = torch.from_numpy(images).pin_memory()
    pin_out = torch.empty((2, 201, 384), dtype=torch.float32).pin_memory()

    def poisoned(call):
        with pytest.raises(dv.DINOv3Error) as e:
            call()
        assert e.value.code == dv.POISONED, str(e.value)
        assert "session is unusable after a GPU failure" in str(e.value)

    # synchronous forward
    with dv.DINOv3.load(path, dv.Options(0, 4)) as model:
        want = model.forward(images)
        model.debug_inject_fault(1 << 30)
        poisoned(lambda: model.forward(images))
        poisoned(lambda: model.forward(images))
        poisoned(lambda: model.cls(images))
        poisoned(lambda: model.patch_mean(images))
        poisoned(lambda: model.run(2))
        poisoned(lambda: model.submit(pin_in, pin_out))
        poisoned(lambda: model.debug_inject_fault(1))
    # device-resident replay: the failure is reported by the next synchronize
    with dv.DINOv3.load(path, dv.Options(0, 4)) as model:
        np.testing.assert_array_equal(model.forward(images), want)  # stages the input
        model.run(2)
        model.synchronize()
        model.debug_inject_fault(1 << 30)
        model.run(2)
        poisoned(model.synchronize)
        poisoned(lambda: model.run(2))
        poisoned(lambda: model.forward(images))
    # serving path: a non-finite submission is an argument error and does not poison; the
    # faulted submission reports DV3_POISONED and the model stays poisoned
    with dv.DINOv3.load(path, dv.Options(0, 4)) as model:
        bad = images.copy()
        bad[1, 2, 3, 4] = np.nan
        bad_in = torch.from_numpy(bad).pin_memory()
        outs = [torch.empty((2, 201, 384), dtype=torch.float32).pin_memory() for _ in range(3)]
        tb = model.submit(bad_in, outs[0])
        with pytest.raises(dv.DINOv3Error) as e:
            model.wait(tb)
        assert e.value.code == dv.INVALID_ARGUMENT and "input must be finite" in str(e.value)
        tg = model.submit(pin_in, outs[1])
        model.wait(tg)
        np.testing.assert_array_equal(outs[1].numpy(), want)
        model.debug_inject_fault(1 << 30)
        tf = model.submit(pin_in, outs[2])
        poisoned(lambda: model.wait(tf))
        poisoned(lambda: model.submit(pin_in, outs[2]))
        poisoned(lambda: model.forward(images))


def test_profile_forward_in_plan_order(models):
    """dv3_profile_forward times every launch inside whole forwards (L2 flushed before each)
    as the differences of timed graphs of the plan's first j launches: the plan's launches in
    order, and their sum is one forward."""
    model = models("baseline", max_batch=64)
    images = synth.images(17, 64)
    model.forward(images)  # stages the input
    prof = model.profile_forward(64, 3, 256 << 20)
    assert len(prof) == model.launches_per_forward(64)
    # batch 64 folds the first LayerNorm into the QKV GEMM: only its row statistics
    assert [n for n, _ in prof][:3] == ["patchify", "gemm_patch_embed", "layernorm_rowstat"]
    gemms = [ms for n, ms in prof if n.startswith("gemm_gateup")]
    assert len(gemms) == 12 and all(ms > 0.005 for ms in gemms)
    total = sum(ms for _, ms in prof)
    assert 0.3 < total < 5.0, total  # ms for a batch-64 forward
    with pytest.raises(dv.DINOv3Error):
        model.profile_forward(65, 1)


@pytest.mark.parametrize("b", [12, 40])
def test_mid_size_batch_plans(models, oracles, b):
    """Batch sizes between the batch-1 and batch-64 plans: 12 images run the down projection as 2
    K slices and attention as one CTA per query tile; 40 images run 128-wide residual tiles with
    narrow 128x64 units for their partial second wave and QKV with a partial last wave. Every
    image matches its single-image forward, two match the float64 oracle, repeats are bitwise."""
    model = models("stress", max_batch=64)
    images = synth.images(300 + b, b)
    out = model.forward(images)
    assert np.isfinite(out).all()
    for i in (0, b // 2, b - 1):
        assert cos(out[i], model.forward(images[i:i + 1])[0]) > 0.99999, f"image {i}"
    want = oracles("stress").forward(images[[1, b - 2]], threads=0)
    for got, ref in zip(out[[1, b - 2]], want):
        assert cos(got, ref) > 0.9999 and cos(got[0], ref[0]) > 0.9999
        assert np.abs(got - ref).max() < MAX_ABS
    np.testing.assert_array_equal(model.forward(images), out)


def test_every_batch_size_matches_single_images(models, oracles):
    """Every resident batch size 1..64 (each crosses its own mix of plan variants: split-K down
    projection up to 15 images, one attention CTA per query tile up to 12, narrow GEMM units,
    full-row residual GEMMs with the folded LayerNorms from 32): each image of a batch matches that image's
    single-image forward, and two images of the largest batch match the float64 oracle."""
    model = models("stress", max_batch=64)
    images = synth.images(4096, 64)
    single = np.stack([model.forward(images[i:i + 1])[0] for i in range(64)])
    for b in range(1, 65):
        out = model.forward(images[:b])
        assert np.isfinite(out).all(), f"batch {b}"
        for i in range(b):
            assert cos(out[i], single[i]) > 0.99999, f"batch {b} image {i}"
            assert cos(out[i][0], single[i][0]) > 0.99999, f"batch {b} image {i} CLS"
    want = oracles("stress").forward(images[[0, 63]], threads=0)
    for got, ref in zip(out[[0, 63]], want):
        assert cos(got, ref) > 0.9999 and np.abs(got - ref).max() < MAX_ABS


@pytest.mark.parametrize("dtype", ["F16", "BF16"])
def test_low_precision_checkpoint_forward(weights_file_lowp, dtype):
    """An F16 or BF16 checkpoint packs to the same device weights as an F32 file holding the same
    values, so the forwards agree bit for bit (src/weights.rs:19-51)."""
    low, f32 = weights_file_lowp(dtype)
    images = synth.images(77, 3)
    with dv.DINOv3.load(low, dv.Options(0, 4)) as model:
        got = model.forward(images)
    with dv.DINOv3.load(f32, dv.Options(0, 4)) as model:
        want = model.forward(images)
    assert np.isfinite(got).all()
    np.testing.assert_array_equal(got, want)


def test_benchmark_and_profile(models):
    model = models("baseline", max_batch=4)
    images = synth.images(3, 2)
    t = model.benchmark(images, 10)
    assert t.samples == 10 and 0 < t.graph.median_ms <= t.graph.p95_ms
    assert 0 < t.direct.median_ms <= t.direct.p95_ms
    with pytest.raises(dv.DINOv3Error):
        model.benchmark(images, 5)
    with pytest.raises(dv.DINOv3Error):
        model.benchmark(np.zeros(0, np.float32), 10)
    prof = model.profile_launches(2, 2)
    # small batches: patchify, patch GEMM, LN1 of layer 0, then per layer QKV, attention, o,
    # LN2, gate/up, and the down projection as a split-K GEMM plus a reduce that also does the
    # LayerNorm after it (the reference's plan, src/lib.rs:149-263, has 87 launches too)
    assert len(prof) == model.launches_per_forward(2) == 3 + 12 * 7
    assert all(ms > 0 for _, ms in prof)
    names = [name for name, _ in prof]
    assert sum(n.startswith("layernorm") for n in names) == 1 + 12
    assert names.count("gemm_down_splitk") == names.count("splitk_reduce_layernorm") == 12


def test_fused_layernorm_plan(weights_file, monkeypatch):
    """Large batches ride each LayerNorm after the first in the preceding residual GEMM
    (3 + 12*5 launches) and fold all but the final one further into the QKV and gate/up GEMMs
    (the residual GEMM leaves only the row statistics); small ones keep separate LayerNorm
    launches (3 + 12*7, the reference's plan). At 16 images the default is the split plan;
    DV3_FUSE_LAYERNORM=1 (read when a batch size's graph is built) forces fusion and folding,
    DV3_FOLD_LAYERNORM=0 keeps the fused LayerNorms unfolded. All three give the same result
    within f16 rounding."""
    path = weights_file(1, "stress")
    images = synth.images(31, 16)
    with dv.DINOv3.load(path, dv.Options(0, 16)) as model:
        assert model.launches_per_forward(16) == 3 + 12 * 7
        split = model.forward(images)
    monkeypatch.setenv("DV3_FUSE_LAYERNORM", "1")
    monkeypatch.setenv("DV3_FOLD_LAYERNORM", "0")
    with dv.DINOv3.load(path, dv.Options(0, 16)) as model:
        assert model.launches_per_forward(16) == 3 + 12 * 5
        fused = model.forward(images)
        names = [n for n, _ in model.profile_launches(16, 1)]
    assert names.count("gemm_down_resid_layernorm") == 12
    assert names.count("gemm_o_resid_layernorm") == 12 and names[2] == "layernorm_f16"
    monkeypatch.delenv("DV3_FOLD_LAYERNORM")
    with dv.DINOv3.load(path, dv.Options(0, 16)) as model:
        assert model.launches_per_forward(16) == 3 + 12 * 5
        folded = model.forward(images)
        names = [n for n, _ in model.profile_launches(16, 1)]
    assert names[2] == "layernorm_rowstat"
    assert names.count("gemm_qkv_rope_folded") == names.count("gemm_o_resid_rowstat") == 12
    assert names.count("gemm_gateup_swiglu_folded") == 12
    assert names.count("gemm_down_resid_rowstat") == 11  # the final LayerNorm is not folded
    assert names[-1] == "gemm_down_resid_layernorm"
    for i in range(16):
        assert cos(fused[i], split[i]) > 0.99999
        assert cos(folded[i], split[i]) > 0.99999


def test_split_k_plan(weights_file, monkeypatch):
    """Small batches split the down projection's K (and fuse the LayerNorm after it into the
    reduce); DV3_SPLITK=0 (read when a batch size's graph is built) keeps the unsplit GEMM and a
    separate LayerNorm. Both give the same result within f32 summation order and f16 rounding."""
    path = weights_file(1, "stress")
    images = synth.images(33, 3)
    with dv.DINOv3.load(path, dv.Options(0, 4)) as model:
        names = [n for n, _ in model.profile_launches(3, 1)]
        assert names.count("gemm_down_splitk") == 12
        split = model.forward(images)
    monkeypatch.setenv("DV3_SPLITK", "0")
    with dv.DINOv3.load(path, dv.Options(0, 4)) as model:
        names = [n for n, _ in model.profile_launches(3, 1)]
        assert names.count("gemm_down_resid") == 12 and "gemm_down_splitk" not in names
        plain = model.forward(images)
    for i in range(3):
        assert cos(split[i], plain[i]) > 0.99999


def test_submit_wait_serving_path(models):
    """Serving path (dv3_submit / dv3_wait): submissions of changing size, two in flight and a
    third that first completes the oldest, waited out of order, give exactly the synchronous
    forward's outputs; a non-finite submission reports its own error and leaves the model and
    the other submissions usable; a waited ticket cannot be waited again."""
    import torch

    model = models("stress", max_batch=4)
    sizes = [3, 1, 4, 2, 4]
    imgs = [synth.images(100 + i, k) for i, k in enumerate(sizes)]
    want = [model.forward(x) for x in imgs]
    ins = [torch.from_numpy(x).pin_memory() for x in imgs]
    outs = [torch.empty((k, 201, 384), dtype=torch.float32).pin_memory() for k in sizes]
    t = [model.submit(ins[i], outs[i]) for i in range(3)]
    model.wait(t[1])
    model.wait(t[0])
    model.wait(t[2])
    t3 = model.submit(ins[3], outs[3])
    t4 = model.submit(ins[4], outs[4])
    model.wait(t3)
    model.wait(t4)
    for o, w in zip(outs, want):
        np.testing.assert_array_equal(o.numpy(), w)
    with pytest.raises(dv.DINOv3Error):
        model.wait(t4)
    bad = imgs[0].copy()
    bad[1, 2, 3, 4] = np.nan
    bad_out = torch.empty((3, 201, 384), dtype=torch.float32).pin_memory()
    tb = model.submit(torch.from_numpy(bad).pin_memory(), bad_out)
    outs[1].zero_()
    tg = model.submit(ins[1], outs[1])
    with pytest.raises(dv.DINOv3Error, match="finite"):
        model.wait(tb)
    model.wait(tg)
    np.testing.assert_array_equal(outs[1].numpy(), want[1])
    # synchronous calls after asynchronous ones
    np.testing.assert_array_equal(model.forward(imgs[2]), want[2])
