"""The float64 oracle (oracle/ref_numpy.py and oracle/ref_c.py) against the golden fixtures and
the reference's own known-answer tests. CPU only."""
import glob
import hashlib
import os

import numpy as np
import pytest

import ref_c
import ref_numpy
from dinov3_b200 import synth

from conftest import GOLDEN

CASES = sorted(glob.glob(os.path.join(GOLDEN, "*.npz")))


def _digest(d):
    h = hashlib.sha256()
    for k in sorted(d):
        h.update(k.encode())
        h.update(np.ascontiguousarray(d[k], dtype=np.float32).tobytes())
    return h.hexdigest()


def _case(path, weights_dict):
    g = np.load(path)
    w = weights_dict(int(g["weight_seed"]), str(g["flavor"]))
    if str(g["image_source"]) == "seeded":
        img = synth.images(int(g["image_arg"]), 1)[0]
    else:
        img = synth.reference_test_images(1)[0]
    return g, w, img


def _check(out, g, tol):
    rows = g["rows"]
    assert np.abs(out[rows] - g["values"]).max() < tol
    assert np.abs(np.linalg.norm(out, axis=1) - g["row_norms"]).max() < tol
    assert abs(out.sum() - float(g["total"])) < tol * 100


def test_fixtures_present():
    assert len(CASES) >= 3


@pytest.mark.parametrize("path", CASES, ids=os.path.basename)
def test_generator_matches_fixture_inputs(path, weights_dict):
    g, w, img = _case(path, weights_dict)
    assert _digest(w) == str(g["weights_sha256"])
    assert _digest({"image": img}) == str(g["image_sha256"])


@pytest.mark.parametrize("path", CASES, ids=os.path.basename)
def test_numpy_oracle_matches_golden(path, weights_dict):
    g, w, img = _case(path, weights_dict)
    _check(ref_numpy.forward(w, img), g, 1e-11)


@pytest.mark.parametrize("path", CASES[:2], ids=os.path.basename)
def test_c_oracle_matches_golden(path, weights_dict):
    g, w, img = _case(path, weights_dict)
    out = ref_c.Model(w).forward(img[None], threads=2)[0]
    _check(out, g, 1e-11)


def test_c_oracle_batch_matches_single(weights_dict):
    w = weights_dict(1, "stress")
    imgs = synth.images(11, 3)
    m = ref_c.Model(w)
    batch = m.forward(imgs, threads=3)
    for i in range(3):
        np.testing.assert_array_equal(batch[i], m.forward(imgs[i:i + 1], threads=1)[0])


def test_patchify_preserves_channel_and_spatial_order():
    """src/lib.rs:304-328: dst=(((gy*14+gx)*3+c)*16+dy)*16+dx <- src=(c*224+gy*16+dy)*224+gx*16+dx."""
    image = np.arange(3 * 224 * 224, dtype=np.float32).reshape(3, 224, 224)
    gy, gx, c, dy, dx = np.meshgrid(*(np.arange(n) for n in (14, 14, 3, 16, 16)), indexing="ij")
    dst = ((((gy * 14 + gx) * 3 + c) * 16 + dy) * 16 + dx).ravel()
    src = ((c * 224 + gy * 16 + dy) * 224 + gx * 16 + dx).ravel()
    for out in (ref_numpy.patchify(image).ravel(), ref_c.patchify(image).ravel()):
        assert np.array_equal(out[dst], image.ravel()[src].astype(np.float64))


def test_rope_tables_match_packed_layout():
    """The rotation's per-channel cos/sin equal the reference's packed table, whose 64 entries per
    patch are [row freqs 0..15, column freqs 0..15, row, column] (src/weights.rs:127-144)."""
    packed_cos, packed_sin = [], []
    for y in range(14):
        for x in range(14):
            for _ in range(2):
                for pos in (y, x):
                    for j in range(16):
                        a = 2 * np.pi * (2 * (pos + 0.5) / 14 - 1) / 100 ** (j / 16)
                        packed_cos.append(np.cos(a))
                        packed_sin.append(np.sin(a))
    packed_cos = np.array(packed_cos).reshape(196, 64)
    packed_sin = np.array(packed_sin).reshape(196, 64)
    for cos, sin in (ref_numpy.rope_tables(), ref_c.rope_tables()):
        np.testing.assert_allclose(cos, packed_cos, atol=1e-15)
        np.testing.assert_allclose(sin, packed_sin, atol=1e-15)


def test_oracles_agree_on_reference_test_input(weights_dict):
    """The reference's GPU-test input sin(0.037 i)*0.6 (tests/model.rs:72-74), numpy vs C."""
    w = weights_dict(0, "baseline")
    img = synth.reference_test_images(1)[0]
    a = ref_numpy.forward(w, img)
    b = ref_c.Model(w).forward(img[None], threads=2)[0]
    assert np.abs(a - b).max() < 1e-11
