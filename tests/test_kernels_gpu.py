"""Each sm_100a kernel, called through the per-kernel C ABI (include/dinov3_kernels.h), against
a float64 numpy restatement of the same op on the same f16 inputs.

Tolerances: outputs stored as f16 may differ from the float64 value rounded to f16 by one f16
rounding step plus the f32-accumulation difference, so |gpu - ref| <= 4e-3 * max(1, |ref|);
patchify is a pure conversion and must be bit-exact.
"""
import numpy as np
import pytest

import ref_numpy

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

from dinov3_b200 import _lib  # noqa: E402

DEV = "cuda:0"


def lib():
    return _lib.load()


def t16(a):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float16)).to(DEV)


def t32(a):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(DEV)


def status():
    return torch.zeros(2, dtype=torch.int32, device=DEV)


_KEEP = []


def ptr(t):
    """Device address of `t`, holding a reference until the test ends: a temporary freed at once
    would hand its memory to the next allocation before the asynchronous kernel reads it."""
    if t is None:
        return None
    _KEEP.append(t)
    return t.data_ptr()


@pytest.fixture(autouse=True)
def _keepalive():
    yield
    torch.cuda.synchronize()
    _KEEP.clear()


def stream():
    return torch.cuda.current_stream().cuda_stream


def check_rc(rc):
    assert rc == 0, _lib.last_error()


def assert_close16(got, ref):
    got = got.float().cpu().numpy().astype(np.float64)
    err = np.abs(got - ref) / np.maximum(1.0, np.abs(ref))
    assert err.max() <= 4e-3, f"max scaled error {err.max():.3e}"


def rows_of(b):
    return 201 * b


def f16(a):
    return np.asarray(a, dtype=np.float16).astype(np.float64)


@pytest.mark.parametrize("b", [1, 3, 64])
def test_layernorm(b):
    rng = np.random.default_rng(b)
    r = rows_of(b)
    x = f16(rng.standard_normal((r, 384)) * 3 + rng.standard_normal((r, 1)))
    g = rng.standard_normal(384) * 0.3 + 1
    be = rng.standard_normal(384) * 0.1
    ref = ref_numpy.norm(x, g.astype(np.float32), be.astype(np.float32))
    xd, gd, bd = t16(x), t32(g), t32(be)
    out16 = torch.empty((r, 384), dtype=torch.float16, device=DEV)
    out32 = torch.empty((r, 384), dtype=torch.float32, device=DEV)
    check_rc(lib().dv3k_layernorm_f16(ptr(xd), r, ptr(gd), ptr(bd), ptr(out16), stream()))
    check_rc(lib().dv3k_layernorm_f32out(ptr(xd), r, ptr(gd), ptr(bd), ptr(out32), stream()))
    torch.cuda.synchronize()
    assert_close16(out16, ref)
    assert np.abs(out32.cpu().numpy() - ref).max() < 1e-4


@pytest.mark.parametrize("b", [1, 2, 5])
def test_patchify_and_prefix(b):
    rng = np.random.default_rng(10 + b)
    imgs = rng.standard_normal((b, 3, 224, 224)).astype(np.float32)
    prefix = rng.standard_normal((5, 384)).astype(np.float32)
    patches = torch.empty((196 * b, 768), dtype=torch.float16, device=DEV)
    x = torch.full((201 * b, 384), 7.0, dtype=torch.float16, device=DEV)
    st = status()
    check_rc(lib().dv3k_patchify(ptr(t32(imgs)), b, ptr(t32(prefix)), ptr(patches), ptr(x), ptr(st), stream()))
    torch.cuda.synchronize()
    want = np.concatenate([ref_numpy.patchify(im) for im in imgs]).astype(np.float16)
    np.testing.assert_array_equal(patches.cpu().numpy().view(np.uint16), want.view(np.uint16))
    xs = x.cpu().numpy().reshape(b, 201, 384)
    for i in range(b):
        np.testing.assert_array_equal(xs[i, :5], prefix.astype(np.float16))
        assert np.all(xs[i, 5:] == 7.0)  # patch rows untouched
    assert st.cpu().tolist() == [0, 0]
    imgs[b - 1, 2, 100, 37] = np.inf
    check_rc(lib().dv3k_patchify(ptr(t32(imgs)), b, ptr(t32(prefix)), ptr(patches), ptr(x), ptr(st), stream()))
    torch.cuda.synchronize()
    assert st.cpu().tolist()[1] != 0


@pytest.mark.parametrize("b", [1, 3, 64])
def test_patch_embed(b):
    rng = np.random.default_rng(20 + b)
    p = 196 * b
    a = f16(rng.standard_normal((p, 768)))
    w = f16(rng.standard_normal((384, 768)) / np.sqrt(768))
    bias = rng.standard_normal(384) * 0.1
    ref = a @ w.T + bias.astype(np.float32)
    x = torch.full((201 * b, 384), -3.0, dtype=torch.float16, device=DEV)
    st = status()
    check_rc(lib().dv3k_patch_embed(ptr(t16(a)), p, ptr(t16(w)), ptr(t32(bias)), ptr(x), ptr(st), stream()))
    torch.cuda.synchronize()
    assert st.cpu().tolist() == [0, 0]
    xs = x.reshape(b, 201, 384)
    assert torch.all(xs[:, :5] == -3.0)  # prefix rows untouched
    assert_close16(xs[:, 5:].reshape(p, 384), ref)


def rope_ref(y, rows):
    cos, sin = ref_numpy.rope_tables()
    cos = cos.astype(np.float32).astype(np.float64)
    sin = sin.astype(np.float32).astype(np.float64)
    y = y.copy()
    for row in range(rows):
        t = row % 201
        if t < 5:
            continue
        c, s = cos[t - 5], sin[t - 5]
        for base in range(0, 768, 64):
            v = y[row, base:base + 64].copy()
            rot = np.concatenate([-v[32:], v[:32]])
            y[row, base:base + 64] = v * c + rot * s
    return y


# From 50 images on, the last 128 columns (the narrow unit of each M tile) run after all full
# 256-wide tiles, partly in the last wave of the persistent CTAs.
@pytest.mark.parametrize("b", [1, 3, 50, 64])
def test_qkv_rope(b):
    rng = np.random.default_rng(30 + b)
    r = rows_of(b)
    h = f16(rng.standard_normal((r, 384)))
    w = f16(rng.standard_normal((1152, 384)) / np.sqrt(384))
    bias = rng.standard_normal(1152) * 0.1
    bias[384:768] = 0
    ref = rope_ref(h @ w.T + bias.astype(np.float32), r)
    cos, sin = ref_numpy.rope_tables()
    out = torch.empty((r, 1152), dtype=torch.float16, device=DEV)
    check_rc(lib().dv3k_qkv_rope(ptr(t16(h)), r, ptr(t16(w)), ptr(t32(bias)), ptr(t32(cos)),
                                 ptr(t32(sin)), ptr(out), ptr(status()), stream()))
    torch.cuda.synchronize()
    assert_close16(out, ref)


def attention_ref(qkv, b):
    out = np.zeros((201 * b, 384))
    for i in range(b):
        blk = qkv[201 * i:201 * (i + 1)]
        for hd in range(6):
            q = blk[:, hd * 64:(hd + 1) * 64]
            k = blk[:, 384 + hd * 64:384 + (hd + 1) * 64]
            v = blk[:, 768 + hd * 64:768 + (hd + 1) * 64]
            s = q @ k.T * 0.125
            e = np.exp(s - s.max(axis=1, keepdims=True))
            out[201 * i:201 * (i + 1), hd * 64:(hd + 1) * 64] = (e / e.sum(axis=1, keepdims=True)) @ v
    return out


# 50 and 64 images give 300 and 384 (image, head) items: each persistent CTA walks 2 or 3 of them.
@pytest.mark.parametrize("b", [1, 3, 8, 50, 64])
def test_attention(b):
    rng = np.random.default_rng(40 + b)
    r = rows_of(b)
    qkv = f16(rng.standard_normal((r, 1152)) * 1.5)
    ref = attention_ref(qkv, b)
    out = torch.full((r, 384), 9.0, dtype=torch.float16, device=DEV)
    st = status()
    check_rc(lib().dv3k_attention(ptr(t16(qkv)), r, ptr(out), ptr(st), stream()))
    torch.cuda.synchronize()
    assert st.cpu().tolist() == [0, 0]
    assert_close16(out, ref)


# From 48 to 94 images the residual GEMM runs on full 384-wide rows (one tile per CTA); fewer
# images take 128-wide tiles (narrow 128x64 units at 1 and 3), 100 images 128-wide tiles with
# narrow units for the partial last wave, like 40 (189 tiles: 148, then 41 as 82 narrow units).
@pytest.mark.parametrize("k", [384, 1536])
@pytest.mark.parametrize("b", [1, 3, 40, 64, 100])
def test_matmul_resid(k, b):
    rng = np.random.default_rng(50 + b + k)
    r = rows_of(b)
    a = f16(rng.standard_normal((r, k)))
    w = f16(rng.standard_normal((384, k)) / np.sqrt(k))
    bias = rng.standard_normal(384) * 0.1
    lam = rng.random(384) * 0.2 + 0.05
    x0 = f16(rng.standard_normal((r, 384)))
    ref = x0 + lam.astype(np.float32) * (a @ w.T + bias.astype(np.float32))
    x = t16(x0)
    check_rc(lib().dv3k_matmul_resid(ptr(t16(a)), r, k, ptr(t16(w)), ptr(t32(bias)), ptr(t32(lam)),
                                     ptr(x), ptr(status()), stream()))
    torch.cuda.synchronize()
    assert_close16(x, ref)


@pytest.mark.parametrize("f32_out", [False, True])
@pytest.mark.parametrize("k", [384, 1536])
@pytest.mark.parametrize("b", [1, 3, 64])
def test_matmul_resid_layernorm(k, b, f32_out):
    rng = np.random.default_rng(70 + b + k + f32_out)
    r = rows_of(b)
    a = f16(rng.standard_normal((r, k)))
    w = f16(rng.standard_normal((384, k)) / np.sqrt(k))
    bias = rng.standard_normal(384) * 0.1
    lam = rng.random(384) * 0.2 + 0.05
    x0 = f16(rng.standard_normal((r, 384)) + rng.standard_normal((r, 1)))
    g = rng.standard_normal(384) * 0.3 + 1
    be = rng.standard_normal(384) * 0.1
    ref_x = x0 + lam.astype(np.float32) * (a @ w.T + bias.astype(np.float32))
    x = t16(x0)
    h = None if f32_out else torch.empty((r, 384), dtype=torch.float16, device=DEV)
    o = torch.empty((r, 384), dtype=torch.float32, device=DEV) if f32_out else None
    st = status()
    check_rc(lib().dv3k_matmul_resid_layernorm(ptr(t16(a)), r, k, ptr(t16(w)), ptr(t32(bias)),
                                               ptr(t32(lam)), ptr(x), ptr(t32(g)), ptr(t32(be)),
                                               ptr(h), ptr(o), ptr(st), stream()))
    torch.cuda.synchronize()
    assert st.cpu().tolist() == [0, 0]
    assert_close16(x, ref_x)
    # the LayerNorm normalises the stored f16 rows
    ref_ln = ref_numpy.norm(x.float().cpu().numpy().astype(np.float64), g.astype(np.float32),
                            be.astype(np.float32))
    if f32_out:
        assert np.abs(o.cpu().numpy() - ref_ln).max() < 1e-4
    else:
        assert_close16(h, ref_ln)


def splitk_reduce_ref(partials, bias, lam, x):
    """kernels/splitk_reduce_f16.loom in float32 with its own rounding order: the slabs onto
    zero in order, + bias, * lambda, + the f16 residual, rounded to f16."""
    acc = np.zeros(partials.shape[1:], np.float32)
    for p in partials.astype(np.float32):
        acc = acc + p
    u = x.astype(np.float32) + (acc + bias.astype(np.float32)) * lam.astype(np.float32)
    return u.astype(np.float16)


# The down projection's K split (the reference splits it in 4 at batch 1): every slab against
# numpy; 3 and 8 images need clipped rows inside each slab (201 and 1608 rows, not multiples of
# 128); the slabs of a row must not spill into the next slab.
@pytest.mark.parametrize("splits", [1, 4, 8])
@pytest.mark.parametrize("b", [1, 3, 8])
def test_matmul_splitk(b, splits):
    rng = np.random.default_rng(80 + b + splits)
    r = rows_of(b)
    a = f16(rng.standard_normal((r, 1536)))
    w = f16(rng.standard_normal((384, 1536)) / np.sqrt(1536))
    parts = torch.full((splits, r, 384), 7.0, dtype=torch.float32, device=DEV)
    st = status()
    check_rc(lib().dv3k_matmul_splitk(ptr(t16(a)), r, ptr(t16(w)), splits, ptr(parts), ptr(st), stream()))
    torch.cuda.synchronize()
    assert st.cpu().tolist() == [0, 0]
    got = parts.cpu().numpy().astype(np.float64)
    ks = 1536 // splits
    for s in range(splits):
        ref = a[:, s * ks:(s + 1) * ks] @ w[:, s * ks:(s + 1) * ks].T
        err = np.abs(got[s] - ref) / np.maximum(1.0, np.abs(ref))
        assert err.max() < 1e-4, (s, err.max())
    with pytest.raises(AssertionError):
        check_rc(lib().dv3k_matmul_splitk(ptr(t16(a)), r, ptr(t16(w)), 5, ptr(parts), ptr(st), stream()))


@pytest.mark.parametrize("splits", [1, 4, 8])
@pytest.mark.parametrize("b", [1, 3])
def test_splitk_reduce_bit_exact(b, splits):
    """The reduce follows the reference's rounding order exactly: bitwise equal to float32 numpy."""
    rng = np.random.default_rng(90 + b + splits)
    r = rows_of(b)
    partials = rng.standard_normal((splits, r, 384)).astype(np.float32)
    bias = (rng.standard_normal(384) * 0.1).astype(np.float32)
    lam = (rng.random(384) * 0.2 + 0.05).astype(np.float32)
    x0 = rng.standard_normal((r, 384)).astype(np.float16)
    x = torch.from_numpy(x0.copy()).to(DEV)
    check_rc(lib().dv3k_splitk_reduce(ptr(t32(partials)), r, splits, ptr(t32(bias)), ptr(t32(lam)),
                                      ptr(x), stream()))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(x.cpu().numpy(), splitk_reduce_ref(partials, bias, lam, x0))


@pytest.mark.parametrize("f32_out", [False, True])
@pytest.mark.parametrize("b", [1, 5])
def test_splitk_reduce_layernorm(b, f32_out):
    rng = np.random.default_rng(95 + b + f32_out)
    r, splits = rows_of(b), 8
    partials = rng.standard_normal((splits, r, 384)).astype(np.float32)
    bias = (rng.standard_normal(384) * 0.1).astype(np.float32)
    lam = (rng.random(384) * 0.2 + 0.05).astype(np.float32)
    x0 = (rng.standard_normal((r, 384)) + rng.standard_normal((r, 1))).astype(np.float16)
    g = (rng.standard_normal(384) * 0.3 + 1).astype(np.float32)
    be = (rng.standard_normal(384) * 0.1).astype(np.float32)
    x = torch.from_numpy(x0.copy()).to(DEV)
    h = None if f32_out else torch.empty((r, 384), dtype=torch.float16, device=DEV)
    o = torch.empty((r, 384), dtype=torch.float32, device=DEV) if f32_out else None
    check_rc(lib().dv3k_splitk_reduce_layernorm(ptr(t32(partials)), r, splits, ptr(t32(bias)),
                                                ptr(t32(lam)), ptr(x), ptr(t32(g)), ptr(t32(be)),
                                                ptr(h), ptr(o), stream()))
    torch.cuda.synchronize()
    want_x = splitk_reduce_ref(partials, bias, lam, x0)
    np.testing.assert_array_equal(x.cpu().numpy(), want_x)
    ref_ln = ref_numpy.norm(want_x.astype(np.float64), g, be)
    if f32_out:
        assert np.abs(o.cpu().numpy() - ref_ln).max() < 1e-4
    else:
        assert_close16(h, ref_ln)


# 50 and 64 images leave a partial last wave of at most 74 tiles: those run as two 128-wide
# units each (1008 and 1240 units of work over 148 CTAs).
@pytest.mark.parametrize("b", [1, 3, 50, 64])
def test_matmul_swiglu(b):
    rng = np.random.default_rng(60 + b)
    r = rows_of(b)
    h = f16(rng.standard_normal((r, 384)))
    wg = f16(rng.standard_normal((1536, 384)) / np.sqrt(384) * 2)
    wu = f16(rng.standard_normal((1536, 384)) / np.sqrt(384))
    bg = rng.standard_normal(1536) * 0.1
    bu = rng.standard_normal(1536) * 0.1
    g = h @ wg.T + bg.astype(np.float32)
    u = h @ wu.T + bu.astype(np.float32)
    ref = g / (1 + np.exp(-g)) * u
    concat_w = np.concatenate([wg, wu])
    concat_b = np.concatenate([bg, bu])
    src = np.array([lib().dv3k_gateup_source_row(i) for i in range(3072)])
    act = torch.empty((r, 1536), dtype=torch.float16, device=DEV)
    check_rc(lib().dv3k_matmul_swiglu(ptr(t16(h)), r, ptr(t16(concat_w[src])), ptr(t32(concat_b[src])),
                                      ptr(act), ptr(status()), stream()))
    torch.cuda.synchronize()
    assert_close16(act, ref)


# Folded LayerNorm (no counterpart in the reference): the residual GEMM leaves (rstd, -mean rstd)
# and an f16 aux row (-mean_hi, -mean_lo, -mean_hi, r_hi, r_lo, r_hi, 0...) per row, r = 1/rstd;
# the QKV and gate/up GEMMs read x with W' = f16(W gamma) and a weight aux row (s_hi, s_hi, s_lo,
# c_hi, c_hi, c_lo, 0...) per output column (s = row sums of W', c = b + W beta; weights.cpp),
# which one more K=16 tensor-core step multiplies into -mean s + r c. References: the unrounded
# float64 LayerNorm of x, then the op; the folded kernels are held to the accuracy of the
# unfolded kernels on h = f16(LN(x)).
def ln_stats(x):
    mean = x.mean(axis=1)
    var = ((x - mean[:, None]) ** 2).mean(axis=1)
    rstd = 1.0 / np.sqrt(var + 1e-5)
    return mean, rstd


def split16(v):
    """v as an f16 and the f16 of what it leaves over (hi + lo, 2^-22 of |v|)."""
    hi = np.asarray(v, np.float32).astype(np.float16)
    return hi, (np.asarray(v, np.float64) - hi.astype(np.float64)).astype(np.float16)


def fold(w, b, g, be):
    """The folded weights of weights.cpp from f16 weights w [n][384], bias b, LayerNorm g, be:
    wf = f16(w g) and the weight aux rows [n][16]."""
    g32, be32 = g.astype(np.float32), be.astype(np.float32)
    wf = (w.astype(np.float32) * g32).astype(np.float16)
    s = wf.astype(np.float64).sum(axis=1)
    c = b.astype(np.float32).astype(np.float64) + w @ be32.astype(np.float64)
    aux = np.zeros((len(s), 16), np.float16)
    aux[:, 0], aux[:, 2] = split16(s)
    aux[:, 1] = aux[:, 0]
    aux[:, 3], aux[:, 5] = split16(c)
    aux[:, 4] = aux[:, 3]
    return wf, aux


def ln64(x, g, be):
    mean, rstd = ln_stats(x)
    return (x - mean[:, None]) * rstd[:, None] * g.astype(np.float32) + be.astype(np.float32)


def rowstat_of(x):
    """(rstd, -mean rstd) f32 and the f16 aux rows, as the producers write them."""
    mean, rstd = ln_stats(x)
    rstd32 = rstd.astype(np.float32)
    st = np.stack([rstd32, (-mean * rstd).astype(np.float32)], axis=1)
    aux = np.zeros((len(mean), 16), np.float16)
    aux[:, 0], aux[:, 1] = split16(-mean)
    aux[:, 2] = aux[:, 0]
    aux[:, 3], aux[:, 4] = split16(np.float32(1) / rstd32)
    aux[:, 5] = aux[:, 3]
    return st, aux


def check_stats(st, aux, x):
    """Producer outputs against the float64 statistics of x."""
    mean, rstd = ln_stats(x)
    st, aux = st.cpu().numpy(), aux.cpu().numpy().astype(np.float64)
    assert np.abs(st[:, 0] / rstd - 1).max() < 1e-5
    assert np.abs(st[:, 1] + mean * rstd).max() < 1e-5 * np.abs(mean * rstd).max() + 1e-6
    assert np.abs(aux[:, 0] + aux[:, 1] + mean).max() < 1e-6 * np.abs(mean).max() + 1e-7
    assert np.abs((aux[:, 3] + aux[:, 4]) * rstd - 1).max() < 1e-5
    assert np.array_equal(aux[:, 2], aux[:, 0]) and np.array_equal(aux[:, 5], aux[:, 3])
    assert not aux[:, 6:].any()


def scaled_err(got, ref):
    got = got.float().cpu().numpy().astype(np.float64)
    return np.abs(got - ref) / np.maximum(1.0, np.abs(ref))


def assert_as_accurate(folded, plain, ref):
    """The folded GEMM rounds W gamma to f16 where the unfolded one rounds LN(x) to f16 (h), so
    both carry one f16 rounding of their inputs: against the unrounded float64 reference the
    folded output must be about as accurate as the unfolded kernel on h = f16(LN(x))."""
    ef, ep = scaled_err(folded, ref), scaled_err(plain, ref)
    rms_f, rms_p = np.sqrt((ef ** 2).mean()), np.sqrt((ep ** 2).mean())
    assert ef.max() <= max(4e-3, 2.0 * ep.max()), f"max {ef.max():.3e} vs unfolded {ep.max():.3e}"
    assert rms_f <= 1.5 * rms_p + 1e-6, f"rms {rms_f:.3e} vs unfolded {rms_p:.3e}"


@pytest.mark.parametrize("b", [1, 64])
def test_layernorm_rowstat(b):
    rng = np.random.default_rng(80 + b)
    r = rows_of(b)
    x = f16(rng.standard_normal((r, 384)) * 3 + rng.standard_normal((r, 1)))
    st = torch.empty((r, 2), dtype=torch.float32, device=DEV)
    aux = torch.full((r, 16), 7.0, dtype=torch.float16, device=DEV)
    check_rc(lib().dv3k_layernorm_rowstat(ptr(t16(x)), r, ptr(st), ptr(aux), stream()))
    torch.cuda.synchronize()
    check_stats(st, aux, x)


@pytest.mark.parametrize("k", [384, 1536])
@pytest.mark.parametrize("b", [1, 3, 64])
def test_matmul_resid_rowstat(k, b):
    """x is updated bit for bit as by dv3k_matmul_resid_layernorm; rowstat and the aux rows hold
    the statistics of the stored f16 rows."""
    rng = np.random.default_rng(90 + b + k)
    r = rows_of(b)
    a = f16(rng.standard_normal((r, k)))
    w = f16(rng.standard_normal((384, k)) / np.sqrt(k))
    bias = rng.standard_normal(384) * 0.1
    lam = rng.random(384) * 0.2 + 0.05
    x0 = f16(rng.standard_normal((r, 384)) + rng.standard_normal((r, 1)))
    g = rng.standard_normal(384) * 0.3 + 1
    be = rng.standard_normal(384) * 0.1
    x_ln, x_st = t16(x0), t16(x0)
    h = torch.empty((r, 384), dtype=torch.float16, device=DEV)
    rs = torch.empty((r, 2), dtype=torch.float32, device=DEV)
    aux = torch.full((r, 16), 7.0, dtype=torch.float16, device=DEV)
    st = status()
    ad, wd, bd, ld = t16(a), t16(w), t32(bias), t32(lam)
    check_rc(lib().dv3k_matmul_resid_layernorm(ptr(ad), r, k, ptr(wd), ptr(bd), ptr(ld), ptr(x_ln),
                                               ptr(t32(g)), ptr(t32(be)), ptr(h), None, ptr(st),
                                               stream()))
    check_rc(lib().dv3k_matmul_resid_rowstat(ptr(ad), r, k, ptr(wd), ptr(bd), ptr(ld), ptr(x_st),
                                             ptr(rs), ptr(aux), ptr(st), stream()))
    torch.cuda.synchronize()
    assert st.cpu().tolist() == [0, 0]
    np.testing.assert_array_equal(x_st.cpu().numpy().view(np.uint16), x_ln.cpu().numpy().view(np.uint16))
    check_stats(rs, aux, x_st.float().cpu().numpy().astype(np.float64))


# offset: rows with a large common mean (|mean| about 32 standard deviations), where the folded
# form's x W'^T and mean s nearly cancel in the f32 accumulator; the f16 rounding of x itself is
# the same for both forms.
@pytest.mark.parametrize("b,offset", [(1, 0.0), (3, 0.0), (64, 0.0), (3, 64.0)])
def test_qkv_rope_folded(b, offset):
    rng = np.random.default_rng(100 + b)
    r = rows_of(b)
    x = f16(rng.standard_normal((r, 384)) * 2 + rng.standard_normal((r, 1)) + offset)
    g = rng.standard_normal(384) * 0.3 + 1
    be = rng.standard_normal(384) * 0.1
    w = f16(rng.standard_normal((1152, 384)) / np.sqrt(384))
    bias = rng.standard_normal(1152) * 0.1
    bias[384:768] = 0
    ref = rope_ref(ln64(x, g, be) @ w.T + bias.astype(np.float32), r)
    wf, waux = fold(w, bias, g, be)
    rst, raux = rowstat_of(x)
    cos, sin = ref_numpy.rope_tables()
    out = torch.empty((r, 1152), dtype=torch.float16, device=DEV)
    plain = torch.empty((r, 1152), dtype=torch.float16, device=DEV)
    check_rc(lib().dv3k_qkv_rope_folded(ptr(t16(x)), r, ptr(t16(wf)), ptr(t16(waux)), ptr(t32(rst)),
                                        ptr(t16(raux)), ptr(t32(cos)), ptr(t32(sin)), ptr(out),
                                        ptr(status()), stream()))
    check_rc(lib().dv3k_qkv_rope(ptr(t16(ln64(x, g, be))), r, ptr(t16(w)), ptr(t32(bias)),
                                 ptr(t32(cos)), ptr(t32(sin)), ptr(plain), ptr(status()), stream()))
    torch.cuda.synchronize()
    assert_as_accurate(out, plain, ref)


@pytest.mark.parametrize("b,offset", [(1, 0.0), (3, 0.0), (50, 0.0), (64, 0.0), (3, 64.0)])
def test_matmul_swiglu_folded(b, offset):
    rng = np.random.default_rng(110 + b)
    r = rows_of(b)
    x = f16(rng.standard_normal((r, 384)) * 2 + rng.standard_normal((r, 1)) + offset)
    gam = rng.standard_normal(384) * 0.3 + 1
    be = rng.standard_normal(384) * 0.1
    wg = f16(rng.standard_normal((1536, 384)) / np.sqrt(384) * 2)
    wu = f16(rng.standard_normal((1536, 384)) / np.sqrt(384))
    bg = rng.standard_normal(1536) * 0.1
    bu = rng.standard_normal(1536) * 0.1
    h = ln64(x, gam, be)
    gv = h @ wg.T + bg.astype(np.float32)
    uv = h @ wu.T + bu.astype(np.float32)
    ref = gv / (1 + np.exp(-gv)) * uv
    src = np.array([lib().dv3k_gateup_source_row(i) for i in range(3072)])
    w_packed, b_packed = np.concatenate([wg, wu])[src], np.concatenate([bg, bu])[src]
    wf, waux = fold(w_packed, b_packed, gam, be)
    rst, raux = rowstat_of(x)
    act = torch.empty((r, 1536), dtype=torch.float16, device=DEV)
    plain = torch.empty((r, 1536), dtype=torch.float16, device=DEV)
    check_rc(lib().dv3k_matmul_swiglu_folded(ptr(t16(x)), r, ptr(t16(wf)), ptr(t16(waux)),
                                             ptr(t32(rst)), ptr(t16(raux)), ptr(act), ptr(status()),
                                             stream()))
    check_rc(lib().dv3k_matmul_swiglu(ptr(t16(h)), r, ptr(t16(w_packed)), ptr(t32(b_packed)),
                                      ptr(plain), ptr(status()), stream()))
    torch.cuda.synchronize()
    assert_as_accurate(act, plain, ref)


def test_bounded_wait_expires_and_context_survives():
    """The failure path every kernel uses, made to run out on the device without a fault: a wait
    on an mbarrier that nothing arrives at expires after its limit and records its bit, the
    second role leaves on the abort flag (well before its own, thousand-fold limit) and records
    its bit, the kernel returns, and the context keeps running kernels."""
    import time

    st = status()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    check_rc(lib().dv3k_bounded_wait_selftest(20_000_000, ptr(st), stream()))  # 20 ms
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    assert st.cpu().tolist() == [(1 << 4) | (1 << 5), 0]
    assert 0.015 < elapsed < 2.0  # the second role's own limit would be 20 s
    # the context is intact: a regular kernel still runs and its status stays clean
    rng = np.random.default_rng(3)
    r = rows_of(1)
    qkv = f16(rng.standard_normal((r, 1152)))
    out = torch.empty((r, 384), dtype=torch.float16, device=DEV)
    st2 = status()
    check_rc(lib().dv3k_attention(ptr(t16(qkv)), r, ptr(out), ptr(st2), stream()))
    torch.cuda.synchronize()
    assert st2.cpu().tolist() == [0, 0]
    assert_close16(out, attention_ref(qkv, 1))
