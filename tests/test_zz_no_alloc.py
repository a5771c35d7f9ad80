"""The no-alloc split-K entry point (include/dinov3_kernels.h, dv3k_down_splitk_noalloc).

Some callers cannot allocate device memory (an embedding that owns no allocator, a caller inside
a region where cudaMalloc is forbidden), so this entry point keeps its partial slabs in a
file-scope device array of the library instead of a caller workspace. Checks:
  * two calls in a row (different sizes, no synchronisation between them) give bitwise the same
    x as dv3k_matmul_splitk followed by dv3k_splitk_reduce with a workspace of the caller (same
    kernels, same summation order);
  * a call leaves the device's free memory unchanged (it allocates nothing);
  * a request past the array's 6144 partial rows is refused with a clear message.
Collected last (the file name sorts after every other test file), after every other GPU test;
it also passes when run alone in a fresh process.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

from dinov3_b200 import _lib  # noqa: E402

DEV = "cuda:0"


def _dev(a, dtype):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=dtype)).to(DEV)


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _case(seed, b):
    rng = np.random.default_rng(seed)
    r = 201 * b
    return {
        "r": r,
        "a": _dev(rng.standard_normal((r, 1536)), np.float16),
        "w": _dev(rng.standard_normal((384, 1536)) / np.sqrt(1536), np.float16),
        "bias": _dev(rng.standard_normal(384) * 0.1, np.float32),
        "lam": _dev(rng.random(384) * 0.2 + 0.05, np.float32),
        "x0": rng.standard_normal((r, 384)).astype(np.float16),
    }


def _workspace_result(lib, c, splits, st):
    """x after the two workspace entry points (the existing path)."""
    x = _dev(c["x0"], np.float16)
    parts = torch.empty((splits, c["r"], 384), dtype=torch.float32, device=DEV)
    assert lib.dv3k_matmul_splitk(c["a"].data_ptr(), c["r"], c["w"].data_ptr(), splits,
                                  parts.data_ptr(), st.data_ptr(), _stream()) == 0, _lib.last_error()
    assert lib.dv3k_splitk_reduce(parts.data_ptr(), c["r"], splits, c["bias"].data_ptr(),
                                  c["lam"].data_ptr(), x.data_ptr(), _stream()) == 0, _lib.last_error()
    torch.cuda.synchronize()
    return x.cpu().numpy()


def _noalloc(lib, c, splits, x, st):
    return lib.dv3k_down_splitk_noalloc(c["a"].data_ptr(), c["r"], c["w"].data_ptr(), splits,
                                        c["bias"].data_ptr(), c["lam"].data_ptr(), x.data_ptr(),
                                        st.data_ptr(), _stream())


def test_no_alloc_split_k_matches_workspace_entry_points():
    lib = _lib.load()
    st = torch.zeros(2, dtype=torch.int32, device=DEV)
    cases = [(_case(200, 1), 8), (_case(201, 3), 4)]
    want = [_workspace_result(lib, c, s, st) for c, s in cases]
    xs = [_dev(c["x0"], np.float16) for c, _ in cases]
    # two calls in a row on one stream, no synchronisation between them: the second call's
    # split-K GEMM reuses the shared array only after the first call's reduce has read it
    for (c, s), x in zip(cases, xs):
        assert _noalloc(lib, c, s, x, st) == 0, _lib.last_error()
    torch.cuda.synchronize()
    assert st.cpu().tolist() == [0, 0]
    for (c, _), x, w in zip(cases, xs, want):
        got = x.cpu().numpy()
        np.testing.assert_array_equal(got, w)
        assert not np.array_equal(got, c["x0"])  # the update happened

    # a call allocates nothing: the device's free memory is the same before and after
    c, s = cases[1]
    x = _dev(c["x0"], np.float16)
    torch.cuda.synchronize()
    free_before, _ = torch.cuda.mem_get_info()
    assert _noalloc(lib, c, s, x, st) == 0, _lib.last_error()
    torch.cuda.synchronize()
    free_after, _ = torch.cuda.mem_get_info()
    assert free_after == free_before
    np.testing.assert_array_equal(x.cpu().numpy(), want[1])

    # 8 slices of 1005 rows (5 images) need 8040 partial rows: more than the array holds
    r = 201 * 5
    a = torch.zeros((r, 1536), dtype=torch.float16, device=DEV)
    w = torch.zeros((384, 1536), dtype=torch.float16, device=DEV)
    v = torch.zeros(384, dtype=torch.float32, device=DEV)
    x = torch.zeros((r, 384), dtype=torch.float16, device=DEV)
    rc = lib.dv3k_down_splitk_noalloc(a.data_ptr(), r, w.data_ptr(), 8, v.data_ptr(), v.data_ptr(),
                                      x.data_ptr(), st.data_ptr(), _stream())
    assert rc != 0 and "6144" in _lib.last_error()
