"""The no-alloc split-K entry point (include/dinov3_kernels.h, dv3k_down_splitk_noalloc): its
partial slabs live in a file-scope device array of the library instead of a caller workspace.
Two calls of different sizes give bitwise the same x as dv3k_matmul_splitk followed by
dv3k_splitk_reduce with a workspace of the caller (same kernels, same summation order), and a
size past the array's 6144 partial rows is refused. Collected last, after every other GPU test.
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


def test_no_alloc_split_k_matches_workspace_entry_points():
    lib = _lib.load()
    st = torch.zeros(2, dtype=torch.int32, device=DEV)
    for call, (b, splits) in enumerate([(1, 8), (3, 4)]):
        rng = np.random.default_rng(200 + call)
        r = 201 * b
        a = _dev(rng.standard_normal((r, 1536)), np.float16)
        w = _dev(rng.standard_normal((384, 1536)) / np.sqrt(1536), np.float16)
        bias = _dev(rng.standard_normal(384) * 0.1, np.float32)
        lam = _dev(rng.random(384) * 0.2 + 0.05, np.float32)
        x0 = rng.standard_normal((r, 384)).astype(np.float16)
        x_ref = _dev(x0, np.float16)
        x_new = _dev(x0, np.float16)
        parts = torch.empty((splits, r, 384), dtype=torch.float32, device=DEV)
        assert lib.dv3k_matmul_splitk(a.data_ptr(), r, w.data_ptr(), splits, parts.data_ptr(),
                                      st.data_ptr(), _stream()) == 0, _lib.last_error()
        assert lib.dv3k_splitk_reduce(parts.data_ptr(), r, splits, bias.data_ptr(), lam.data_ptr(),
                                      x_ref.data_ptr(), _stream()) == 0, _lib.last_error()
        assert lib.dv3k_down_splitk_noalloc(a.data_ptr(), r, w.data_ptr(), splits, bias.data_ptr(),
                                            lam.data_ptr(), x_new.data_ptr(), st.data_ptr(),
                                            _stream()) == 0, _lib.last_error()
        torch.cuda.synchronize()
        assert st.cpu().tolist() == [0, 0]
        np.testing.assert_array_equal(x_new.cpu().numpy(), x_ref.cpu().numpy())
        assert not np.array_equal(x_new.cpu().numpy(), x0)  # the update happened
    # 8 slices of 1005 rows (5 images) need 8040 partial rows: more than the array holds
    r = 201 * 5
    a = torch.zeros((r, 1536), dtype=torch.float16, device=DEV)
    w = torch.zeros((384, 1536), dtype=torch.float16, device=DEV)
    v = torch.zeros(384, dtype=torch.float32, device=DEV)
    x = torch.zeros((r, 384), dtype=torch.float16, device=DEV)
    rc = lib.dv3k_down_splitk_noalloc(a.data_ptr(), r, w.data_ptr(), 8, v.data_ptr(), v.data_ptr(),
                                      x.data_ptr(), st.data_ptr(), _stream())
    assert rc != 0 and "6144" in _lib.last_error()
