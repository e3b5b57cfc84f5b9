"""bst_matmul_static — the matmul entry point that allocates nothing.

It exists for callers that may not call cudaMalloc while they run (a host runtime that owns the
device memory pool, a fixed device-memory budget, a latency-critical thread that must not trigger
the allocator's device-wide synchronisation). Its temporaries live in a fixed scratch array inside
the library, so it only accepts problems whose scratch fits there.

The test calls it through the C ABI twice in a row on the same inputs (the scratch keeps the first
call's contents when the second one starts) and compares each result with bst_matmul's, within the
same tolerance the matmul tests use. This file is collected last, so a stop-at-first-failure run has
already run every other test; it also passes on its own in a fresh process.
"""
import numpy as np
import pytest

from basalt_b200 import _lib

pytestmark = pytest.mark.gpu


def _call(fn_name, ta, tb, tc, m, k, n):
    import torch

    lib = _lib.load()
    code = getattr(lib, fn_name)(torch.cuda.current_device(), None, ta.data_ptr(), tb.data_ptr(),
                                 tc.data_ptr(), m, k, n)
    torch.cuda.synchronize()
    return code


@pytest.mark.parametrize("m,k,n", [(256, 512, 512), (5, 300, 77), (100, 96, 40)])
def test_static_matmul_matches_matmul_on_two_calls_in_a_row(runtime, m, k, n):
    import torch

    rng = np.random.default_rng(7 * m + n)
    a = torch.from_numpy(rng.standard_normal((m, k)).astype(np.float32)).cuda()
    b = torch.from_numpy((rng.standard_normal((k, n)) * 0.05).astype(np.float32)).cuda()
    want = torch.empty((m, n), dtype=torch.float32, device="cuda")
    assert _call("bst_matmul", a, b, want, m, k, n) == 0, _lib.last_error()
    scale = (a.abs().double() @ b.abs().double()).cpu().numpy()
    expected = want.cpu().numpy()
    for _ in range(2):
        got = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
        assert _call("bst_matmul_static", a, b, got, m, k, n) == 0, _lib.last_error()
        diff = np.abs(got.cpu().numpy() - expected) / (scale + 1e-30)
        assert np.all(np.isfinite(got.cpu().numpy()))
        assert diff.max() < 1e-5


def test_static_matmul_rejects_problems_larger_than_its_scratch(runtime):
    import torch

    m, k, n = 4096, 1024, 1024  # needs 40 MiB of scratch; the static array holds 16 MiB
    a = torch.zeros((m, k), device="cuda")
    b = torch.zeros((k, n), device="cuda")
    c = torch.zeros((m, n), device="cuda")
    assert _call("bst_matmul_static", a, b, c, m, k, n) == _lib.BST_SHAPE
    assert "static scratch" in _lib.last_error()
