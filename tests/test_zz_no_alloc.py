"""bst_matmul_static — the matmul entry point that allocates nothing.

It exists for callers that may not call cudaMalloc while they run (a host runtime that owns the
device memory pool, a fixed device-memory budget, a latency-critical thread that must not trigger
the allocator's device-wide synchronisation). Its temporaries live in a fixed scratch array inside
the library, so it only accepts problems whose operand planes fit there.

The test calls it through the C ABI twice in a row on the same inputs (the scratch keeps the first
call's contents when the second one starts) and compares each result with bst_matmul's, within the
same tolerance the matmul tests use, and with the float64 product. It also checks that the calls
take nothing from the device's stream-ordered memory pool and that the second call changes the
device's free memory by nothing. This file is collected last, so a stop-at-first-failure run has
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


def _pool_usage(device):
    """(reserved, used) bytes of the device's default stream-ordered memory pool."""
    from cuda.bindings import runtime as rt

    err, pool = rt.cudaDeviceGetDefaultMemPool(device)
    assert err == rt.cudaError_t.cudaSuccess
    out = []
    for attr in (rt.cudaMemPoolAttr.cudaMemPoolAttrReservedMemCurrent,
                 rt.cudaMemPoolAttr.cudaMemPoolAttrUsedMemCurrent):
        err, value = rt.cudaMemPoolGetAttribute(pool, attr)
        assert err == rt.cudaError_t.cudaSuccess
        out.append(int(value))
    return tuple(out)


def _free_bytes():
    from cuda.bindings import runtime as rt

    err, free, _total = rt.cudaMemGetInfo()
    assert err == rt.cudaError_t.cudaSuccess
    return int(free)


# (512, 1024, 1024) fits the scratch only with fewer K splits than bst_matmul plans for it.
@pytest.mark.parametrize("m,k,n", [(256, 512, 512), (5, 300, 77), (100, 96, 40),
                                   (512, 1024, 1024)])
def test_static_matmul_matches_matmul_on_two_calls_in_a_row(runtime, m, k, n):
    import torch

    rng = np.random.default_rng(7 * m + n)
    a_host = rng.standard_normal((m, k)).astype(np.float32)
    b_host = (rng.standard_normal((k, n)) * 0.05).astype(np.float32)
    a = torch.from_numpy(a_host).cuda()
    b = torch.from_numpy(b_host).cuda()
    want = torch.empty((m, n), dtype=torch.float32, device="cuda")
    assert _call("bst_matmul", a, b, want, m, k, n) == 0, _lib.last_error()
    exact = a_host.astype(np.float64) @ b_host.astype(np.float64)
    scale = np.abs(a_host).astype(np.float64) @ np.abs(b_host).astype(np.float64)
    expected = want.cpu().numpy()
    device = torch.cuda.current_device()
    pool_before = _pool_usage(device)
    for call in range(2):
        got = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
        torch.cuda.synchronize()
        free_before = _free_bytes()
        assert _call("bst_matmul_static", a, b, got, m, k, n) == 0, _lib.last_error()
        if call == 1:
            # The first call may load the library's module (its code and the scratch array);
            # a second call allocates nothing at all.
            assert _free_bytes() == free_before
        result = got.cpu().numpy()
        assert np.all(np.isfinite(result))
        assert (np.abs(result - expected) / (scale + 1e-30)).max() < 1e-5
        assert (np.abs(result - exact) / (scale + 1e-30)).max() < 1e-5
    assert _pool_usage(device) == pool_before


def test_static_matmul_rejects_problems_larger_than_its_scratch(runtime):
    import torch

    m, k, n = 4096, 1024, 1024  # operand planes alone need 40 MiB; the static array holds 16 MiB
    a = torch.zeros((m, k), device="cuda")
    b = torch.zeros((k, n), device="cuda")
    c = torch.zeros((m, n), device="cuda")
    assert _call("bst_matmul_static", a, b, c, m, k, n) == _lib.BST_SHAPE
    assert "static scratch" in _lib.last_error()
