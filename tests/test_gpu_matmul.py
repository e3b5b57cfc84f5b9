"""bst_matmul (Tensor.matMul -> gemm::matmul on device buffers) against the oracle's gemm.rs
restatement: the reference's own NativeTestSuite and gemm.rs cases, then shapes that exercise the
GEMV (m <= 8) and tcgen05 (m > 8) paths, including K tails and N below one tile."""
import ctypes
import json

import numpy as np
import pytest

from basalt_b200 import _lib
from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def gpu_matmul(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    import torch

    m, k = a.shape
    n = b.shape[1]
    ta = torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()
    tb = torch.from_numpy(np.ascontiguousarray(b, np.float32)).cuda()
    tc = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    code = _lib.load().bst_matmul(torch.cuda.current_device(), None, ta.data_ptr(), tb.data_ptr(),
                                  tc.data_ptr(), m, k, n)
    assert code == 0, _lib.last_error()
    return tc.cpu().numpy()


@pytest.fixture(scope="module")
def known(golden_dir):
    return json.loads((golden_dir / "reference_known_answers.json").read_text())


def test_native_test_suite_shapes(runtime, known):
    spec = known["native_matmul"]
    r = orc.JavaRandom(spec["seed"])
    for m, k, n in spec["shapes"]:
        left = np.array([r.next_float() * np.float32(2) - np.float32(1) for _ in range(m * k)],
                        np.float32).reshape(m, k)
        right = np.array([r.next_float() * np.float32(2) - np.float32(1) for _ in range(k * n)],
                         np.float32).reshape(k, n)
        got = gpu_matmul(left, right)
        assert np.all(np.isfinite(got))
        np.testing.assert_allclose(got, orc.matmul(left, right), rtol=0, atol=spec["tolerance"],
                                   err_msg=f"{m}x{k}x{n}")


def test_gemm_unit_cases(runtime, known):
    g = known["gemm_unit"]
    for m, k, n in g["cases"] + g["pooled_cases"]:
        a = ((np.arange(m * k) * 7 % 13) - 6).astype(np.float32).reshape(m, k)
        b = ((np.arange(k * n) * 5 % 11) - 5).astype(np.float32).reshape(k, n)
        exact = a.astype(np.float64) @ b.astype(np.float64)
        np.testing.assert_allclose(gpu_matmul(a, b), exact, rtol=0, atol=g["pooled_tolerance"],
                                   err_msg=f"{m}x{k}x{n}")


@pytest.mark.parametrize("m,k,n", [(1, 768, 2304), (5, 300, 77), (8, 512, 512), (9, 64, 16),
                                   (33, 36, 9), (100, 512, 1536), (256, 2048, 512),
                                   (300, 120, 200), (1024, 768, 3072),
                                   # more tiles than SMs: CTAs loop over units and alternate
                                   # accumulators; tails in M, N and K
                                   (3000, 200, 1000), (4096, 512, 1536)])
def test_random_shapes_match_fp32(runtime, m, k, n):
    rng = np.random.default_rng(m * 1000 + n)
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = (rng.standard_normal((k, n)) * 0.05).astype(np.float32)
    want = orc.matmul(a, b)
    got = gpu_matmul(a, b)
    # 3xTF32 products agree with fp32 to ~2^-21 relative and sums differ only in order, so the
    # error stays near fp32 rounding (single-pass tf32 would be ~5e-4 of the scale).
    scale = np.abs(a).astype(np.float64) @ np.abs(b).astype(np.float64)
    assert np.max(np.abs(got - want) / (scale + 1e-30)) < 1e-5, (m, k, n)


def test_empty_and_invalid_arguments(runtime):
    import torch

    lib = _lib.load()
    dev = torch.cuda.current_device()
    c = torch.zeros((3, 4), device="cuda")
    a = torch.ones((3, 0), device="cuda")
    b = torch.ones((0, 4), device="cuda")
    c.fill_(7.0)
    assert lib.bst_matmul(dev, None, a.data_ptr() or 1, b.data_ptr() or 1, c.data_ptr(), 3, 0, 4) == 0
    assert float(c.abs().max()) == 0.0  # k = 0: C is overwritten with zeros
    assert lib.bst_matmul(dev, None, None, None, c.data_ptr(), 3, 2, 4) == _lib.BST_INVALID
    assert lib.bst_matmul(dev, None, c.data_ptr(), c.data_ptr(), c.data_ptr(), -1, 2, 4) == _lib.BST_SHAPE
