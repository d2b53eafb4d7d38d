"""The allocation-free GEMM entry point (omg_gemm_splitk_noalloc).

It serves callers that hand this library device buffers but cannot let it
allocate (their own memory pool, or code where a cudaMalloc would synchronise
the device); its split-K partials live in a static device array instead.
The test gives it device buffers (allocated here, by the test, with torch),
calls it twice in a row through the C ABI with different inputs, and checks
each result against an f64 product of the same f16 operands and against the
allocating entry point (omg_debug_gemm), at the GEMM tests' tolerance. This file is collected last so that a failure here cannot
stop the other GPU tests under `-x`.
"""
import ctypes as C

import numpy as np
import pytest

from grande_b200 import _lib as L

pytestmark = pytest.mark.gpu

TOL = 2e-3


def reference_gemm(device, x16, w16, splits):
    m, k = x16.shape
    n = w16.shape[0]
    out = np.zeros((m, n), np.float32)
    L.check(L.lib().omg_debug_gemm(device, L.ptr(x16.view(np.uint16), C.c_uint16), m, k, k,
                                   L.ptr(w16.view(np.uint16), C.c_uint16), n, n, 0, 128, splits,
                                   out.ctypes.data_as(C.c_void_p), n))
    return out


def test_noalloc_gemm_matches_allocating_entry_point(device):
    torch = pytest.importorskip("torch")
    dev = torch.device(f"cuda:{device}")
    m, k, n, splits = 300, 2048, 520, 2
    rng = np.random.default_rng(11)
    out_d = torch.zeros((m, n), dtype=torch.float32, device=dev)
    for call in range(2):
        x16 = rng.standard_normal((m, k)).astype(np.float16)
        w16 = (rng.standard_normal((n, k)) * 0.05).astype(np.float16)
        x_d = torch.from_numpy(x16).to(dev)
        w_d = torch.from_numpy(w16).to(dev)
        torch.cuda.synchronize(dev)
        L.check(L.lib().omg_gemm_splitk_noalloc(device, C.c_void_p(x_d.data_ptr()), m, k, k,
                                                C.c_void_p(w_d.data_ptr()), n, splits,
                                                C.c_void_p(out_d.data_ptr()), n, None))
        got = out_d.cpu().numpy()
        f64 = x16.astype(np.float64) @ w16.astype(np.float64).T
        err64 = float(np.max(np.abs(got - f64) / np.maximum(np.abs(f64), 1.0)))
        assert err64 < TOL, (call, err64)
        exp = reference_gemm(device, x16, w16, splits)
        err = float(np.max(np.abs(got - exp) / np.maximum(np.abs(exp), 1.0)))
        assert err < TOL, (call, err)


def test_noalloc_rejects_oversized_problems(device):
    # 4 slabs of 4096 x 1024 f32 = 64 MiB > the 32 MiB static scratch; the
    # size check runs before any device pointer is touched.
    bogus = C.c_void_p(16)
    rc = L.lib().omg_gemm_splitk_noalloc(device, bogus, 4096, 4096, 4096, bogus, 1024, 4, bogus,
                                         1024, None)
    assert rc == -1
    assert "static scratch holds" in L.lib().omg_last_error().decode()


def test_noalloc_rejects_short_row_stride(device):
    # An lda below k would make the operand rows overlap; it is refused before
    # any device pointer is touched.
    bogus = C.c_void_p(16)
    rc = L.lib().omg_gemm_splitk_noalloc(device, bogus, 64, 256, 128, bogus, 64, 1, bogus, 64,
                                         None)
    assert rc == -1
    assert "lda 128 < k 256" in L.lib().omg_last_error().decode()
