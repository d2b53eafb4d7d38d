"""The tcgen05 GEMM against an fp32 reference of the same op, rounded the way
the reference's matmul kernels round (X and W to f16, f32 accumulate:
crates/omg-wgpu/shaders/matmul.wgsl:1-9, tests/matmul.rs:187-192,221).

Shapes are the reference's odd ones (partial row / column tiles,
tests/matmul.rs:273-290) plus the BASELINE configs' projection shapes.
Tolerance 2e-3 relative to max(|expected|, 1), as tests/matmul.rs:232.
"""
import numpy as np
import pytest

from grande_b200 import _lib as L

pytestmark = pytest.mark.gpu

TOL = 2e-3


def gelu_tanh(x):
    z = np.clip(0.7978845608028654 * (x + 0.044715 * x ** 3), -15, 15)
    return 0.5 * x * (1.0 + np.tanh(z))


def run_gemm(device, x16, w16, n_out, epi, bn=0, splits=1):
    m, k = x16.shape
    f32 = epi == 0
    ldo = n_out if f32 else n_out
    ldo = (ldo + 7) // 8 * 8
    out = np.zeros((m, ldo), dtype=np.float32 if f32 else np.float16)
    L.check(L.lib().omg_debug_gemm(
        device, L.ptr(x16.view(np.uint16), L.C.c_uint16), m, k, k,
        L.ptr(np.ascontiguousarray(w16).view(np.uint16), L.C.c_uint16), w16.shape[0], n_out,
        epi, bn, splits, out.ctypes.data_as(L.C.c_void_p), ldo))
    return out[:, :n_out].astype(np.float32)


def interleave_gate_up(wg, wu):
    n, k = wg.shape
    npad = (n + 127) // 128 * 128
    out = np.zeros((2 * npad, k), dtype=wg.dtype)
    for b in range(npad // 128):
        g = wg[128 * b:128 * b + 128]
        u = wu[128 * b:128 * b + 128]
        out[256 * b:256 * b + len(g)] = g
        out[256 * b + 128:256 * b + 128 + len(u)] = u
    return out


def rel_err(got, exp):
    return float(np.max(np.abs(got - exp) / np.maximum(np.abs(exp), 1.0)))


@pytest.mark.parametrize("m,n,k", [(23, 96, 64), (130, 200, 96), (64, 128, 32), (300, 520, 256)])
@pytest.mark.parametrize("bn", [128, 256])
def test_matmul_odd_shapes(device, m, n, k, bn):
    rng = np.random.default_rng(m * n * k + bn)
    x16 = (rng.uniform(-1, 1, (m, k)) * 4).astype(np.float16)
    w16 = rng.uniform(-1, 1, (n, k)).astype(np.float16)
    exp = x16.astype(np.float64) @ w16.astype(np.float64).T
    got = run_gemm(device, x16, w16, n, 0, bn=bn, splits=1)
    assert rel_err(got, exp) < TOL


@pytest.mark.parametrize("m,n,k", [(23, 96, 64), (70, 100, 160), (200, 300, 128)])
def test_gated_odd_shapes(device, m, n, k):
    rng = np.random.default_rng(m + n + k)
    x16 = rng.uniform(-1, 1, (m, k)).astype(np.float16)
    wg = rng.uniform(-1, 1, (n, k)).astype(np.float16)
    wu = rng.uniform(-1, 1, (n, k)).astype(np.float16)
    w = interleave_gate_up(wg, wu)
    xd = x16.astype(np.float64)
    gate = xd @ wg.astype(np.float64).T
    up = xd @ wu.astype(np.float64).T
    exp = gelu_tanh(gate) * up
    got = run_gemm(device, x16, w, n, 1)
    # the f16 output rounding adds up to 2^-11 relative
    assert rel_err(got, exp) < TOL + 1e-3


@pytest.mark.parametrize("m,n,k,splits", [
    (788, 3072, 2048, 1),   # E2B qkv
    (788, 2048, 2048, 2),   # E2B o, split-K
    (788, 2048, 8192, 2),   # E2B down, split-K
    (150, 1536, 640, 1),    # 270M qkv
])
def test_matmul_config_shapes(device, m, n, k, splits):
    rng = np.random.default_rng(n + k)
    x16 = rng.standard_normal((m, k)).astype(np.float16)
    w16 = (rng.standard_normal((n, k)) * 0.02).astype(np.float16)
    exp = x16.astype(np.float32) @ w16.astype(np.float32).T
    got = run_gemm(device, x16, w16, n, 0, bn=128, splits=splits)
    assert rel_err(got, exp) < TOL


def test_gated_config_shape(device):
    m, n, k = 788, 8192, 2048
    rng = np.random.default_rng(7)
    x16 = rng.standard_normal((m, k)).astype(np.float16)
    wg = (rng.standard_normal((n, k)) * 0.02).astype(np.float16)
    wu = (rng.standard_normal((n, k)) * 0.02).astype(np.float16)
    w = interleave_gate_up(wg, wu)
    xf = x16.astype(np.float32)
    exp = gelu_tanh(xf @ wg.astype(np.float32).T) * (xf @ wu.astype(np.float32).T)
    got = run_gemm(device, x16, w, n, 1)
    assert rel_err(got, exp) < TOL + 1e-3


def gelu_erf(x):
    from scipy.special import erf
    return 0.5 * x * (1.0 + erf(x / np.sqrt(2.0)))


@pytest.mark.parametrize("bn", [128, 256])
def test_matmul_n_fastest_order(device, bn):
    """Rows outnumber weight rows more than four to one: the tiles are
    walked N-fastest (the encoder's shapes); same result."""
    m, n, k = 4100, 300, 192
    rng = np.random.default_rng(bn)
    x16 = rng.uniform(-1, 1, (m, k)).astype(np.float16)
    w16 = rng.uniform(-1, 1, (n, k)).astype(np.float16)
    exp = x16.astype(np.float64) @ w16.astype(np.float64).T
    got = run_gemm(device, x16, w16, n, 0, bn=bn, splits=1)
    assert rel_err(got, exp) < TOL


def test_gated_erf_encoder_rows(device):
    """The erf GeGLU epilogue (matmul_gated.wgsl:114-134, GELU_ERF = 1) on
    an encoder-like shape, against the exact erf GELU."""
    m, n, k = 2100, 200, 128
    rng = np.random.default_rng(5)
    x16 = rng.uniform(-1, 1, (m, k)).astype(np.float16)
    wg = (rng.uniform(-1, 1, (n, k)) * 0.3).astype(np.float16)
    wu = (rng.uniform(-1, 1, (n, k)) * 0.3).astype(np.float16)
    w = interleave_gate_up(wg, wu)
    xd = x16.astype(np.float64)
    exp = gelu_erf(xd @ wg.astype(np.float64).T) * (xd @ wu.astype(np.float64).T)
    got = run_gemm(device, x16, w, n, 2)
    assert rel_err(got, exp) < TOL + 1e-3


PAIR_SHAPES = [
    (788, 3072, 2048, 0, 1),    # E2B qkv, 7 row tiles: the last pair has one empty half
    (788, 2048, 8192, 0, 2),    # E2B down, split-K
    (300, 520, 256, 0, 1),      # partial row and column tiles
    (23, 96, 64, 0, 1),         # one partial tile
    (1000, 700, 192, 3, 1),     # f16 out
    (4100, 300, 192, 0, 1),     # N-fastest order
]


@pytest.mark.parametrize("m,n,k,epi,splits", PAIR_SHAPES)
def test_pair_kernel_matches_one_cta_kernel(device, m, n, k, epi, splits):
    """The CTA-pair (cta_group::2) kernel against the one-CTA kernel on the
    same operands: same products in the same K order, so the same bits."""
    rng = np.random.default_rng(m + 3 * n + k)
    x16 = rng.uniform(-1, 1, (m, k)).astype(np.float16)
    w16 = rng.uniform(-1, 1, (n, k)).astype(np.float16)
    one = run_gemm(device, x16, w16, n, epi, bn=256, splits=splits)
    pair = run_gemm(device, x16, w16, n, epi, bn=512, splits=splits)
    assert np.array_equal(one, pair)
    exp = x16.astype(np.float64) @ w16.astype(np.float64).T
    assert rel_err(pair, exp) < TOL + (1e-3 if epi == 3 else 0.0)


@pytest.mark.parametrize("epi", [1, 2])
def test_pair_kernel_gated(device, epi):
    m, n, k = 788, 600, 256
    rng = np.random.default_rng(epi)
    x16 = rng.uniform(-1, 1, (m, k)).astype(np.float16)
    wg = (rng.uniform(-1, 1, (n, k)) * 0.3).astype(np.float16)
    wu = (rng.uniform(-1, 1, (n, k)) * 0.3).astype(np.float16)
    w = interleave_gate_up(wg, wu)
    one = run_gemm(device, x16, w, n, epi, bn=256)
    pair = run_gemm(device, x16, w, n, epi, bn=512)
    assert np.array_equal(one, pair)
    xd = x16.astype(np.float64)
    act = gelu_tanh if epi == 1 else gelu_erf
    exp = act(xd @ wg.astype(np.float64).T) * (xd @ wu.astype(np.float64).T)
    assert rel_err(pair, exp) < TOL + 1e-3


def run_mlp(device, x16, w_up, w_dn, ff, pair):
    m, d = x16.shape
    act = np.zeros((m, ff), np.float16)
    y = np.zeros((m, d), np.float32)
    L.check(L.lib().omg_debug_mlp(
        device, L.ptr(x16.view(np.uint16), L.C.c_uint16), m, d,
        L.ptr(np.ascontiguousarray(w_up).view(np.uint16), L.C.c_uint16), ff,
        L.ptr(np.ascontiguousarray(w_dn).view(np.uint16), L.C.c_uint16), pair,
        L.ptr(act.view(np.uint16), L.C.c_uint16), L.ptr(y, L.C.c_float)))
    return act, y


@pytest.mark.parametrize("m", [2100, 700])
def test_fused_mlp_pair_matches_one_cta(device, m):
    """The fused FFN launch (gate+up with the GeGLU epilogue, then the split-K
    down units gated on the activation bands) on CTA pairs and on one-CTA
    tiles: the same bits; and both against an f64 reference of the two
    projections (the activation rounded to f16 as the kernel stores it)."""
    d, ff = 256, 1024
    rng = np.random.default_rng(m)
    x16 = rng.uniform(-1, 1, (m, d)).astype(np.float16)
    wg = (rng.uniform(-1, 1, (ff, d)) * 0.2).astype(np.float16)
    wu = (rng.uniform(-1, 1, (ff, d)) * 0.2).astype(np.float16)
    wd = (rng.uniform(-1, 1, (d, ff)) * 0.2).astype(np.float16)
    w_up = interleave_gate_up(wg, wu)
    a1, y1 = run_mlp(device, x16, w_up, wd, ff, 0)
    a2, y2 = run_mlp(device, x16, w_up, wd, ff, 1)
    assert np.array_equal(a1, a2)
    assert np.array_equal(y1, y2)
    xd = x16.astype(np.float64)
    act = gelu_tanh(xd @ wg.astype(np.float64).T) * (xd @ wu.astype(np.float64).T)
    assert rel_err(a2.astype(np.float32), act) < TOL + 1e-3
    exp = a2.astype(np.float64) @ wd.astype(np.float64).T
    assert rel_err(y2, exp) < TOL
