"""Projection GEMMs over weights kept packed as Q4_0 / Q8_0 (packed.cuh):
each K step's blocks are fetched by a bulk copy and decoded into the f16
tile in shared memory by converter warps (the reference decodes per use as
well: crates/omg-wgpu/src/shaders/weight.wgsl:29-54). The decode is
f16(QTensor::get) exactly, and the MMA then sees the same tiles as the f16
path, so every output must equal the f16-weight kernels' on the
dequantized weights bit for bit, and those are checked against an f64
reference in test_gpu_gemm.py. Shapes include partial row and column tiles,
K with a half K step (k % 64 == 32), split-K and both tile widths."""
import numpy as np
import pytest

from grande_b200 import _lib as L
from oracle import oracle as O

from test_gpu_gemm import interleave_gate_up, run_gemm, run_mlp

pytestmark = pytest.mark.gpu


def quantized(dtype, w32):
    data, scales = O.quantize(dtype, w32.ravel())
    f16 = O.dequantize(dtype, data, scales, w32.size).reshape(w32.shape).astype(np.float16)
    codes = np.frombuffer(data, np.uint8).copy()
    sc = np.frombuffer(scales, np.uint8).copy()
    return codes, sc, f16


def run_gemm_q(device, x16, dtype, codes, sc, w_rows, n_out, epi, bn=0, splits=1):
    m, k = x16.shape
    f32 = epi == 0
    ldo = (n_out + 7) // 8 * 8
    out = np.zeros((m, ldo), dtype=np.float32 if f32 else np.float16)
    L.check(L.lib().omg_debug_gemm_q(
        device, L.ptr(x16.view(np.uint16), L.C.c_uint16), m, k, k, dtype,
        L.ptr(codes, L.C.c_uint8), L.ptr(sc, L.C.c_uint8), w_rows, n_out, epi, bn, splits,
        out.ctypes.data_as(L.C.c_void_p), ldo))
    return out[:, :n_out].astype(np.float32)


@pytest.mark.parametrize("dtype", [O.Q4, O.Q8])
@pytest.mark.parametrize("m,n,k,bn,splits", [
    (23, 96, 64, 128, 1), (130, 200, 96, 256, 1), (300, 520, 2080, 256, 2), (1, 128, 32, 128, 1),
    (788, 2048, 2048, 256, 2), (788, 3072, 2048, 256, 1), (150, 640, 2048, 256, 1),
    (300, 520, 2080, 512, 2), (788, 2048, 2048, 512, 2), (130, 200, 96, 512, 1),
])
def test_packed_gemm_equals_f16_gemm(device, dtype, m, n, k, bn, splits):
    rng = np.random.default_rng(m + n + k + dtype)
    x16 = (rng.uniform(-1, 1, (m, k)) * 2).astype(np.float16)
    w32 = (rng.standard_normal((n, k)) * 0.05).astype(np.float32)
    codes, sc, w16 = quantized(dtype, w32)
    exp = run_gemm(device, x16, w16, n, 0, bn=min(bn, 256), splits=splits)
    got = run_gemm_q(device, x16, dtype, codes, sc, n, n, 0, bn=bn, splits=splits)
    assert np.array_equal(got, exp)
    # f16 epilogue too
    exp16 = run_gemm(device, x16, w16, n, 3, bn=min(bn, 256))
    got16 = run_gemm_q(device, x16, dtype, codes, sc, n, n, 3, bn=bn)
    assert np.array_equal(got16, exp16)


@pytest.mark.parametrize("dtype", [O.Q4, O.Q8])
@pytest.mark.parametrize("m,n,k", [(70, 100, 160), (300, 384, 256)])
def test_packed_gated_equals_f16_gated(device, dtype, m, n, k):
    rng = np.random.default_rng(m * n + dtype)
    x16 = rng.uniform(-1, 1, (m, k)).astype(np.float16)
    w32 = interleave_gate_up((rng.standard_normal((n, k)) * 0.1).astype(np.float32),
                             (rng.standard_normal((n, k)) * 0.1).astype(np.float32))
    codes, sc, w16 = quantized(dtype, w32)
    exp = run_gemm(device, x16, w16, n, 1)
    got = run_gemm_q(device, x16, dtype, codes, sc, w16.shape[0], n, 1)
    assert np.array_equal(got, exp)


@pytest.mark.parametrize("dtype", [O.Q4, O.Q8])
@pytest.mark.parametrize("pair", [0, 1])
@pytest.mark.parametrize("m,d,ff", [(700, 256, 1024), (788, 2048, 8192), (130, 256, 512)])
def test_packed_fused_mlp_equals_f16(device, dtype, m, d, ff, pair):
    """The fused FFN launch (gate+up, GeGLU, split-K down units gated on the
    activation bands) on packed weights, one-CTA tiles and CTA pairs: the
    f16 launch's bits."""
    rng = np.random.default_rng(m + d + dtype)
    x16 = rng.uniform(-1, 1, (m, d)).astype(np.float16)
    w_up32 = interleave_gate_up((rng.standard_normal((ff, d)) * 0.05).astype(np.float32),
                                (rng.standard_normal((ff, d)) * 0.05).astype(np.float32))
    wd32 = (rng.standard_normal((d, ff)) * 0.05).astype(np.float32)
    uc, us, w_up16 = quantized(dtype, w_up32)
    dc, ds, wd16 = quantized(dtype, wd32)
    a1, y1 = run_mlp(device, x16, w_up16, wd16, ff, 0)
    act = np.zeros((m, ff), np.float16)
    y = np.zeros((m, d), np.float32)
    L.check(L.lib().omg_debug_mlp_q(
        device, L.ptr(x16.view(np.uint16), L.C.c_uint16), m, d, dtype, L.ptr(uc, L.C.c_uint8),
        L.ptr(us, L.C.c_uint8), ff, L.ptr(dc, L.C.c_uint8), L.ptr(ds, L.C.c_uint8), pair,
        L.ptr(act.view(np.uint16), L.C.c_uint16), L.ptr(y, L.C.c_float)))
    assert np.array_equal(act, a1)
    assert np.array_equal(y, y1)


@pytest.mark.parametrize("config", ["e2b-q4", "gemma3-270m-q8"])
def test_packed_engine_equals_f16_engine(device, config):
    """Whole passes (QKV with the fused qk_prep, o, the fused FFN, logits) of
    an engine keeping its Q4_0 / Q8_0 linears packed and of one decoding them
    once into f16 rows: the same bits."""
    import dataclasses

    from grande_b200 import synth
    from grande_b200.engine import Want
    shape = dataclasses.replace(synth.CONFIGS[config], layers=2)
    req = synth.request(shape, seed=9)
    tensors = synth.generate(shape, seed=0)
    rows = {}
    for packed in (True, False):
        eng = synth.build_engine(shape, shape.tokens() + 64, shape.branches, device=device,
                                 tensors=tensors, packed=packed)
        hid = eng.evaluate(req.prefix, req.branches, Want.HIDDEN)
        eng.evict_resident()
        lg = eng.evaluate(req.prefix, req.branches, Want.LOGITS)
        rows[packed] = [o.rows for o in hid] + [o.rows for o in lg]
        eng.close()
    for a, b in zip(rows[True], rows[False]):
        assert np.array_equal(a, b)
