"""Q4_0 / Q8_0 unpacking and dequantization on the device, bit for bit
against QTensor::get (crates/omg-wgpu/src/model.rs:508-525, restated in
oracle/): the load-time decoder the engine runs on every pushed linear, the
f16 weights of whole layers read back from engines at the BASELINE shapes
(an E2B Q4_0 layer, a 270M Q8_0 layer), and the lm_head's in-shared-memory
decoder, whose f16 hi + lo split must reconstruct every weight exactly."""
import ctypes as C
import dataclasses

import numpy as np
import pytest

from grande_b200 import _lib as L
from grande_b200 import synth
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def f16_bits(x):
    return O.f32_to_f16_bits(np.asarray(x, np.float32))


def edge_values(n, rng):
    """Normal draws plus the quantizers' corner cases: zeros, block maxima of
    either sign, tiny blocks whose products fall in the f16 subnormal range,
    and huge blocks whose products overflow f16."""
    v = (rng.standard_normal(n) * 0.02).astype(np.float32)
    v[:32] = 0.0
    v[32:64] = np.linspace(-1, 1, 32)
    v[64:96] *= 1e-4
    v[96:128] = np.linspace(-7e4, 7e4, 32)
    return v


@pytest.mark.parametrize("dtype", [O.Q4, O.Q8, O.F16])
def test_load_time_and_lm_head_decoders_are_exact(device, dtype):
    rng = np.random.default_rng(dtype)
    rows, k = 96, 256
    v = edge_values(rows * k, rng)
    data, scales = O.quantize(dtype, v)
    ref = O.dequantize(dtype, data, scales, rows * k)      # f32, QTensor::get
    codes = np.frombuffer(data, np.uint8).copy()
    sc = np.frombuffer(scales, np.uint8).copy() if scales else np.zeros(2, np.uint8)
    hi = np.empty(rows * k, np.uint16)
    lo = np.empty(rows * k, np.uint16)
    for mode in (0, 1):
        L.check(L.lib().omg_debug_dequant(device, dtype, L.ptr(codes, C.c_uint8),
                                          L.ptr(sc, C.c_uint8), rows, k, mode,
                                          L.ptr(hi, C.c_uint16), L.ptr(lo, C.c_uint16)))
        assert np.array_equal(hi, f16_bits(ref)), f"mode {mode}: hi != f16(QTensor::get)"
        if mode == 1:
            # hi + lo is the f32 weight exactly (finite weights).
            fin = np.isfinite(O.f16_bits_to_f32(hi))
            recon = O.f16_bits_to_f32(hi).astype(np.float64) + O.f16_bits_to_f32(lo)
            assert np.array_equal(recon[fin].astype(np.float32), ref[fin])


@pytest.mark.parametrize("packed", [False, True])
@pytest.mark.parametrize("config,layer", [("e2b-q4", 4), ("gemma3-270m-q8", 5)])
def test_engine_weights_are_f16_of_the_reference_dequant(device, config, layer, packed):
    # f16 rows: the load-time decoder's output; packed: the chunks decoded by
    # the GEMMs' own tile decoder.
    shape = dataclasses.replace(synth.CONFIGS[config], layers=layer + 1)
    eng = synth.build_engine(shape, 64, 4, device=device, packed=packed)
    try:
        d, ff = shape.d, shape.ff
        qkv = (shape.heads + 2 * shape.kv_heads) * 256
        for name, dims in ((f"blk.{layer}.qkv", [qkv, d]), (f"blk.{layer}.o", [d, shape.heads * 256]),
                           (f"blk.{layer}.gate", [ff, d]), (f"blk.{layer}.up", [ff, d]),
                           (f"blk.{layer}.down", [d, ff])):
            ref = O.synth_tensor(0, name, dims, int(shape.dtype))
            got = eng.weight_f16(name, dims)
            assert np.array_equal(got.ravel(), f16_bits(ref)), name
    finally:
        eng.close()
