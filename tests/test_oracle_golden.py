"""Pin the oracle before trusting it: its quantizers, visibility rule and
decoder forward against fixtures generated from the reference's own Python
code (tests/golden/make_golden.py), plus the reference's own known-answer
bounds (tests/reference.rs:600-610)."""
import json
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O

GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.mark.parametrize("name,dtype", [("q8", O.Q8), ("q4", O.Q4)])
def test_quantizers_match_gguf_and_exporter(name, dtype):
    g = np.load(GOLDEN / f"quant_{name}.npz")
    codes, scales = O.quantize(dtype, g["values"])
    assert codes == g["codes"].tobytes()
    assert scales == g["scales"].tobytes()


def test_quantization_roundtrips():
    """tests/reference.rs:600-610."""
    v = O.Rng(5).values(256, 0.3)
    d8 = np.max(np.abs(O.dequantize(O.Q8, *O.quantize(O.Q8, v), 256) - v))
    assert d8 < 0.3 / 127.0 * 1.01
    d4 = np.max(np.abs(O.dequantize(O.Q4, *O.quantize(O.Q4, v), 256) - v))
    assert d4 < 0.3 / 8.0 * 1.01


def test_dequant_layout():
    """model.rs:508-525: Q4 low nibbles are elements 0..16, high 16..32."""
    codes = bytes(range(16))  # byte j = j: lo nibble j, hi nibble 0
    scales = np.array([1.0], np.float16).tobytes()
    out = O.dequantize(O.Q4, codes, scales, 32)
    assert list(out[:16]) == [j - 8.0 for j in range(16)]
    assert list(out[16:]) == [-8.0] * 16
    q8 = np.arange(-16, 16, dtype=np.int8).tobytes()
    out = O.dequantize(O.Q8, q8, np.array([0.5], np.float16).tobytes(), 32)
    assert list(out) == [0.5 * x for x in range(-16, 16)]


def test_f16_conversion_edges():
    vals = np.array([0.0, -0.0, 1.0, 65504.0, 65520.0, 1e-8, 5.96e-8, 2.98e-8, 6.1e-5,
                     -3.14159, np.inf, -np.inf, 1.0 + 2**-11, 1.0 + 3 * 2**-11], np.float32)
    got = O.f32_to_f16_bits(vals)
    exp = vals.astype(np.float16).view(np.uint16)  # numpy: IEEE round-to-nearest-even
    assert list(got) == list(exp)
    allbits = np.arange(65536, dtype=np.uint16)
    f = O.f16_bits_to_f32(allbits)
    ref = allbits.view(np.float16).astype(np.float32)
    ok = (f == ref) | (np.isnan(f) & np.isnan(ref))
    assert ok.all()
    rng = np.random.default_rng(1)
    x = (rng.standard_normal(200000) * 10.0 ** rng.uniform(-8, 4, 200000)).astype(np.float32)
    assert (O.f32_to_f16_bits(x) == x.astype(np.float16).view(np.uint16)).all()


def _engine_packing(seg):
    """Positions as the engine assigns them (engine.rs:1519-1571): prefix
    0..P, each branch P.. again."""
    p = sum(1 for s in seg if s == 0)
    pos, seen = [], {}
    for i, s in enumerate(seg):
        if s == 0:
            pos.append(i)
        else:
            pos.append(p + seen.get(s, 0))
            seen[s] = seen.get(s, 0) + 1
    return pos


def test_visibility_matches_branch_mask():
    g = np.load(GOLDEN / "branch_mask.npz")
    for name in ("single", "two", "three", "noprefix"):
        seg = list(g[f"{name}_seg"])
        pos = _engine_packing(seg)
        windows = (0, 3, 6) if name == "single" else (0,)  # index == position only there
        for w in windows:
            exp = g[f"{name}_w{w}"]
            n = len(seg)
            got = np.array([[O.visible(pos[i], seg[i], pos[j], seg[j], w) for j in range(n)]
                            for i in range(n)])
            assert (got == exp).all(), (name, w)


def _gemma3_from_fixture(g):
    c = json.loads(str(g["config"]))
    layers = c["num_hidden_layers"]
    sliding = [t == "sliding_attention" for t in c["layer_types"]]
    hd = c["head_dim"]
    cfg = O.OracleConfig(
        vocab=c["vocab_size"], d=c["hidden_size"], layers=layers,
        heads=c["num_attention_heads"], kv_heads=c["num_key_value_heads"],
        head_dim=[hd] * layers, ff=[c["intermediate_size"]] * layers, sliding=sliding,
        kv_source=list(range(layers)), rope_dims=[hd] * layers, eps=c["rms_norm_eps"],
        window=c["sliding_window"],
        theta_global=c["rope_parameters"]["full_attention"]["rope_theta"],
        theta_local=c["rope_parameters"]["sliding_attention"]["rope_theta"],
        query_scale=c["query_pre_attn_scalar"] ** -0.5, norm_offset=1.0, v_norm=False)
    tensors = [O.f16_bits_to_f32(g[f"t:{name}"]) for name, _ in cfg.tensors()]
    return cfg, tensors


@pytest.mark.parametrize("name", ["sliding", "branches"])
def test_forward_matches_transformers_gemma3(name):
    g = np.load(GOLDEN / f"gemma3_{name}.npz")
    cfg, tensors = _gemma3_from_fixture(g)
    hid = O.forward(cfg, tensors, g["ids"], g["pos"], g["seg"], O.ORACLE_EXACT)
    exp = g["hidden"]
    scale = np.maximum(np.abs(exp).max(axis=1, keepdims=True), 1.0)
    err = np.abs(hid - exp) / scale
    assert err.max() < 1e-4, err.max()
