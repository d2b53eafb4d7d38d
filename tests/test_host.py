"""Host-side logic on the CPU: the C ABI loads and exports every symbol of
include/omg_b200.h, the engine's config parser and catalogue match the
reference's (via the oracle), the product quantizers are byte-identical to
the oracle's, and the GRWS1 state format / FNV key behave as
crates/omg-wgpu/src/engine.rs:503-641 specifies. No GPU calls."""
import re
import struct
from pathlib import Path

import numpy as np
import pytest

from grande_b200 import _lib as L
from grande_b200.engine import (Dtype, EngineBuilder, QTensor, SavedState, config_tensors,
                                state_key)
from oracle import oracle as O

from refmodels import gemma3, gemma4, gemma4_gqa

ROOT = Path(__file__).resolve().parent.parent
GOLDEN = Path(__file__).resolve().parent / "golden"


def header_functions():
    text = (ROOT / "include" / "omg_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(omg_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_header_symbol():
    lib = L.lib()
    names = header_functions()
    assert len(names) >= 30
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    # ...and the Python prototypes cover the whole header.
    assert set(names) <= set(L.PROTOTYPES), sorted(set(names) - set(L.PROTOTYPES))


def test_version_and_no_gpu_is_an_error():
    assert b"sm_100a" in L.lib().omg_version()


@pytest.mark.parametrize("make", [gemma3, gemma4, gemma4_gqa])
def test_config_from_json_matches_reference_configs(make):
    cfg, js = make()
    assert config_tensors(js) == [(n, list(s)) for n, s in cfg.tensors()]


def test_config_errors():
    with pytest.raises(L.OmgError, match="missing num_hidden_layers"):
        config_tensors('{"vocab_size": 4}')
    bad = '{"num_hidden_layers": 2, "layer_types": ["sliding_attention"], "head_dim": 256}'
    with pytest.raises(L.OmgError, match="layer_types has 1 entries for 2 layers"):
        config_tensors(bad)


def test_config_validate_errors():
    _, js = gemma3()
    import json
    c = json.loads(js)
    c["num_key_value_heads"] = 3
    buf = L.C.create_string_buffer(256)
    assert L.lib().omg_config_check(json.dumps(c).encode(), buf, 256) == -1
    assert "must divide" in L.lib().omg_last_error().decode()
    c = json.loads(js)
    c["head_dim"] = 128
    assert L.lib().omg_config_check(json.dumps(c).encode(), buf, 256) == -1
    assert "head_dim must be 256 or 512" in L.lib().omg_last_error().decode()


@pytest.mark.parametrize("dtype", [O.F16, O.Q8, O.Q4])
def test_product_quantizers_match_oracle(dtype):
    vals = [np.load(GOLDEN / "quant_q8.npz")["values"], O.Rng(3).values(32 * 999, 0.15),
            (np.random.default_rng(2).standard_normal(32 * 500) * 0.02).astype(np.float32)]
    for v in vals:
        q = QTensor._encode(Dtype(dtype), [v.size], v)
        data, scales = O.quantize(dtype, v)
        assert q.data == data and q.scales == scales
        assert np.array_equal(q.to_f32(), O.dequantize(dtype, data, scales, v.size))


@pytest.mark.parametrize("name", ["q8", "q4"])
def test_product_quantizers_match_golden(name):
    g = np.load(GOLDEN / f"quant_{name}.npz")
    q = QTensor._encode(Dtype.parse(name), [g["values"].size], g["values"])
    assert q.data == g["codes"].tobytes() and q.scales == g["scales"].tobytes()


def test_qtensor_from_raw_checks():
    with pytest.raises(L.OmgError, match="payload bytes"):
        QTensor.from_raw(Dtype.Q4, [2, 32], b"\0" * 31, b"\0" * 4)
    with pytest.raises(L.OmgError, match="scale bytes"):
        QTensor.from_raw(Dtype.Q8, [2, 32], b"\0" * 64, b"\0" * 2)


def grws(model_id: str, prefix, layers):
    out = b"GRWS1\0" + struct.pack("<I", len(model_id)) + model_id.encode()
    out += struct.pack("<I", len(prefix)) + b"".join(struct.pack("<I", t) for t in prefix)
    out += struct.pack("<I", len(layers))
    for l, r0, data in layers:
        out += struct.pack("<III", l, r0, len(data)) + data
    return out


def test_state_file_roundtrip_and_errors():
    img = grws("m:1", [2, 5, 9], [(0, 0, bytes(range(24))), (3, 1, b"\x01\x02" * 6)])
    s = SavedState.from_bytes(img, "m:1")
    assert s.prefix == [2, 5, 9]
    assert s.byte_len() == 3 * 4 + 24 + 12
    assert s.to_bytes("m:1") == img
    with pytest.raises(L.OmgError, match="different model"):
        SavedState.from_bytes(img, "m:2")
    with pytest.raises(L.OmgError, match="truncated"):
        SavedState.from_bytes(img[:-1], "m:1")
    with pytest.raises(L.OmgError, match="not a omg wgpu state file"):
        SavedState.from_bytes(b"XXXXX\0" + img[6:], "m:1")


def test_state_key_is_fnv1a():
    def fnv(model_id, prefix):
        h = 0xcbf29ce484222325
        for b in model_id.encode() + b"\0" + b"".join(struct.pack("<I", t) for t in prefix):
            h ^= b
            h = (h * 0x100000001b3) & 0xFFFFFFFFFFFFFFFF
        return h
    for mid, p in (("wgpu", [2, 3, 4]), ("e2b:123", list(range(100))), ("", [])):
        assert state_key(mid, p) == fnv(mid, p)


def test_builder_without_gpu_fails_loudly():
    if L.lib().omg_device_count() > 0:
        pytest.skip("a GPU is visible")
    _, js = gemma3()
    with pytest.raises(L.OmgError):
        EngineBuilder(js, 0)


def test_synth_normal_is_seeded_and_normal():
    import ctypes as C
    out = np.empty(200000, np.float32)
    L.check(L.lib().omg_synth_normal(0, b"blk.0.qkv", 0.0, 0.02, L.ptr(out, C.c_float), out.size))
    again = np.empty_like(out)
    L.check(L.lib().omg_synth_normal(0, b"blk.0.qkv", 0.0, 0.02, L.ptr(again, C.c_float),
                                     out.size))
    assert np.array_equal(out, again)
    assert abs(out.mean()) < 2e-4 and abs(out.std() - 0.02) < 2e-4
    other = np.empty_like(out)
    L.check(L.lib().omg_synth_normal(0, b"blk.1.qkv", 0.0, 0.02, L.ptr(other, C.c_float),
                                     out.size))
    assert not np.array_equal(out, other)


@pytest.mark.parametrize("name,shape,dtype,laya", [
    ("blk.3.gate", [64, 128], Dtype.Q4, False),
    ("blk.0.qkv", [96, 64], Dtype.Q8, False),
    ("blk.1.ffn_norm", [256], Dtype.F16, False),
    ("embed", [40, 64], Dtype.Q4, False),
    ("blk.2.wi_b", [192], Dtype.F16, True),
    ("scorer.l1", [64, 64], Dtype.Q8, True),
    ("blk.0.wo", [64, 96], Dtype.Q8, True),
])
def test_oracle_synthetic_models_match_the_product_generator(name, shape, dtype, laya):
    # The CPU baseline builds the benchmark's random models with oracle/ only;
    # they must be the product's models bit for bit (draws, codes, scales).
    from grande_b200 import synth
    n = int(np.prod(shape))
    for mean in (0.0, 1.0):
        a = synth.normal(5, name, n, mean, 0.02)
        b = O.synth_normal(5, name, n, mean, 0.02)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    qt = (synth.laya_tensor if laya else synth.tensor)(5, name, shape, dtype)
    got = O.synth_tensor(5, name, shape, int(dtype), laya=laya)
    assert np.array_equal(qt.to_f32().view(np.uint32), got.view(np.uint32))


def test_label_readout_matches_the_oracle_math():
    # readout.rs:130-147 on math.rs:5-17: the product's f64 softmax and
    # log-sum-exp against the oracle's C restatement.
    from grande_b200.readout import label_distribution, log_sum_exp, softmax
    rng = np.random.default_rng(4)
    row = (rng.standard_normal(25000) * 3).astype(np.float32)
    ids = [17, 4000, 24999]
    for temp in (1.0, 0.7, 0.0):
        dist = label_distribution(row, ids, temp)
        assert np.array_equal(dist.logits, row[ids])
        exp = O.softmax(row[ids], temp)
        assert np.allclose(dist.probs, exp, rtol=1e-12, atol=1e-15)
        assert np.allclose(softmax(row[ids], temp), exp, rtol=1e-12, atol=1e-15)
    lse = O.log_sum_exp(row)
    assert abs(log_sum_exp(row) - lse) < 1e-9
    mass = np.exp(O.log_sum_exp(row[ids]) - lse)
    assert abs(dist.candidate_mass - mass) < 1e-12
    with pytest.raises(ValueError):
        label_distribution(row, [25000])
