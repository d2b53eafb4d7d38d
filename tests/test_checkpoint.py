"""The model-directory loader on the host: safetensors parsing and the
Gemma 3 name mapping of Weights::load (crates/omg-wgpu/src/model.rs:556-740),
the exported-directory manifest (model.rs:742-795,
tools/export_wgpu_gguf.py:46-96) and the state cache's model id
(backend.rs:80-96), with the reference's error messages. The tensors are the
golden Gemma 3 fixture's and the reference test models'."""
import json
from pathlib import Path

import numpy as np
import pytest

from checkpoints import f32_to_bf16_bits, hf_name, write_export, write_safetensors
from grande_b200 import checkpoint as ck
from grande_b200._lib import OmgError
from grande_b200.engine import Dtype, QTensor
from oracle import oracle as O
from refmodels import RefModel, gemma3, gemma4

GOLDEN = Path(__file__).parent / "golden"


def fixture_tensors(name="sliding"):
    g = np.load(GOLDEN / f"gemma3_{name}.npz")
    return str(g["config"]), {k[2:]: g[k] for k in g.files if k.startswith("t:")}


def hf_tensors(config_json, bits: dict, prefix="model.", dtypes=("F32", "F16")):
    """The fixture as an HF checkpoint: q/k/v split back out of qkv, the
    tensors stored alternately in the given dtypes."""
    c = json.loads(config_json)
    q_rows = c["num_attention_heads"] * c["head_dim"]
    kv_rows = c["num_key_value_heads"] * c["head_dim"]
    out, k = {}, 0
    for name, b in bits.items():
        names = hf_name(name)
        parts = [b] if len(names) == 1 else [b[:q_rows], b[q_rows:q_rows + kv_rows],
                                             b[q_rows + kv_rows:]]
        for hn, p in zip(names, parts):
            dt = dtypes[k % len(dtypes)]
            k += 1
            if dt == "F16":
                raw = np.ascontiguousarray(p, dtype="<u2").tobytes()
            else:
                raw = O.f16_bits_to_f32(p).astype("<f4").tobytes()
            out[prefix + hn] = (dt, list(p.shape), raw)
    return out


@pytest.mark.parametrize("prefix", ["model.", ""])
def test_gemma3_safetensors_maps_every_tensor(tmp_path, prefix):
    cfg, bits = fixture_tensors()
    path = tmp_path / "model.safetensors"
    write_safetensors(path, hf_tensors(cfg, bits, prefix))
    w = ck.gemma3_weights(cfg, path.read_bytes())
    assert set(w) == set(bits)
    for name, b in bits.items():
        t = w[name]
        assert t.dtype == Dtype.F16 and t.scales == b""
        assert t.shape == list(b.shape), name
        assert t.data == np.ascontiguousarray(b, dtype="<u2").tobytes(), name
    # The same through the file mapping load_engine uses.
    view = ck._map(tmp_path, "model.safetensors")
    w2 = ck.gemma3_weights(cfg, view)
    ck._release(view)
    assert all(w2[n].data == w[n].data for n in w)


def test_safetensors_conversions_round_to_nearest_even(tmp_path):
    """F32 and BF16 become f16 by f16::from_f32 (round to nearest even,
    subnormals, overflow to infinity): the oracle's conversion."""
    r = np.random.default_rng(5)
    v = np.concatenate([
        r.normal(0, 1, 4000), r.normal(0, 1e-5, 1000), r.normal(0, 3e4, 500),
        [0.0, -0.0, 65504.0, 65519.0, 65520.0, 1e6, -1e6, 5.96e-8, 2.98e-8, 1 + 2 ** -11,
         1 + 3 * 2 ** -11, np.inf, -np.inf],
    ]).astype(np.float32)
    bf = f32_to_bf16_bits(v)
    bf_f32 = (bf.astype(np.uint32) << 16).view(np.float32)
    st = ck.SafeTensors.parse(_st(tmp_path, {
        "a": ("F32", [v.size], v.astype("<f4").tobytes()),
        "b": ("BF16", [v.size], bf.astype("<u2").tobytes()),
        "c": ("F16", [v.size], O.f32_to_f16_bits(v).astype("<u2").tobytes())}))
    shape, a = st.tensor("a")
    assert shape == [v.size]
    assert (a == O.f32_to_f16_bits(v)).all()
    _, b = st.tensor("b")
    assert (b == O.f32_to_f16_bits(bf_f32)).all()
    _, c = st.tensor("c")
    assert (c == O.f32_to_f16_bits(v)).all()


def _st(tmp_path, tensors) -> bytes:
    p = tmp_path / "t.safetensors"
    write_safetensors(p, tensors)
    return p.read_bytes()


def test_safetensors_errors(tmp_path):
    with pytest.raises(OmgError, match="^safetensors: too short$"):
        ck.SafeTensors.parse(b"1234")
    with pytest.raises(OmgError, match="^safetensors: header out of range$"):
        ck.SafeTensors.parse((100).to_bytes(8, "little") + b"{}")
    st = ck.SafeTensors.parse(_st(tmp_path, {
        "ok": ("F16", [2], b"\0\0\0\0"),
        "int": ("I8", [4], b"\0\0\0\0"),
        "short": ("F16", [3], b"\0\0\0\0"),
    }))
    with pytest.raises(OmgError, match="^safetensors: missing nope$"):
        st.tensor("nope")
    with pytest.raises(OmgError, match="^int: unsupported dtype I8$"):
        st.tensor("int")
    with pytest.raises(OmgError, match=r"^short: 2 values for shape \[3\]$"):
        st.tensor("short")
    raw = bytearray(_st(tmp_path, {"x": ("F16", [2], b"\0\0\0\0")}))
    h = json.loads(raw[8:8 + int.from_bytes(raw[:8], "little")])
    h["x"]["data_offsets"] = [0, 64]
    hb = json.dumps(h).encode()
    st = ck.SafeTensors.parse(len(hb).to_bytes(8, "little") + hb + b"\0\0\0\0")
    with pytest.raises(OmgError, match="^x: offsets out of range$"):
        st.tensor("x")


def test_gemma3_loader_errors(tmp_path):
    cfg, bits = fixture_tensors()
    hf = hf_tensors(cfg, bits)
    _, g4 = gemma4()
    with pytest.raises(OmgError, match="^safetensors loading is for Gemma 3 checkpoints; "
                                       "export Gemma 4 with tools/export_wgpu_gguf.py$"):
        ck.gemma3_weights(g4, _st(tmp_path, hf))
    # The embedding's shape against the config.
    bad = dict(hf)
    dt, shape, raw = bad["model.embed_tokens.weight"]
    bad["model.embed_tokens.weight"] = (dt, [shape[0] // 2, shape[1] * 2], raw)
    with pytest.raises(OmgError, match=r"^embed_tokens is \[20, 128\], config says \[40, 64\]$"):
        ck.gemma3_weights(cfg, _st(tmp_path, bad))
    # A missing tensor, named with the checkpoint's prefix.
    bad = {k: v for k, v in hf.items() if k != "model.layers.1.mlp.up_proj.weight"}
    with pytest.raises(OmgError, match=r"^safetensors: missing model\.layers\.1\.mlp\.up_proj"):
        ck.gemma3_weights(cfg, _st(tmp_path, bad))
    # Weights::check: a tensor of the wrong shape.
    bad = dict(hf)
    dt, shape, raw = bad["model.layers.0.self_attn.q_norm.weight"]
    bad["model.layers.0.self_attn.q_norm.weight"] = (dt, [shape[0] // 2, 2], raw)
    with pytest.raises(OmgError, match=r"^blk\.0\.q_norm: shape \[128, 2\], expected \[256\]$"):
        ck.gemma3_weights(cfg, _st(tmp_path, bad))
    # A multimodal config nesting the text model still loads.
    nested = json.dumps({"model_type": "gemma3", "text_config": json.loads(cfg)})
    assert set(ck.gemma3_weights(nested, _st(tmp_path, hf))) == set(bits)


def test_manifest_round_trip_quantized(tmp_path):
    """Every entry of an exported Gemma 4 directory (Q4_0 linears, Q8_0
    embedding, f16 norms, the per-layer table) decodes to the tensor that
    was written, codes and scales byte for byte."""
    m = RefModel(*gemma4(), 11, O.Q4, O.Q8)
    manifest = write_export(tmp_path, m.config_json, m.qtensors, m.per_layer_table)
    assert {f["path"] for f in manifest["files"]} == {"embed.bin"} | {
        f"blk.{i}.bin" for i in range(4)}
    parsed = ck.Manifest.parse((tmp_path / "manifest.json").read_bytes())
    seen = set()
    for f in parsed.files:
        data = (tmp_path / f.path).read_bytes()
        for e in f.tensors:
            assert e.offset % 4 == 0 and e.scales_offset % 4 == 0
            t = e.tensor(data)
            want = m.qtensors[e.name]
            assert (t.dtype, t.shape, t.data, t.scales) == (want.dtype, want.shape, want.data,
                                                           want.scales), e.name
            seen.add(e.name)
    assert seen == set(m.qtensors)
    e = parsed.per_layer_table
    assert e.path == "per_layer_table.bin"
    t = e.tensor((tmp_path / e.path).read_bytes())
    assert (t.data, t.scales, t.shape) == (m.per_layer_table.data, m.per_layer_table.scales,
                                           m.per_layer_table.shape)
    ck.check_weights(m.config_json, {e.name: e for f in parsed.files for e in f.tensors}, t)


def test_manifest_errors(tmp_path):
    m = RefModel(*gemma3(), 3, O.F16, O.F16)
    write_export(tmp_path, m.config_json, m.qtensors)
    parsed = ck.Manifest.parse((tmp_path / "manifest.json").read_bytes())
    e = parsed.files[0].tensors[0]
    short = (tmp_path / parsed.files[0].path).read_bytes()[:e.offset + e.nbytes - 1]
    with pytest.raises(OmgError, match=rf"^{e.name}: byte range {e.offset}\.\.{e.offset + e.nbytes} "
                                       "outside the file$"):
        e.tensor(short)
    bad = ck.ManifestEntry(**{**e.__dict__, "dtype": "q5"})
    with pytest.raises(OmgError, match="^unsupported dtype q5$"):
        bad.tensor((tmp_path / parsed.files[0].path).read_bytes())
    with pytest.raises(OmgError, match="manifest.json: missing field `files`"):
        ck.Manifest.parse(b"{}")
    with pytest.raises(OmgError, match="manifest.json: missing field `nbytes`"):
        ck.Manifest.parse(json.dumps({"files": [{"path": "a.bin", "tensors": [
            {"name": "x", "dtype": "f16", "shape": [2], "offset": 0}]}]}))
    with pytest.raises(OmgError, match="^missing tensor blk.2.o$"):
        ck.check_weights(m.config_json, {k: v for k, v in m.qtensors.items() if k != "blk.2.o"},
                         None)
    _, g4 = gemma4()
    m4 = RefModel(*gemma4(), 3, O.Q8, O.Q8)
    with pytest.raises(OmgError, match="^missing per-layer token table$"):
        ck.check_weights(g4, m4.qtensors, None)
    with pytest.raises(OmgError, match=r"^per-layer table: shape \[64, 64\], expected \[64, 128\]$"):
        ck.check_weights(g4, m4.qtensors, QTensor(Dtype.F16, [64, 64], b"", b""))


def test_model_id_counts_bin_files(tmp_path):
    d = tmp_path / "gemma-3-270m-wgpu"
    d.mkdir()
    (d / "embed.bin").write_bytes(b"x" * 10)
    (d / "blk.0.bin").write_bytes(b"x" * 5)
    (d / "config.json").write_bytes(b"x" * 100)
    (d / ".bin").write_bytes(b"x" * 7)
    assert ck.model_id(d) == "gemma-3-270m-wgpu:15"
    assert ck.model_id(tmp_path / "absent") == "absent:0"


def test_load_engine_reports_missing_files(tmp_path):
    with pytest.raises(OmgError, match=r"^reading .*config\.json"):
        ck.load_engine(tmp_path, 64, 16)
    cfg, _ = fixture_tensors()
    (tmp_path / "config.json").write_text(cfg)
    with pytest.raises(OmgError, match=r"^reading .*model\.safetensors"):
        ck.load_engine(tmp_path, 64, 16)
